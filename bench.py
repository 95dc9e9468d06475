"""Benchmark of invokerl's log-prob + GRPO-loss hot path (forward and backward) on 1..8 B200s.

Default workload, the headline: the Qwen3-8B LM-head configuration.

* hidden bf16 [B*T, 4096] ~ N(0,1) and untied W_lm bf16 [151936, 4096] ~ N(0, 0.02);
* B = 128 (16 prompts x group 8), T = 4096, completion length U[512, 3584];
* one step = the fused LM-head log-prob forward over all B*T rows, GRPO group advantages, the
  GRPO clipped-ratio + k3-KL loss with the token-count all-reduce, and the backward through the
  loss and the LM head (dHidden and dW).

Rows are sharded over ranks by whole prompt groups. The global batch stays B = 128, so
scaling is strong. Inputs are synthetic and seeded.

Other workloads (`--workload`), one JSON line each:

* lmhead-0.6b: the Qwen3-0.6B head (H=1024, tied, B=64, T=2048) with the same step.
* logits: the unfused logits -> log-prob forward + backward, bf16 [16384, 151936].
* grpo / grpo-hbm: GRPO advantages + loss + backward on a [16, 512] batch, or on its HBM-sized
  variant [1024, 8192].

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--workload W]

`--impl reference` times the reference algorithm on the host CPU cores, on a bounded sample of
the same workload. The reference is torch on the CPU, restated in oracle/.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# Keep stdout to the one JSON line: NCCL prints its version banner to stdout at the VERSION and
# WARN debug levels, so those (and an unset level) become NONE; INFO / TRACE are left for
# debugging.  Set before torch loads NCCL.
if os.environ.get("NCCL_DEBUG", "VERSION").upper() in ("VERSION", "WARN"):
    os.environ["NCCL_DEBUG"] = "NONE"

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "log-prob+GRPO loss tokens/s fwd+bwd"
UNIT = "tokens/s"
V = 151936
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


# ---- clocks sampler -------------------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


class EventTimer:
    """CUDA events around every call of the wrapped functions while active (the launching stream
    is the current stream; every op here launches on it)."""

    def __init__(self):
        self.pairs: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
        self.names: list[str] = []
        self.active = False

    def wrap(self, fn):
        def inner(*a, **k):
            if not self.active:
                return fn(*a, **k)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*a, **k)
            e.record()
            self.pairs.append((s, e))
            self.names.append(fn.__name__)
            return out

        return inner

    def total_ms(self) -> float:
        return sum(s.elapsed_time(e) for s, e in self.pairs)

    def by_name_ms(self) -> dict:
        out: dict = {}
        for n, (s, e) in zip(self.names, self.pairs):
            out[n] = out.get(n, 0.0) + s.elapsed_time(e)
        return out


def to_device_batch(b, device):
    from invokerl_b200.algorithms import RolloutBatch

    return RolloutBatch(**{k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v)
                           for k, v in vars(b).items() if k != "extras"}, extras={})


def host_batch(b):
    """Pinned host copy of a RolloutBatch's tensors."""
    from invokerl_b200.algorithms import RolloutBatch

    return RolloutBatch(**{k: (v.pin_memory() if isinstance(v, torch.Tensor) else v)
                           for k, v in vars(b).items() if k != "extras"}, extras={})


def batch_bytes(b) -> int:
    return sum(v.numel() * v.element_size() for v in vars(b).values() if isinstance(v, torch.Tensor))


class Prefetch:
    """Host-to-device input copies of end-to-end steps, issued one step ahead on a copy stream
    into two sets of device buffers, as a pinned-memory data loader does.  Every step's copies
    lie inside the timed region: step 0's are issued after the start event, each step's compute
    waits for its own copies, and step i+1's are issued before step i computes."""

    serial = False  # --e2e-serial: copy each step's inputs in line with the step instead

    def __init__(self, host: dict, device):
        self.host, self.device = host, device
        self.bufs = [{k: torch.empty(v.shape, dtype=v.dtype, device=device) for k, v in host.items()}
                     for _ in range(2)]
        self.stream = torch.cuda.Stream(device)
        self.done = [torch.cuda.Event(), torch.cuda.Event()]

    def _issue(self, i):
        s = self.stream if not Prefetch.serial else torch.cuda.current_stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))  # after the start event / the buffer's last user
        with torch.cuda.stream(s):
            for k, v in self.host.items():
                self.bufs[i % 2][k].copy_(v, non_blocking=True)
            self.done[i % 2].record(s)

    def get(self, i: int, n: int) -> dict:
        """Device inputs of step i of n (steps run in order; the host has finished step i-1)."""
        if i == 0 or Prefetch.serial:
            self._issue(i)
        torch.cuda.current_stream(self.device).wait_event(self.done[i % 2])
        if i + 1 < n and not Prefetch.serial:
            self._issue(i + 1)
        return self.bufs[i % 2]


def batch_from(hb, d: dict):
    """RolloutBatch with the tensor fields of host batch `hb` taken from the device buffers `d`."""
    from invokerl_b200.algorithms import RolloutBatch

    return RolloutBatch(**{k: d.get(k, v) for k, v in vars(hb).items() if k != "extras"}, extras={})


_REF_PKG: list = []


def ops_stats() -> dict:
    """Rows the logit cache held in the last forward that needed a gradient, and its candidates."""
    from invokerl_b200 import ops

    return ops.LOGIT_CACHE_STATS


def reference_package():
    """The unmodified reference package (invokerl, pure Python) from baseline/_ref, imported once;
    None when it is not there."""
    if not _REF_PKG:
        ref_root = ROOT / "baseline" / "_ref"
        mod = None
        if (ref_root / "invokerl" / "policy.py").exists():
            if str(ref_root) not in sys.path:
                sys.path.insert(0, str(ref_root))
            import invokerl.algorithms
            import invokerl.policy

            mod = invokerl
        _REF_PKG.append(mod)
    return _REF_PKG[0]


def time_cpu(fn, steps: int) -> float:
    """Seconds per call of fn on the host (one untimed call first)."""
    fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    return (time.perf_counter() - t0) / max(1, steps)


# ---- workloads -------------------------------------------------------------------------------------


class LMHeadGRPO:
    """Fused LM-head log-prob + GRPO loss, forward and backward (configs 3 and 4)."""

    PRESETS = {
        "lmhead-8b": dict(H=4096, B=128, T=4096, prompt=(64, 512), completion=(512, 3584),
                          name="Qwen3-8B LM head: hidden bf16 [128*4096, 4096], W bf16 [151936, 4096] untied"),
        "lmhead-0.6b": dict(H=1024, B=64, T=2048, prompt=(64, 256), completion=(32, 256),
                            name="Qwen3-0.6B LM head: hidden bf16 [64*2048, 1024], W bf16 [151936, 1024] tied"),
    }
    G = 8

    def __init__(self, key, args):
        p = dict(self.PRESETS[key])
        if args.batch:
            if args.batch % self.G:
                raise SystemExit(f"--batch must be a multiple of the group size {self.G}")
            p["B"] = args.batch
        self.key, self.p = key, p
        self.H, self.B, self.T = p["H"], p["B"], p["T"]

    def setup(self, rank, world, device):
        from invokerl_b200 import ops
        from invokerl_b200.algorithms import GRPO
        from invokerl_b200.distributed import shard_batch
        from invokerl_b200.synthetic import rollout_batch

        H, B, T, G = self.H, self.B, self.T, self.G
        batch = rollout_batch(B // G, G, T, prompt_len=self.p["prompt"], completion_len=self.p["completion"],
                              vocab=V, seed=0)
        # Ranks take whole groups balanced by work (rows for the forward, response tokens for the
        # backward), not by count.
        local = shard_batch(batch, rank, world, balance=world > 1)
        local.extras = {}
        Bl = local.token_ids.shape[0]
        gids = [int(local.group_ids[j * G]) for j in range(Bl // G)]
        # Hidden rows and W are generated on the device per prompt group, so the global data is
        # the same for any number of ranks.
        hidden = torch.empty(Bl * T, H, dtype=torch.bfloat16, device=device)
        for j, gid in enumerate(gids):
            gen = torch.Generator(device=device).manual_seed(1000 + gid)
            hidden[j * G * T:(j + 1) * G * T] = torch.randn(G * T, H, device=device, generator=gen).to(torch.bfloat16)
        gw = torch.Generator(device=device).manual_seed(7)
        weight = (0.02 * torch.randn(V, H, device=device, generator=gw)).to(torch.bfloat16)
        ids = local.token_ids.reshape(-1).to(device)
        # Rollout-time log-probs of the same policy: old = lp + N(0, 0.05), ref = lp + N(0, 0.1), so
        # ratios and KL terms have realistic sizes for this random-init head.
        lp, _ = ops.lmhead_forward_raw(hidden, weight, ids)
        lp = lp.view(Bl, T)
        old = torch.empty_like(lp)
        ref = torch.empty_like(lp)
        for j, gid in enumerate(gids):
            gr = torch.Generator(device=device).manual_seed(11 + gid)
            rows = slice(j * G, (j + 1) * G)
            old[rows] = lp[rows] + 0.05 * torch.randn(G, T, device=device, generator=gr)
            ref[rows] = lp[rows] + 0.1 * torch.randn(G, T, device=device, generator=gr)
        local.old_log_probs, local.ref_log_probs = old.cpu(), ref.cpu()
        del lp, old, ref
        self.local, self.Bl = local, Bl
        self.dev_batch = to_device_batch(local, device)
        self.hidden = hidden.requires_grad_(True)
        self.weight = weight.requires_grad_(True)
        self.ids = ids
        self.algo = GRPO(clip_eps=0.2, beta=0.04, row_sharded=world > 1)
        self.device = device

    def timed_functions(self):
        return ["lmhead_forward_raw", "lmhead_backward_raw"]

    def _step(self, batch, hidden, ids):
        from invokerl_b200 import ops

        # The attended rows may carry a gradient (the loss weights the response tokens among them),
        # as PolicyModel.forward passes them.
        lp = ops.lmhead_logprob(hidden, self.weight, ids, cache_rows=batch.attention_mask.reshape(-1))
        lp = lp.view(self.Bl, self.T)
        adv = self.algo.compute_advantages(batch)
        loss, metrics = self.algo.compute_loss(lp, batch, adv)
        loss.backward()
        return float(loss.detach()), metrics

    def step(self):
        self.hidden.grad = None
        self.weight.grad = None
        return self._step(self.dev_batch, self.hidden, self.ids)

    def tokens_per_step(self):
        return self.B * self.T

    def roofline(self, kernel_ms_per_step, peaks, peak_src):
        n = self.Bl * self.T
        n_act = int(self.dev_batch.response_mask.sum())  # rows with a nonzero upstream gradient
        flops = (2.0 * n + 4.0 * n_act) * self.H * V
        achieved = flops / (kernel_ms_per_step / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        return {
            "kernel": "fused LM-head log-prob fwd+bwd: tcgen05 GEMMs with online-LSE / dlogits epilogues",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "frac_of_burst_peak": achieved / peaks["bf16_tflops"],
            "peak_source": f"{peak_src} bf16 sustained (kernel timed inside a multi-second step)",
            "algorithmic": "2*N*H*V (fwd over all N rows) + 4*N_act*H*V (dH and dW over the N_act rows whose "
                           "upstream gradient is nonzero; masked rows contribute exact zeros and are skipped); "
                           "the backward's logits recompute of active rows without a logit-cache slot is executed "
                           "but not counted",
            "rows": n, "active_rows": n_act,
            "logit_cache": dict(ops_stats()),
            "executed_tflop_per_step": (2.0 * n + 4.0 * n_act + 2.0 * max(0, n_act - ops_stats()["rows"]))
                                       * self.H * V / 1e12,
            "traffic": self._traffic(n, n_act),
            "traffic_unit": "bytes per step (all K1 launches of one step)",
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the K1 launches of a 65,536-row "
                              "step, scaled by rows (forward) and active rows (backward chunks)",
        }

    def _traffic(self, n, n_act):
        cached = ops_stats()["rows"] > 0
        f = TRAFFIC["lmhead_fwd_per_row_cached" if cached else "lmhead_fwd_per_row"].get(self.H)
        b = TRAFFIC["lmhead_bwd_per_active_row_cached" if cached else "lmhead_bwd_per_active_row"].get(self.H)
        return None if f is None or b is None else f * n + b * n_act

    def config(self, world):
        return {
            "workload": self.p["name"] + f", GRPO G={self.G} k3 KL, fwd+bwd (dHidden, dW), row-sharded by group",
            "global_batch": self.B,
            "seq_len": self.T,
            "hidden": self.H,
            "vocab": V,
            "group_size": self.G,
            "parallelism": f"dp{world} (whole groups per rank, balanced by rows + response tokens; "
                           "scalar NCCL all-reduces)",
            "l2": f"inputs larger than L2 (hidden {self.B * self.T * self.H * 2 / 1e9:.1f} GB per step), no flush",
        }

    def e2e(self):
        """The same step through the public API with inputs in pinned host memory: every step copies
        the rank's hidden rows, token ids, log-probs, masks and rewards to the device and reads the
        loss and metrics back."""
        host_hidden = self.hidden.detach().cpu().pin_memory()
        hb = host_batch(self.local)
        h2d = host_hidden.numel() * 2 + batch_bytes(hb)
        d2h = 4 + 4 * 12
        pf = Prefetch({"hidden": host_hidden, **{k: v for k, v in vars(hb).items() if isinstance(v, torch.Tensor)}},
                      self.device)

        def one(i=0, n=1):
            d = pf.get(i, n)
            hid = d["hidden"].detach().requires_grad_(True)
            b = batch_from(hb, d)
            self.weight.grad = None
            return self._step(b, hid, b.token_ids.reshape(-1))

        one.pipelined = True
        return one, h2d, d2h

    def cpu_sample(self, rows, steps):
        """The reference's own CPU path on a bounded sample: invokerl's PolicyModel._chunked_lm_head_ce
        (policy.py:124-191; bf16 F.linear + -F.cross_entropy) and its GRPO compute_advantages /
        compute_loss (grpo.py:46-143) + autograd, on G sequences of rows/G tokens.  Without the
        reference package, the oracle's fp32 restatement of the same arithmetic."""
        ref = reference_package()
        if ref is None:
            return self._cpu_sample_port(rows, steps)
        from invokerl.algorithms import GRPO as RefGRPO
        from invokerl.algorithms import RolloutBatch as RefBatch
        from invokerl.policy import PolicyModel as RefPolicy

        from invokerl_b200.synthetic import lmhead_inputs

        torch.set_num_threads(os.cpu_count() or 1)
        G = self.G
        Ts = max(1, rows // G)
        rows = G * Ts
        li = lmhead_inputs(rows, self.H, V, seed=3)
        head = torch.nn.Linear(self.H, V, bias=False, dtype=torch.bfloat16)
        with torch.no_grad():
            head.weight.copy_(li.weight)
        pm = RefPolicy.__new__(RefPolicy)
        pm.model = torch.nn.Module()
        pm.model.lm_head = head
        hidden = li.hidden.view(G, Ts, self.H).clone().requires_grad_(True)
        targets = li.targets.view(G, Ts)
        g = torch.Generator().manual_seed(5)
        rm = torch.rand(G, Ts, generator=g) < 0.6
        rm[:, 0] = True
        old = -torch.empty(G, Ts).exponential_(1.0, generator=g)
        rb = RefBatch(token_ids=targets, prompt_mask=~rm, response_mask=rm, attention_mask=torch.ones_like(rm),
                      rewards=torch.bernoulli(torch.full((G,), 0.5), generator=g), token_rewards=None,
                      old_log_probs=old, ref_log_probs=old + 0.1 * torch.randn(G, Ts, generator=g),
                      group_ids=torch.zeros(G, dtype=torch.long), group_size=G)
        algo = RefGRPO(clip_eps=0.2, beta=0.04)

        def one():
            hidden.grad = None
            head.weight.grad = None
            lp = pm._chunked_lm_head_ce(hidden, targets, 64)
            adv = algo.compute_advantages(rb)
            loss, _ = algo.compute_loss(lp, rb, adv)
            loss.backward()

        dt = time_cpu(one, steps)
        return rows / dt, dt, (f"{G} sequences x {Ts} tokens = {rows} rows x H={self.H} x V={V} per step: invokerl's "
                               "own _chunked_lm_head_ce (bf16) + GRPO + autograd on the host CPU"), "reference"

    def _cpu_sample_port(self, rows, steps):
        """The oracle's fp32 restatement of the same step (reference package absent)."""
        import oracle
        from invokerl_b200.synthetic import lmhead_inputs

        torch.set_num_threads(os.cpu_count() or 1)
        li = lmhead_inputs(rows, self.H, V, seed=3)
        hh = li.hidden.float().requires_grad_(True)
        ww = li.weight.float().requires_grad_(True)
        g = torch.Generator().manual_seed(5)
        old = -torch.empty(rows).exponential_(1.0, generator=g)
        ref = old + 0.1 * torch.randn(rows, generator=g)
        mask = torch.rand(rows, generator=g) < 0.6
        rewards = torch.bernoulli(torch.full((self.G,), 0.5), generator=g)
        adv = oracle.group_advantages(rewards, torch.ones(self.G, 1, dtype=torch.bool), self.G).reshape(-1)
        adv = adv.repeat_interleave((rows + self.G - 1) // self.G)[:rows]

        def one():
            hh.grad = None
            ww.grad = None
            lp = oracle.lmhead_logprob(hh, ww, li.targets)
            ratio = torch.exp(lp - old)
            pl = -torch.minimum(ratio * adv, torch.clamp(ratio, 0.8, 1.2) * adv)
            d = ref - lp
            loss = ((pl + 0.04 * (torch.exp(d) - d - 1)) * mask).sum() / mask.sum().clamp(min=1)
            loss.backward()

        dt = time_cpu(one, steps)
        return rows / dt, dt, f"{rows} rows x H={self.H} x V={V} per step (the oracle, fp32 torch on the host CPU)", "port"


class LogitsLogProb:
    """Unfused logits -> log-prob forward + backward (config 2): bf16 [16384, 151936] ~ N(0, 2),
    uniform targets, upstream N(0,1) times a 50% mask."""

    def __init__(self, key, args):
        self.N = args.rows or 16384

    def setup(self, rank, world, device):
        gen = torch.Generator(device=device).manual_seed(0)
        self.logits = (2.0 * torch.randn(self.N, V, device=device, generator=gen)).to(torch.bfloat16)
        self.t = torch.randint(0, V, (self.N,), device=device, generator=gen)
        self.up = torch.randn(self.N, device=device, generator=gen) * (
            torch.rand(self.N, device=device, generator=gen) < 0.5).float()
        self.n_act = int((self.up != 0).sum())
        self.x = self.logits.requires_grad_(True)
        self.device = device

    def timed_functions(self):
        return []  # the step is the two kernels; the whole step is timed

    def step(self):
        from invokerl_b200 import ops

        self.x.grad = None
        lp = ops.logits_logprob(self.x, self.t)
        lp.backward(self.up)
        return 0.0, {}

    def tokens_per_step(self):
        return self.N

    def roofline(self, kernel_ms_per_step, peaks, peak_src):
        nbytes = 2.0 * self.N * V + 2.0 * self.N * V + 2.0 * self.n_act * V
        achieved = nbytes / (kernel_ms_per_step / 1e3) / 1e9
        return {"kernel": "logits log-prob fwd + bwd (one CTA per row, 16-byte streaming loads)", "bound": "hbm",
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "peak_source": f"{peak_src} HBM copy",
                "algorithmic": "fwd reads 2NV bytes; bwd writes 2NV and reads 2*N_active*V (rows with a zero "
                               "upstream are written as zeros without reading)",
                "traffic": TRAFFIC["logits_per_row"] * self.N, "traffic_unit": "bytes per step",
                "traffic_source": "ncu dram bytes of the fwd + bwd kernels on [4096, 151936], scaled by rows"}

    def config(self, world):
        return {"workload": "unfused logits->log-prob fwd+bwd: logits bf16 [16384, 151936] N(0,2), 50% masked upstream",
                "rows": self.N, "vocab": V, "l2": "5 GB of logits per step, larger than L2, no flush"}

    def e2e(self):
        host_logits = self.logits.detach().cpu().pin_memory()
        host_t, host_up = self.t.cpu().pin_memory(), self.up.cpu().pin_memory()
        h2d = host_logits.numel() * 2 + host_t.numel() * 8 + host_up.numel() * 4
        d2h = 4

        def one():
            from invokerl_b200 import ops

            x = host_logits.to(self.device, non_blocking=True).requires_grad_(True)
            lp = ops.logits_logprob(x, host_t.to(self.device, non_blocking=True))
            lp.backward(host_up.to(self.device, non_blocking=True))
            return float(lp.detach().sum()), {}

        return one, h2d, d2h

    def cpu_sample(self, rows, steps):
        """The reference's FSDP-branch log-prob (policy.py:100-104): -F.cross_entropy on bf16 logits
        [rows, V], reduction="none", and its autograd, on the host CPU."""
        from invokerl_b200.synthetic import logits_inputs

        torch.set_num_threads(os.cpu_count() or 1)
        logits, t, up = logits_inputs(rows, V, seed=1)
        x = logits.requires_grad_(True)

        def one():
            x.grad = None
            lp = -torch.nn.functional.cross_entropy(x, t, reduction="none")
            lp.backward(up.to(lp.dtype))

        dt = time_cpu(one, steps)
        return rows / dt, dt, (f"{rows} rows x V={V} bf16 per step: invokerl's FSDP-branch -F.cross_entropy "
                               "(policy.py:100-104) + autograd on the host CPU"), "reference"


class GRPOHooks:
    """GRPO compute_advantages + compute_loss + backward on a synthetic RolloutBatch (config 1 and its
    HBM-sized variant)."""

    PRESETS = {"grpo": (4, 4, 512, (64, 256), (32, 256)), "grpo-hbm": (128, 8, 8192, (64, 256), (512, 4096))}

    def __init__(self, key, args):
        self.key = key
        self.P, self.G, self.T, self.pl, self.cl = self.PRESETS[key]

    def setup(self, rank, world, device):
        from invokerl_b200.algorithms import GRPO
        from invokerl_b200.distributed import shard_batch
        from invokerl_b200.synthetic import rollout_batch

        b = rollout_batch(self.P, self.G, self.T, prompt_len=self.pl, completion_len=self.cl, seed=0)
        self.local = shard_batch(b, rank, world)
        self.new = self.local.extras["new_log_probs"].contiguous()
        self.dev_batch = to_device_batch(self.local, device)
        self.lp = self.new.to(device).requires_grad_(True)
        self.algo = GRPO(clip_eps=0.2, beta=0.04, row_sharded=world > 1)
        self.device = device

    def timed_functions(self):
        return []

    def kernel_ms(self, reps: int = 20) -> dict:
        """Device time of the fused loss kernel and of the advantage kernel, each launched `reps`
        times back to back between two CUDA events (the step itself is bound by host launches)."""
        from invokerl_b200 import _native as N
        from invokerl_b200 import ops

        b = self.dev_batch
        adv = self.algo.compute_advantages(b)
        params = self.algo._params()
        m = N.as_mask(b.response_mask)
        ntok = ops.mask_count(m)
        lp = self.lp.detach()
        Bn, T = lp.shape
        dlp = torch.empty_like(lp)
        sums = torch.empty(N.LOSS_NSUMS, dtype=torch.float64, device=lp.device)
        nbytes = int(N.lib().ikrl_clip_loss_workspace_bytes(Bn * T))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=lp.device)
        st = N.stream_of(lp.device)

        def loss_once():
            N.call("ikrl_clip_loss_fwd", N.ptr(lp), N.i32(N.IKRL_DTYPE_F32), N.ptr(b.old_log_probs),
                   N.ptr(b.ref_log_probs), N.ptr(adv), N.ptr(m), N.ptr(b.rewards), N.i32(Bn), N.i32(T),
                   N.i32(self.G), N.ptr(ntok), None, None, None, params, N.ptr(dlp), None, N.ptr(sums),
                   N.ptr(ws), N.sz(nbytes), st)

        out = torch.empty_like(adv)
        r = b.rewards.contiguous().float()

        def adv_once():
            N.call("ikrl_group_advantages", N.ptr(r), N.ptr(m), None, N.i32(Bn), N.i32(T), N.i32(self.G), N.i32(0),
                   N.f32(0.0), N.ptr(out), None, st)

        res = {}
        for name, fn in (("loss", loss_once), ("advantages", adv_once)):
            for _ in range(3):
                fn()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s.record()
            for _ in range(reps):
                fn()
            e.record()
            torch.cuda.synchronize()
            res[name] = s.elapsed_time(e) / reps
        return res

    def _step(self, batch, lp):
        adv = self.algo.compute_advantages(batch)
        loss, metrics = self.algo.compute_loss(lp, batch, adv)
        loss.backward()
        return float(loss.detach()), metrics

    def step(self):
        self.lp.grad = None
        return self._step(self.dev_batch, self.lp)

    def tokens_per_step(self):
        return self.P * self.G * self.T

    def roofline(self, kernel_ms_per_step, peaks, peak_src):
        km = self.kernel_ms()
        n = self.lp.numel()
        achieved = 21.0 * n / (km["loss"] / 1e3) / 1e9
        adv_gbs = 5.0 * n / (km["advantages"] / 1e3) / 1e9
        return {"kernel": "fused ratio+clip+KL+masked-sum loss with d loss/d lp (one pass)", "bound": "hbm",
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "peak_source": f"{peak_src} HBM copy",
                "algorithmic": "21 B/token: reads new, old, ref, adv (fp32) + mask (1 B), writes dlp (fp32)",
                "kernel_ms": km["loss"], "timing": "20 back-to-back launches between CUDA events",
                "advantages_kernel": {"ms": km["advantages"], "achieved_gbs": adv_gbs,
                                      "frac": adv_gbs / peaks["hbm_gbs"],
                                      "algorithmic": "5 B/token: reads mask (1 B), writes adv (fp32)"},
                "traffic": TRAFFIC["grpo_loss_per_token"] * n, "traffic_unit": "bytes per loss-kernel launch",
                "traffic_source": "ncu dram bytes of the loss kernel on 8,388,608 tokens, scaled by tokens"}

    def config(self, world):
        B = self.P * self.G
        return {"workload": f"GRPO compute_advantages+compute_loss+backward, fp32 RolloutBatch B={B} "
                            f"({self.P} prompts x group {self.G}), T={self.T}",
                "global_batch": B, "seq_len": self.T, "group_size": self.G,
                "l2": ("inputs smaller than L2 (launch-bound); timed back to back" if self.key == "grpo"
                       else "inputs larger than L2 (176 MB per step), no flush")}

    def e2e(self):
        hb = host_batch(self.local)
        host_lp = self.new.pin_memory()
        h2d = batch_bytes(hb) + host_lp.numel() * 4
        d2h = 4 + 4 * 12

        def one():
            b = to_device_batch(hb, self.device)
            lp = host_lp.to(self.device, non_blocking=True).requires_grad_(True)
            return self._step(b, lp)

        return one, h2d, d2h

    def cpu_sample(self, rows, steps):
        """invokerl's own GRPO compute_advantages + compute_loss + backward (grpo.py:46-143) on the
        host CPU, on the first `rows` prompt groups of the same synthetic batch (all of them when
        rows is 0)."""
        from invokerl_b200.synthetic import rollout_batch

        ref = reference_package()
        torch.set_num_threads(os.cpu_count() or 1)
        P = self.P if rows <= 0 else min(self.P, rows)
        b = rollout_batch(P, self.G, self.T, prompt_len=self.pl, completion_len=self.cl, seed=0)
        new = b.extras["new_log_probs"]
        if ref is None:
            import oracle

            def one():
                adv = oracle.group_advantages(b.rewards, b.response_mask, self.G)
                oracle.clip_ratio_loss(new, b.old_log_probs, b.ref_log_probs, adv, b.response_mask, b.rewards)

            kind, what = "port", "the oracle's restatement"
        else:
            from invokerl.algorithms import GRPO as RefGRPO
            from invokerl.algorithms import RolloutBatch as RefBatch

            rb = RefBatch(token_ids=b.token_ids, prompt_mask=b.prompt_mask, response_mask=b.response_mask,
                          attention_mask=b.attention_mask, rewards=b.rewards, token_rewards=None,
                          old_log_probs=b.old_log_probs, ref_log_probs=b.ref_log_probs, group_ids=b.group_ids,
                          group_size=self.G)
            algo = RefGRPO(clip_eps=0.2, beta=0.04)

            def one():
                lp = new.clone().requires_grad_(True)
                adv = algo.compute_advantages(rb)
                loss, _ = algo.compute_loss(lp, rb, adv)
                loss.backward()

            kind, what = "reference", "invokerl's own GRPO"
        dt = time_cpu(one, steps)
        n = P * self.G * self.T
        return n / dt, dt, f"{P * self.G} rows x T={self.T} ({n} tokens) per step: {what} + autograd on the host CPU", kind


def init_single_rank_group(device) -> None:
    """A one-rank NCCL process group (FSDP needs one) when not launched under torchrun."""
    if dist.is_initialized():
        return
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1, device_id=device)


class E2EGRPO:
    """One GRPO training step of a random-init Qwen3-0.6B (28 layers, H=1024, 16 q / 8 kv heads of
    128, SwiGLU 3072, V=151936, tied, bf16, sdpa attention, gradient checkpointing as the
    reference's PolicyModel sets it): advantages -> policy forward -> GRPO loss -> backward ->
    AdamW step, as invokerl's Trainer.train_step plus the optimizer step (trainer.py:335-346).
    The log-prob path is the fused LM-head kernel and the loss is K3; the transformer is
    HuggingFace's.  Rollout log-probs (old, ref) are made once at setup."""

    B, T, G = 64, 2048, 8

    def __init__(self, key, args):
        self.key = key
        self.fsdp = bool(getattr(args, "fsdp", False))
        if args.batch:
            if args.batch % self.G:
                raise SystemExit(f"--batch must be a multiple of the group size {self.G}")
            self.B = args.batch

    @staticmethod
    def qwen3_0p6b_config():
        from transformers import Qwen3Config

        return Qwen3Config(vocab_size=V, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                           num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                           rms_norm_eps=1e-6, max_position_embeddings=40960, tie_word_embeddings=True,
                           use_cache=False)

    @classmethod
    def build_model(cls, device):
        from transformers import Qwen3ForCausalLM

        cfg = cls.qwen3_0p6b_config()
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(0)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(device):
                model = Qwen3ForCausalLM(cfg)
        finally:
            torch.set_default_dtype(prev)
        model.train()
        model.config.use_cache = False
        model.gradient_checkpointing_enable()
        return model

    @staticmethod
    def wrap_fsdp(model, device):
        """FSDP as invokerl's PolicyModel.fsdp() / distributed.wrap_fsdp set it up
        (distributed.py:100-160): FULL_SHARD, one unit per decoder layer, original parameters."""
        import functools

        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
        from torch.distributed.fsdp import ShardingStrategy
        from torch.distributed.fsdp.wrap import transformer_auto_wrap_policy
        from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer

        policy = functools.partial(transformer_auto_wrap_policy, transformer_layer_cls={Qwen3DecoderLayer})
        return FSDP(model, sharding_strategy=ShardingStrategy.FULL_SHARD, auto_wrap_policy=policy,
                    device_id=device, use_orig_params=True)

    @staticmethod
    def model_flops_per_token(cfg, T) -> float:
        """6 x matmul parameters (LM head included) + causal attention (QK^T and AV, fwd + bwd);
        the checkpointing recompute is not counted."""
        H, L, I = cfg.hidden_size, cfg.num_hidden_layers, cfg.intermediate_size
        dq, dkv = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
        per_layer = H * dq + 2 * H * dkv + dq * H + 3 * H * I
        params = L * per_layer + H * cfg.vocab_size
        attn = L * 3 * 2 * 2 * (T / 2) * dq
        return 6.0 * params + attn

    def setup(self, rank, world, device):
        from invokerl_b200.algorithms import GRPO
        from invokerl_b200.distributed import shard_batch
        from invokerl_b200.policy import PolicyModel
        from invokerl_b200.synthetic import rollout_batch

        self.model = self.build_model(device)
        self.cfg = self.model.config
        if self.fsdp:
            init_single_rank_group(device)
            self.model = self.wrap_fsdp(self.model, device)
        self.policy = PolicyModel.from_model(self.model, device=device, fsdp_wrapped=self.fsdp)
        b = rollout_batch(self.B // self.G, self.G, self.T, prompt_len=(64, 256), completion_len=(32, 256),
                          vocab=V, seed=0)
        local = shard_batch(b, rank, world)
        local.extras = {}
        lp = self.policy.forward_no_grad(local.token_ids.to(device), local.attention_mask.to(device))
        g = torch.Generator(device=device).manual_seed(11 + int(local.group_ids[0]))
        local.old_log_probs = (lp + 0.05 * torch.randn(lp.shape, device=device, generator=g)).cpu()
        local.ref_log_probs = (lp + 0.1 * torch.randn(lp.shape, device=device, generator=g)).cpu()
        del lp
        self.local = local
        self.dev_batch = to_device_batch(local, device)
        self.algo = GRPO(clip_eps=0.2, beta=0.04, row_sharded=world > 1)
        self.opt = torch.optim.AdamW(self.model.parameters(), lr=1e-6, fused=True)
        self.params = [p for p in self.model.parameters() if p.requires_grad]
        self.world = world
        self.device = device

    def timed_functions(self):
        return ["lmhead_forward_raw", "lmhead_backward_raw"]

    def _reduce_grads(self):
        # Row shards of whole groups: the rank losses sum to the global loss, so the gradients sum.
        grads = [p.grad for p in self.params if p.grad is not None]
        flat = torch._utils._flatten_dense_tensors(grads)
        dist.all_reduce(flat)
        for g, r in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
            g.copy_(r)

    def _step(self, batch):
        adv = self.algo.compute_advantages(batch)
        lp = self.policy.forward(batch.token_ids, batch.attention_mask)
        loss, metrics = self.algo.compute_loss(lp, batch, adv)
        # Row-sharded losses are shares of the global loss, so the rank gradients must be summed;
        # FSDP averages them over the ranks, hence the factor.
        (loss * self.world if (self.fsdp and self.world > 1) else loss).backward()
        if self.world > 1 and not self.fsdp:
            self._reduce_grads()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return float(loss.detach()), metrics

    def step(self):
        return self._step(self.dev_batch)

    def tokens_per_step(self):
        return self.B * self.T

    def roofline(self, kernel_ms_per_step, peaks, peak_src):
        return {}

    def step_roofline(self, ms_per_step, kernel_ms_per_step, peaks, peak_src):
        fpt = self.model_flops_per_token(self.cfg, self.T)
        flops = fpt * self.B * self.T / max(1, self.world)
        achieved = flops / (ms_per_step / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        H = self.cfg.hidden_size
        n_rows = self.dev_batch.token_ids.numel()
        # The head's algorithmic FLOPs: the forward over every row, dH and dW over the rows with a
        # nonzero upstream gradient (the response tokens; the last position of a row has no target).
        n_act = int(self.dev_batch.response_mask[:, 1:].sum())
        head_flops = (2.0 * n_rows + 4.0 * n_act) * H * V
        head_tf = head_flops / (kernel_ms_per_step / 1e3) / 1e12 if kernel_ms_per_step > 0 else None
        return {"kernel": "whole GRPO step (HF transformer + fused LM-head log-prob + K3 loss + AdamW); MFU",
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{peak_src} bf16 sustained",
                "algorithmic": f"model FLOPs {fpt / 1e9:.2f} GFLOP/token: 6 x matmul params (LM head included) "
                               "+ causal attention fwd+bwd; checkpoint recompute not counted",
                "lmhead_kernels_ms_per_step": kernel_ms_per_step,
                "lmhead_tflops": head_tf,
                "lmhead_active_rows": n_act,
                "traffic": None}

    def config(self, world):
        return {"workload": "GRPO train step, random-init Qwen3-0.6B (28 layers, H=1024, tied V=151936, bf16, "
                            "sdpa, gradient checkpointing) + AdamW; log-probs via the fused LM-head kernel",
                "global_batch": self.B, "seq_len": self.T, "group_size": self.G,
                "parallelism": (f"fsdp{world} (FULL_SHARD per decoder layer; materialised logits + the "
                                "logits kernel, as invokerl's FSDP branch)") if self.fsdp else
                               f"dp{world} (row shards of whole groups; gradient all-reduce)",
                "l2": "activations and weights far larger than L2, no flush"}

    def e2e(self):
        hb = host_batch(self.local)
        h2d = batch_bytes(hb)

        def one():
            return self._step(to_device_batch(hb, self.device))

        return one, h2d, 4 + 4 * 12

    def cpu_sample(self, rows, steps):
        return None


WORKLOADS = {"lmhead-8b": LMHeadGRPO, "lmhead-0.6b": LMHeadGRPO, "logits": LogitsLogProb, "grpo": GRPOHooks,
             "grpo-hbm": GRPOHooks, "e2e-0.6b": E2EGRPO}
# Rows of the bounded CPU sample per step (the reference's CPU path; 0 = every prompt group).
CPU_ROWS = {"lmhead-8b": 32, "lmhead-0.6b": 96, "logits": 1024, "grpo": 0, "grpo-hbm": 8, "e2e-0.6b": 0}
# Lines the default run adds after the headline, each a workload of its own with the same keys.
SECONDARY = ("logits", "lmhead-0.6b", "grpo-hbm", "e2e-0.6b")
SECONDARY_STEPS = {"logits": 20, "lmhead-0.6b": 10, "grpo-hbm": 20, "e2e-0.6b": 3}

# DRAM traffic of the dominant kernel per unit of work, from ncu captures (dram__bytes_read.sum +
# dram__bytes_write.sum); the line's roofline.traffic is this figure times the units of one step.
TRAFFIC = {
    # K1 at H = 4096, V = 151936 (profiles/lmhead_8b_dram_traffic.md; bench.py --batch 16): the forward
    # over 65,536 rows moved 51.37 GB, one full 28,160-row backward chunk (dS recompute, dW, dH)
    # 106.1 GB.  The forward's W re-reads grow with the rows, the backward's with the chunks.
    # At H = 1024 (profiles/lmhead_0.6b_dram_traffic.md; the whole Qwen3-0.6B config): the forward
    # over 131,072 rows moved 4.66 GB, the one backward chunk of 10,066 active rows 13.0 GB.
    "lmhead_fwd_per_row": {4096: 51.37e9 / 65536, 1024: 4.66e9 / 131072},
    "lmhead_bwd_per_active_row": {4096: 106.1e9 / 28160, 1024: 13.0e9 / 10066},
    # With the logit cache (H = 4096, the same step, 36,992 of 65,536 rows cached): the caching
    # forward moved 75.97 GB (12.1 GB of it the cache), one full backward chunk 110.3 GB (dS from
    # the cache 17.6 GB, dW 47.8 GB, dH 44.9 GB).
    "lmhead_fwd_per_row_cached": {4096: 75.97e9 / 65536},
    "lmhead_bwd_per_active_row_cached": {4096: 110.3e9 / 28160},
    # K2 forward + backward over [4096, 151936] bf16 logits, 51% active rows
    # (profiles/logits_logprob_fwd_bwd_4096x151936.md): 3.069 GB.
    "logits_per_row": 3.069e9 / 4096,
    # K3 GRPO loss kernel over 8,388,608 tokens (profiles/grpo_loss_and_advantages_1024x8192.md):
    # 160.9 MB.
    "grpo_loss_per_token": 160.9e6 / 8388608,
}


class Timed:
    """Device time of `steps` calls of `step` after `warmup` untimed ones, bracketed by a barrier and
    a synchronize on both sides and taken as the max over ranks, with nvidia-smi clocks sampled
    during the timed region and this library's launch count."""

    def __init__(self, step, steps, warmup, world, device, timer=None):
        from invokerl_b200 import _native

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        sampler = ClockSampler(device.index)
        sampler.start()
        time.sleep(0.3)
        launches0 = _native.lib().ikrl_launch_count()
        if timer is not None:
            timer.active = True
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record()
        out = None
        for _ in range(steps):
            out = step()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if timer is not None:
            timer.active = False
        self.launches = int(_native.lib().ikrl_launch_count() - launches0)
        self.clocks = sampler.stop()
        ms = start.elapsed_time(end)
        kms = timer.total_ms() if (timer is not None and timer.pairs) else ms
        t = torch.tensor([ms, kms], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        self.ms, self.kms = float(t[0]), float(t[1])
        self.has_kernel_time = timer is not None and bool(timer.pairs)
        # this rank's CUDA-event time of each timed function, per step
        self.kms_by_fn = {k: v / steps for k, v in timer.by_name_ms().items()} if self.has_kernel_time else {}
        self.out = out
        self.steps = steps


def input_copies(one) -> str:
    if getattr(one, "pipelined", False) and not Prefetch.serial:
        return "one step ahead on a copy stream (two device buffer sets)"
    return "in line with each step"


def time_e2e(one, n, world, device) -> float:
    """ms for n end-to-end steps (max over ranks), after one untimed step.  A step function marked
    `pipelined` takes (step index, steps) and copies its inputs through a Prefetch."""
    pipelined = getattr(one, "pipelined", False)
    one(0, 1) if pipelined else one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(n):
        one(i, n) if pipelined else one()
    e.record()
    torch.cuda.synchronize()
    te = torch.tensor([s.elapsed_time(e)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return float(te[0])


def run_native(args, key, rank, world, device, steps, warmup, cpu_baseline=True) -> dict | None:
    """One JSON line for workload `key` on this package's kernels."""
    from invokerl_b200 import ops

    wl = WORKLOADS[key](key, args)
    wl.setup(rank, world, device)
    timer = EventTimer()
    saved = {}
    for name in wl.timed_functions():
        saved[name] = getattr(ops, name)
        setattr(ops, name, timer.wrap(saved[name]))
    try:
        tm = Timed(wl.step, steps, warmup, world, device, timer)
        loss = tm.out[0] if tm.out else 0.0

        # Outside the timed region: the data-parallel reduction of the LM-head weight gradient that a
        # DP / FSDP layer adds per step (one NCCL all-reduce of dW in its dtype), timed apart and also
        # added to the step in value_with_dw_allreduce.
        dw_allreduce = None
        if world > 1 and isinstance(wl, LMHeadGRPO) and wl.weight.grad is not None:
            gw = wl.weight.grad
            for _ in range(2):
                dist.all_reduce(gw)
            torch.cuda.synchronize()
            dist.barrier()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            for _ in range(5):
                dist.all_reduce(gw)
            s1.record()
            torch.cuda.synchronize()
            ta = torch.tensor([s0.elapsed_time(s1) / 5], dtype=torch.float64, device=device)
            dist.all_reduce(ta, op=dist.ReduceOp.MAX)
            nbytes = gw.numel() * gw.element_size()
            dw_allreduce = {"ms": float(ta[0]), "bytes": int(nbytes), "dtype": str(gw.dtype).replace("torch.", ""),
                            "bus_gbs": 2 * (world - 1) / world * nbytes / (float(ta[0]) / 1e3) / 1e9,
                            "note": "NCCL all-reduce of dW per step, timed after the timed region"}
        rank_rows = None
        if world > 1 and isinstance(wl, LMHeadGRPO):
            mine = torch.tensor([wl.Bl * wl.T, int(wl.dev_batch.response_mask.sum())], dtype=torch.float64,
                                device=device)
            allr = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allr, mine)
            rows = [int(x[0]) for x in allr]
            act = [int(x[1]) for x in allr]
            rank_rows = {"rows_max": max(rows), "rows_mean": sum(rows) / world, "active_rows_max": max(act),
                         "active_rows_mean": sum(act) / world, "active_rows_per_rank": act}

        e2e = None
        if not args.no_e2e:
            one, h2d, d2h = wl.e2e()
            n = max(1, min(steps, 5))
            te = time_e2e(one, n, world, device)
            e2e = {"value": wl.tokens_per_step() * n / (te / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                   "d2h_bytes_per_step": int(d2h), "steps": n, "input_copies": input_copies(one)}
    finally:
        for name, fn in saved.items():
            setattr(ops, name, fn)

    if rank != 0:
        del wl
        return None
    peaks, peak_src = load_peaks()
    ms, kms = tm.ms, tm.kms
    res = {
        "metric": METRIC,
        "value": wl.tokens_per_step() * steps / (ms / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms / steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32" if key.startswith("grpo") else "bf16",
        "data": "synthetic (seeded; random-init weights)",
        "config": wl.config(world),
        "roofline": (wl.step_roofline(ms / steps, (kms / steps) if tm.has_kernel_time else 0.0, peaks, peak_src)
                     if isinstance(wl, E2EGRPO) else wl.roofline(kms / steps, peaks, peak_src)),
        "e2e": e2e,
        "gpu_launches": tm.launches,
        "kernel_ms_per_step": {k: round(v, 3) for k, v in tm.kms_by_fn.items()} or None,
        "clocks": tm.clocks,
        "loss": loss,
    }
    if dw_allreduce is not None:
        res["dw_allreduce"] = dw_allreduce
        step_ms = ms / steps + dw_allreduce["ms"]
        res["value_with_dw_allreduce"] = wl.tokens_per_step() / (step_ms / 1e3)
    if rank_rows is not None:
        res["rank_rows"] = rank_rows
    if world == 1 and cpu_baseline and not args.no_cpu_baseline and not isinstance(wl, E2EGRPO):
        tok_s, dt, sample, kind = wl.cpu_sample(CPU_ROWS[key], 3)
        res["cpu_baseline"] = {"value": tok_s, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
                               "sample": sample + f"; 3 steps of {dt:.3f} s"}
    del wl
    return res


def run_reference(args, rank, world) -> dict | None:
    """The reference's own CPU implementation of the path on the host cores (rank 0 only), same
    metric, unit and config; each step a bounded sample of the workload."""
    if rank != 0:
        return None
    if args.workload == "e2e-0.6b":
        return {"impl": "reference", "unavailable": "a 0.6B-parameter training step on the host CPU is not a "
                "meaningful baseline; bench.py --workload e2e-0.6b --reference-gpu times the reference's GPU path"}
    wl = WORKLOADS[args.workload](args.workload, args)
    rows = CPU_ROWS[args.workload]
    for _ in range(max(0, args.warmup - 1)):
        wl.cpu_sample(rows, 1)
    tok_s, dt, sample, kind = wl.cpu_sample(rows, max(1, args.steps))
    cfg = dict(wl.config(world))
    cfg["sample"] = sample
    return {
        "metric": METRIC,
        "value": tok_s,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32" if args.workload.startswith("grpo") else "bf16",
        "data": "synthetic (seeded)",
        "impl": "reference",
        "config": cfg,
        "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
                         "sample": sample},
        "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---- the reference's own GPU path on the same box -------------------------------------------------


def ref_batch_of(db):
    from invokerl.algorithms import RolloutBatch as RefBatch

    return RefBatch(token_ids=db.token_ids, prompt_mask=db.prompt_mask, response_mask=db.response_mask,
                    attention_mask=db.attention_mask, rewards=db.rewards, token_rewards=None,
                    old_log_probs=db.old_log_probs, ref_log_probs=db.ref_log_probs, group_ids=db.group_ids,
                    group_size=db.group_size)


def ref_gpu_lmhead(key, args, device):
    """invokerl's PolicyModel._chunked_lm_head_ce (F.linear + -F.cross_entropy per 64-token chunk
    under torch.utils.checkpoint, cuBLAS GEMMs; policy.py:124-191) and its GRPO (grpo.py:46-143)."""
    from invokerl.algorithms import GRPO as RefGRPO
    from invokerl.policy import PolicyModel as RefPolicy

    wl = LMHeadGRPO(key, args)
    wl.setup(0, 1, device)
    H, B, T = wl.H, wl.B, wl.T
    head = torch.nn.Linear(H, V, bias=False, device=device, dtype=torch.bfloat16)
    with torch.no_grad():
        head.weight.copy_(wl.weight.detach())
    pm = RefPolicy.__new__(RefPolicy)
    pm.model = torch.nn.Module()
    pm.model.lm_head = head
    hidden = wl.hidden.detach().view(B, T, H).clone().requires_grad_(True)
    host_hidden = hidden.detach().cpu().pin_memory()
    hb = host_batch(wl.local)
    rb = ref_batch_of(wl.dev_batch)
    algo = RefGRPO(clip_eps=0.2, beta=0.04)
    del wl

    def run(h, b):
        head.weight.grad = None
        lp = pm._chunked_lm_head_ce(h, b.token_ids, 64)
        adv = algo.compute_advantages(b)
        loss, _ = algo.compute_loss(lp, b, adv)
        loss.backward()
        return loss

    def step():
        hidden.grad = None
        return run(hidden, rb)

    pf = Prefetch({"hidden": host_hidden, **{k: v for k, v in vars(hb).items() if isinstance(v, torch.Tensor)}},
                  device)

    def e2e(i=0, n=1):
        d = pf.get(i, n)
        h = d["hidden"].detach().requires_grad_(True)
        b = ref_batch_of(batch_from(hb, d))
        return float(run(h, b).detach())  # the reference reads its metrics with .item() as well

    e2e.pipelined = True
    return dict(step=step, e2e=e2e, tokens=B * T, h2d=host_hidden.numel() * 2 + batch_bytes(hb), d2h=4,
                workload=LMHeadGRPO.PRESETS[key]["name"] + ", invokerl's own chunked F.linear + cross_entropy "
                "path and GRPO on the same GPU")


def ref_gpu_hooks(key, args, device):
    """invokerl's own GRPO compute_advantages + compute_loss + backward (its eager ATen ops and
    metric .item() calls) on the same batch as the grpo workloads."""
    from invokerl.algorithms import GRPO as RefGRPO

    wl = GRPOHooks(key, args)
    wl.setup(0, 1, device)
    rb = ref_batch_of(wl.dev_batch)
    hb = host_batch(wl.local)
    host_lp = wl.new.pin_memory()
    algo = RefGRPO(clip_eps=0.2, beta=0.04)
    lp0 = wl.lp.detach()
    tokens = wl.tokens_per_step()
    cfg = wl.config(1)["workload"]
    del wl

    def run(lp, b):
        adv = algo.compute_advantages(b)
        loss, _ = algo.compute_loss(lp, b, adv)
        loss.backward()
        return loss

    def step():
        return run(lp0.clone().requires_grad_(True), rb)

    def e2e():
        b = ref_batch_of(to_device_batch(hb, device))
        return float(run(host_lp.to(device, non_blocking=True).requires_grad_(True), b).detach())

    return dict(step=step, e2e=e2e, tokens=tokens, h2d=batch_bytes(hb) + host_lp.numel() * 4, d2h=4,
                workload=cfg + ", invokerl's own GRPO on the same GPU")


def ref_gpu_logits(key, args, device):
    """The reference's materialised-logits log-prob (policy.py:100-104: -F.cross_entropy over
    [N, V] bf16 logits, reduction="none") forward + autograd backward."""
    import torch.nn.functional as F

    wl = LogitsLogProb(key, args)
    wl.setup(0, 1, device)
    x = wl.logits.detach().requires_grad_(True)
    t, up = wl.t, wl.up
    host_logits = x.detach().cpu().pin_memory()
    host_t, host_up = t.cpu().pin_memory(), up.cpu().pin_memory()
    n = wl.N
    del wl

    def run(xx, tt, uu):
        lp = -F.cross_entropy(xx, tt, reduction="none")
        lp.backward(uu.to(lp.dtype))
        return lp

    def step():
        x.grad = None
        return run(x, t, up)

    def e2e():
        xx = host_logits.to(device, non_blocking=True).requires_grad_(True)
        lp = run(xx, host_t.to(device, non_blocking=True), host_up.to(device, non_blocking=True))
        return float(lp.detach().float().sum())

    return dict(step=step, e2e=e2e, tokens=n,
                h2d=host_logits.numel() * 2 + host_t.numel() * 8 + host_up.numel() * 4, d2h=4,
                workload=f"logits bf16 [{n}, {V}]: invokerl's -F.cross_entropy fwd + autograd bwd on the same GPU")


def reference_gpu_line(key, args, device, steps, warmup) -> dict:
    """The reference's own GPU path for workload `key` on this GPU: value, ms_per_step, e2e and the
    clocks of its timed region, for the same config as this package's line."""
    if reference_package() is None:
        return {"impl": "reference-gpu", "unavailable": "the reference package is not in baseline/_ref"}
    if key == "e2e-0.6b":
        return run_reference_gpu_e2e(args, device, steps, warmup)
    make = ref_gpu_lmhead if key in LMHeadGRPO.PRESETS else ref_gpu_hooks if key.startswith("grpo") else ref_gpu_logits
    torch.cuda.reset_peak_memory_stats(device)
    leg = make(key, args, device)
    torch.cuda.synchronize()
    sampler = ClockSampler(device.index)
    for _ in range(warmup):
        leg["step"]()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        leg["step"]()
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = s.elapsed_time(e) / steps
    ne = max(1, min(steps, 5))
    te = time_e2e(leg["e2e"], ne, 1, device)
    out = {"impl": "reference-gpu", "metric": METRIC, "value": leg["tokens"] / (ms / 1e3), "unit": UNIT,
           "ms_per_step": ms, "steps": steps, "warmup": warmup, "same_config": True,
           "e2e": {"value": leg["tokens"] * ne / (te / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(leg["h2d"]),
                   "d2h_bytes_per_step": int(leg["d2h"]), "steps": ne, "input_copies": input_copies(leg["e2e"])},
           "clocks": clocks, "config": {"workload": leg["workload"]},
           "peak_mem_gb": torch.cuda.max_memory_allocated(device) / 1e9}
    del leg
    release(device)
    return out


def release(device):
    import gc

    gc.collect()
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()


def run_reference_gpu_e2e(args, device, steps: int | None = None, warmup: int | None = None) -> dict:
    """The same GRPO train step with invokerl's own PolicyModel.forward (its chunked
    F.linear + cross_entropy log-prob path under torch.utils.checkpoint) and its GRPO, on the same
    random-init model, batch and optimizer."""
    from invokerl.algorithms import GRPO as RefGRPO
    from invokerl.algorithms import RolloutBatch as RefBatch
    from invokerl.policy import PolicyModel as RefPolicy
    from invokerl_b200.synthetic import rollout_batch

    wl = E2EGRPO("e2e-0.6b", args)
    model = E2EGRPO.build_model(device)
    cfg = model.config
    if wl.fsdp:
        init_single_rank_group(device)
        model = E2EGRPO.wrap_fsdp(model, device)
    pm = RefPolicy.__new__(RefPolicy)
    pm.model, pm.device, pm.dtype = model, device, torch.bfloat16
    pm.master_weights_fp32, pm._autocast_dtype, pm._fsdp_wrapped = False, None, wl.fsdp
    b = rollout_batch(wl.B // wl.G, wl.G, wl.T, prompt_len=(64, 256), completion_len=(32, 256), vocab=V, seed=0)
    ids, am = b.token_ids.to(device), b.attention_mask.to(device)
    with torch.no_grad():
        lp = pm.forward(ids, am).float()
    g = torch.Generator(device=device).manual_seed(11)
    old = lp + 0.05 * torch.randn(lp.shape, device=device, generator=g)
    ref = lp + 0.1 * torch.randn(lp.shape, device=device, generator=g)
    del lp
    rb = RefBatch(token_ids=ids, prompt_mask=b.prompt_mask.to(device), response_mask=b.response_mask.to(device),
                  attention_mask=am, rewards=b.rewards.to(device), token_rewards=None, old_log_probs=old,
                  ref_log_probs=ref, group_ids=b.group_ids.to(device), group_size=wl.G)
    algo = RefGRPO(clip_eps=0.2, beta=0.04)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-6, fused=True)

    def step():
        adv = algo.compute_advantages(rb)
        new = pm.forward(rb.token_ids, rb.attention_mask)
        loss, _ = algo.compute_loss(new, rb, adv)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    steps = max(1, min(args.steps, 3)) if steps is None else steps
    warmup = max(1, args.warmup - 1) if warmup is None else warmup
    try:
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
    except torch.cuda.OutOfMemoryError as e:
        return {"metric": METRIC, "impl": "reference-gpu", "value": None, "unit": UNIT,
                "unavailable": f"OOM in invokerl's own step ({'FSDP materialised logits' if wl.fsdp else 'chunked'}"
                               f" path): {str(e).splitlines()[0][:160]}",
                "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9}
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = steps
    sampler = ClockSampler(device.index)
    sampler.start()
    time.sleep(0.3)
    s.record()
    for _ in range(n):
        step()
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = s.elapsed_time(e) / n
    fpt = E2EGRPO.model_flops_per_token(cfg, wl.T)
    peaks, _ = load_peaks()
    achieved = fpt * wl.B * wl.T / (ms / 1e3) / 1e12
    return {"metric": METRIC, "impl": "reference-gpu", "value": wl.B * wl.T / (ms / 1e3), "unit": UNIT,
            "ms_per_step": ms, "steps": n, "warmup": warmup, "same_config": True, "clocks": clocks,
            "mfu_tflops": achieved,
            "mfu_frac": achieved / peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]),
            "config": {"workload": "GRPO train step, random-init Qwen3-0.6B + AdamW, invokerl's own "
                                   "PolicyModel.forward (chunked F.linear + cross_entropy) and GRPO on the same GPU",
                       "global_batch": wl.B, "seq_len": wl.T},
            "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9}


def apply_tuning(args) -> dict:
    """--tune knob=value and --ds-chunk-bytes: launch knobs of the library for A/B runs."""
    from invokerl_b200 import _native, ops

    applied = {}
    for kv in args.tune:
        k, v = kv.split("=", 1)
        _native.set_tuning(k, int(v))
        applied[k] = int(v)
    if args.ds_chunk_bytes:
        ops.set_ds_chunk_bytes(args.ds_chunk_bytes)
        applied["ds_chunk_bytes"] = args.ds_chunk_bytes
    if args.logit_cache != "auto":
        ops.set_logit_cache(args.logit_cache)
        applied["logit_cache"] = args.logit_cache
    return applied


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="lmhead-8b")
    ap.add_argument("--batch", type=int, default=0, help="override the global batch B of the lmhead workloads")
    ap.add_argument("--rows", type=int, default=0, help="override the rows of the logits workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-serial", action="store_true",
                    help="copy each e2e step's inputs in line with the step instead of one step ahead")
    ap.add_argument("--no-secondary", action="store_true",
                    help="only the headline line: no reference_gpu leg and no secondary workloads")
    ap.add_argument("--fsdp", action="store_true",
                    help="e2e-0.6b: wrap the model in FSDP as invokerl's PolicyModel.fsdp() does (per-layer "
                         "FULL_SHARD); the log-prob path then takes the materialised-logits branch")
    ap.add_argument("--reference-gpu", action="store_true",
                    help="time the reference's own GPU path (baseline/_ref) instead; one extra JSON line")
    ap.add_argument("--tune", action="append", default=[], metavar="KNOB=VALUE",
                    help="set a library launch knob (ikrl_set_tuning) for an A/B run")
    ap.add_argument("--ds-chunk-bytes", type=int, default=0, help="bytes of the K1 backward's dlogits chunk")
    ap.add_argument("--logit-cache", choices=["auto", "off"], default="auto",
                    help="the K1 logit cache policy (off: the backward recomputes every active row's logits)")
    args = ap.parse_args()
    Prefetch.serial = args.e2e_serial
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return 0
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    tuned = apply_tuning(args)
    if args.reference_gpu:
        if rank == 0:
            print(json.dumps(reference_gpu_line(args.workload, args, device, max(1, min(args.steps, 5)),
                                                max(1, args.warmup))), flush=True)
        if dist.is_initialized():
            dist.destroy_process_group()
        return 0
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    try:
        res = run_native(args, args.workload, rank, world, device, args.steps, args.warmup)
        release(device)
        if rank == 0 and res is not None:
            if tuned:
                res["tuning"] = tuned
            extra = world == 1 and not args.no_secondary and args.workload == "lmhead-8b" and not tuned
            if extra:
                # The reference's own B200 path on the same config, then the other configs, each a
                # line of its own with its reference leg.
                res["reference_gpu"] = reference_gpu_line(args.workload, args, device, 3, 2)
                res["secondary"] = []
                for key in SECONDARY:
                    line = run_native(args, key, 0, 1, device, SECONDARY_STEPS[key], 3)
                    release(device)
                    line["workload_key"] = key
                    line["reference_gpu"] = reference_gpu_line(key, args, device, min(10, SECONDARY_STEPS[key]), 3)
                    res["secondary"].append(line)
            print(json.dumps(res), flush=True)
    finally:
        if dist.is_initialized():  # torchrun ranks, or the one-rank group of --fsdp
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
