"""Row sharding on 2 GPUs over NCCL: each rank runs the fused LM head and GRPO loss on its whole
prompt groups; the all-reduced metrics and the summed loss shares equal the single-process
oracle on the full batch, and each rank's gradients are the full-batch gradients of its rows.
Skipped when fewer than two GPUs are visible."""

import datetime
import os

import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

P, G, T, H, V = 4, 4, 64, 128, 3000



def free_port() -> int:
    """A TCP port that is free on 127.0.0.1 right now (for a gloo/NCCL rendezvous)."""
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]

def make_inputs():
    from invokerl_b200.synthetic import lmhead_inputs, rollout_batch

    b = rollout_batch(P, G, T, prompt_len=(4, 20), completion_len=(8, 40), vocab=V, seed=3)
    li = lmhead_inputs(P * G * T, H, V, seed=4, w_std=0.3)
    return b, li


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from invokerl_b200 import ops
    from invokerl_b200.algorithms import GRPO
    from invokerl_b200.distributed import group_shard_bounds, shard_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        b, li = make_inputs()
        s, e = group_shard_bounds(P * G, G, rank, world)
        local = shard_batch(b, rank, world)
        local.extras = {}
        db = type(local)(**{k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in vars(local).items()
                            if k != "extras"}, extras={})
        h = li.hidden.reshape(P * G, T, H)[s:e].reshape(-1, H).to(dev).requires_grad_(True)
        w = li.weight.to(dev).requires_grad_(True)
        lp = ops.lmhead_logprob(h, w, db.token_ids.reshape(-1)).view(e - s, T)
        algo = GRPO(row_sharded=True)
        adv = algo.compute_advantages(db)
        loss, metrics = algo.compute_loss(lp, db, adv)
        loss.backward()
        tot = loss.detach().clone()
        dist.all_reduce(tot)
        dw = w.grad.float().clone()
        dist.all_reduce(dw)
        grads = [torch.empty_like(h.grad) for _ in range(world)]
        dist.all_gather(grads, h.grad.contiguous())
        if rank == 0:
            q.put((float(tot), metrics, torch.cat(grads).cpu(), dw.cpu(), lp.detach().cpu()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_row_sharding_matches_full_batch():
    import oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    tot, metrics, dh, dw, _ = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    b, li = make_inputs()
    lp_full = oracle.lmhead_logprob(li.hidden, li.weight, b.token_ids.reshape(-1)).view(P * G, T)
    adv = oracle.group_advantages(b.rewards, b.response_mask, G)
    loss, met, g = oracle.clip_ratio_loss(lp_full, b.old_log_probs, b.ref_log_probs, adv, b.response_mask, b.rewards)
    assert abs(tot - float(loss)) <= 1e-4 * abs(float(loss)) + 1e-6
    for k in ("loss", "reward", "kl", "policy_loss", "clip_frac", "approx_kl", "advantages_mean"):
        assert abs(metrics[k] - met[k]) <= 1e-4 * abs(met[k]) + 1e-6, k
    _, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden, li.weight, b.token_ids.reshape(-1), g.reshape(-1))
    rel = lambda a, c: float((a.float() - c.float()).norm() / c.float().norm())  # noqa: E731
    assert rel(dh, dh_o) <= 1e-2
    assert rel(dw, dw_o) <= 1e-2


def _vp_worker(rank, world, port, q):
    import torch.distributed as dist

    from invokerl_b200.synthetic import lmhead_inputs
    from invokerl_b200.vocab_parallel import lmhead_logprob_vocab_parallel, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        n, h_dim, v = 384, 256, 33000
        li = lmhead_inputs(n, h_dim, v, seed=12, w_std=0.3)
        s, e = shard_bounds(v, world, rank)
        h = li.hidden.to(dev).requires_grad_(True)
        w = li.weight[s:e].contiguous().to(dev).requires_grad_(True)
        up = torch.randn(n, generator=torch.Generator().manual_seed(13)).to(dev)
        lp = lmhead_logprob_vocab_parallel(h, w, li.targets.to(dev), s, v)
        (lp * up).sum().backward()
        dws = [None] * world
        dist.all_gather_object(dws, w.grad.float().cpu())
        if rank == 0:
            q.put((lp.detach().cpu(), h.grad.float().cpu(), torch.cat(dws)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_vocab_parallel_head_matches_oracle():
    import oracle
    from invokerl_b200.synthetic import lmhead_inputs

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_vp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    lp, dh, dw = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    li = lmhead_inputs(384, 256, 33000, seed=12, w_std=0.3)
    up = torch.randn(384, generator=torch.Generator().manual_seed(13))
    lp_o, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden, li.weight, li.targets, up)
    assert float((lp - lp_o).abs().max()) <= 2e-3
    rel = lambda a, c: float((a.float() - c.float()).norm() / c.float().norm())  # noqa: E731
    assert rel(dh, dh_o) <= 1e-2
    assert rel(dw, dw_o) <= 1e-2


def _algo_worker(rank, world, port, q, name):
    import sys
    from pathlib import Path

    import torch.distributed as dist

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from helpers import load, make_batch
    from invokerl_b200.algorithms import DAPO, DPO, GRPO, PPO, SimPO
    from invokerl_b200.distributed import shard_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        g = load(name)
        cls = {"grpo": GRPO, "dapo": DAPO, "ppo": PPO, "simpo": SimPO, "dpo": DPO}[g["kind"]]
        b = make_batch(g["batch"], dev)
        local = shard_batch(b, rank, world)
        nl = shard_batch(type(b)(**{**vars(b), "extras": {"nl": g["new_lp"].to(dev)}}), rank, world).extras["nl"]
        algo = cls(row_sharded=True, **g["kwargs"])
        adv = algo.compute_advantages(local)
        lp = nl.clone().requires_grad_(True)
        loss, metrics = algo.compute_loss(lp, local, adv)
        loss.backward()
        tot = loss.detach().clone().float()
        dist.all_reduce(tot)
        grads = [torch.empty_like(lp.grad) for _ in range(world)]
        dist.all_gather(grads, lp.grad.contiguous())
        if rank == 0:
            q.put((float(tot), metrics, torch.cat(grads).cpu()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["grpo_cfg1", "dapo_default", "ppo_values", "simpo_default", "dpo_default"])
def test_two_rank_algorithms_match_reference_golden(name):
    """Every algorithm row-sharded over 2 ranks (whole groups / pairs per rank): the summed loss
    shares, the global metrics and the gathered gradient equal the reference's own outputs."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from helpers import assert_metrics_close, load

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_algo_worker, args=(r, world, port, q, name)) for r in range(world)]
    for p in procs:
        p.start()
    tot, metrics, grad = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = load(name)["out"]
    assert abs(tot - float(out["loss"])) <= 1e-4 * abs(float(out["loss"])) + 1e-6
    assert_metrics_close(metrics, out["metrics"], rtol=1e-4, atol=1e-6)
    bf = out["grad"].dtype == torch.bfloat16
    torch.testing.assert_close(grad.float(), out["grad"].float(), rtol=1e-2 if bf else 1e-4, atol=1e-7)


def _scatter_nccl_worker(rank, world, port, q):
    import torch.distributed as dist

    from invokerl_b200.distributed import scatter_batch, shard_batch
    from invokerl_b200.synthetic import rollout_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        full = rollout_batch(6, 8, 256, prompt_len=(8, 64), completion_len=(16, 180), vocab=V, seed=12)
        full.extras["truncated"] = torch.arange(48) % 7 == 0
        local = scatter_batch(full if rank == 0 else None, src=0)
        ref = shard_batch(full, rank, world, balance=True)
        ok = local.token_ids.device == dev
        for f in ("token_ids", "prompt_mask", "response_mask", "attention_mask", "rewards", "old_log_probs",
                  "ref_log_probs", "group_ids"):
            ok = ok and torch.equal(getattr(local, f).cpu(), getattr(ref, f))
        for k in ("new_log_probs", "truncated"):
            ok = ok and torch.equal(local.extras[k].cpu(), ref.extras[k])
        q.put((rank, bool(ok), int(local.token_ids.shape[0])))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_scatter_batch_over_nccl_matches_balanced_shards():
    """Rollout distribution over NCCL (replacing invokerl/distributed.py:236-302): each rank
    receives, on its own GPU, exactly the work-balanced groups shard_batch(balance=True) gives it."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_scatter_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in got), got
    assert sum(n for _, _, n in got) == 48
