"""Host-side logic that needs no GPU: group sharding, loss parameters, synthetic inputs."""

import os

import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from invokerl_b200 import _native as N
from invokerl_b200 import ops
from invokerl_b200.algorithms import DAPO, GRPO, PPO
from invokerl_b200.distributed import group_shard_bounds, shard_batch
from invokerl_b200.synthetic import rollout_batch



def free_port() -> int:
    """A TCP port that is free on 127.0.0.1 right now (for a gloo/NCCL rendezvous)."""
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]

@pytest.mark.parametrize("B,G,world", [(16, 4, 1), (16, 4, 2), (16, 4, 3), (128, 8, 8), (8, 8, 4), (12, 2, 5)])
def test_group_shards_cover_whole_groups(B, G, world):
    seen = []
    for r in range(world):
        s, e = group_shard_bounds(B, G, r, world)
        assert s % G == 0 and e % G == 0 and s <= e
        seen.extend(range(s, e))
    assert seen == list(range(B))


def test_shard_bounds_reject_partial_groups():
    with pytest.raises(ValueError):
        group_shard_bounds(10, 4, 0, 2)


def test_shard_batch_slices_every_row_field():
    b = rollout_batch(4, 4, 64, prompt_len=(4, 16), completion_len=(4, 32), seed=0)
    b.extras["truncated"] = torch.arange(16) % 3 == 0
    s = shard_batch(b, 1, 2)
    assert s.token_ids.shape == (8, 64)
    assert torch.equal(s.rewards, b.rewards[8:16])
    assert torch.equal(s.extras["truncated"], b.extras["truncated"][8:16])
    assert s.extras["new_log_probs"].shape == (8, 64)


def test_loss_params_follow_each_algorithm():
    p = GRPO(clip_eps=0.3, beta=0.1, kl_type="simple")._params()
    assert p.family == N.IKRL_LOSS_GRPO and abs(p.ratio_lo - 0.7) < 1e-7 and abs(p.ratio_hi - 1.3) < 1e-7
    assert p.kl_type == N.IKRL_KL_SIMPLE and abs(p.beta - 0.1) < 1e-7
    d = DAPO()._params()
    assert abs(d.ratio_lo - 0.8) < 1e-7 and abs(d.ratio_hi - 1.28) < 1e-6 and abs(d.clip_metric_eps - 0.2) < 1e-7
    q = PPO()._params()
    assert q.family == N.IKRL_LOSS_PPO and q.kl_type == N.IKRL_KL_NONE and abs(q.entropy_coef - 0.01) < 1e-7
    assert ops.make_loss_params(0, 0.8, 1.2, 0.2, 0.0).kl_type == N.IKRL_KL_SCHULMAN


def test_synthetic_batch_layout():
    b = rollout_batch(4, 4, 512, seed=3)
    assert b.token_ids.shape == (16, 512) and b.group_size == 4
    assert not (b.prompt_mask & b.response_mask).any()
    c = b.response_mask.sum(1)
    assert int(c.min()) >= 32 and int(c.max()) <= 256
    assert set(b.rewards.tolist()) <= {0.0, 1.0}
    assert float(b.extras["new_log_probs"].max()) <= 0.0


# ---- row sharding over gloo ranks: sharded loss shares and gradients equal the global ones ----


def _sharded_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        b = rollout_batch(4, 4, 128, prompt_len=(8, 40), completion_len=(8, 80), seed=21)
        local = shard_batch(b, rank, world)
        adv = oracle.group_advantages(local.rewards, local.response_mask, local.group_size)
        n = local.response_mask.sum().to(torch.int64).reshape(1)
        dist.all_reduce(n)  # the one collective before the loss
        lp = local.extras["new_log_probs"].clone().requires_grad_(True)
        m = local.response_mask.float()
        ratio = torch.exp(lp - local.old_log_probs)
        pl = -torch.minimum(ratio * adv, torch.clamp(ratio, 0.8, 1.2) * adv)
        d = local.ref_log_probs - lp
        share = ((pl + 0.04 * (torch.exp(d) - d - 1)) * m).sum() / n.clamp(min=1).float()
        share.backward()
        tot = share.detach().clone()
        dist.all_reduce(tot)
        grads = [torch.zeros(4 * 4 // world * 1, 128) for _ in range(world)]
        dist.all_gather(grads, lp.grad.contiguous())
        if rank == 0:
            q.put((float(tot), torch.cat(grads)))
    finally:
        dist.destroy_process_group()


def test_row_sharded_loss_matches_global_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    tot, grad = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = rollout_batch(4, 4, 128, prompt_len=(8, 40), completion_len=(8, 80), seed=21)
    adv = oracle.group_advantages(b.rewards, b.response_mask, 4)
    loss, _, g = oracle.clip_ratio_loss(b.extras["new_log_probs"], b.old_log_probs, b.ref_log_probs, adv,
                                        b.response_mask, b.rewards)
    assert abs(tot - float(loss)) <= 1e-5 * abs(float(loss)) + 1e-7
    torch.testing.assert_close(grad, g, rtol=1e-5, atol=1e-8)


def _scatter_source_batch():
    b = rollout_batch(6, 4, 48, prompt_len=(4, 16), completion_len=(4, 30), seed=31)
    b.extras["truncated"] = torch.arange(24) % 5 == 0
    b.extras["note"] = "kept"
    b.extras["scale"] = torch.tensor([2.0, 3.0])
    b.extras["values"] = torch.randn(24, 48, generator=torch.Generator().manual_seed(3))
    return b


def _scatter_worker(rank, world, port, q, balance):
    import datetime

    from invokerl_b200.distributed import scatter_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        b = _scatter_source_batch() if rank == 0 else None
        local = scatter_batch(b, src=0, device="cpu", balance=balance)
        q.put((rank, {k: v for k, v in vars(local).items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,balance", [(2, True), (3, True), (2, False), (3, False), (8, True)])
def test_scatter_batch_sends_each_rank_its_groups(world, balance):
    """Every rank receives exactly the rows shard_batch gives it (balanced by work, or contiguous),
    with every field, row-shaped extras sharded and the other extras whole; with 8 ranks and 6
    groups two ranks receive no rows."""
    from invokerl_b200.distributed import shard_batch

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_scatter_worker, args=(r, world, port, q, balance)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _scatter_source_batch()
    nrows = 0
    for rank, loc in got:
        ref = shard_batch(full, rank, world, balance=balance)
        for f in ("token_ids", "prompt_mask", "response_mask", "attention_mask", "rewards", "old_log_probs",
                  "ref_log_probs", "group_ids"):
            assert loc[f].dtype == getattr(ref, f).dtype, f
            assert torch.equal(loc[f], getattr(ref, f)), f
        assert loc["token_rewards"] is None and loc["group_size"] == 4
        assert list(loc["extras"]) == list(full.extras)
        assert torch.equal(loc["extras"]["new_log_probs"], ref.extras["new_log_probs"])
        assert torch.equal(loc["extras"]["truncated"], ref.extras["truncated"])
        assert torch.equal(loc["extras"]["values"], ref.extras["values"])
        assert loc["extras"]["note"] == "kept" and torch.equal(loc["extras"]["scale"], torch.tensor([2.0, 3.0]))
        nrows += loc["token_ids"].shape[0]
    assert nrows == 24


def _pair_share_worker(rank, world, port, q, pairs):
    import datetime

    from invokerl_b200.algorithms import SimPO

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        loss = torch.tensor(0.5 + rank, requires_grad=True)
        metrics = torch.arange(8, dtype=torch.float32) + 10 * rank
        share, mt = SimPO(row_sharded=True)._pair_share(loss, metrics, 2 * pairs[rank])
        share.backward()
        q.put((rank, float(share), mt, float(loss.grad)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pairs", [(3, 5), (0, 4), (0, 0)])
def test_pair_share_over_ranks_gloo(pairs):
    """SimPO / DPO row shards: the loss share is local mean x local pairs / global pairs and the
    metrics are pair-weighted means; a rank without pairs, or a batch with none at all, gives a
    zero share and no division by zero."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_pair_share_worker, args=(r, world, port, q, pairs)) for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    tot = max(1, sum(pairs))
    want_mt = sum((torch.arange(8, dtype=torch.float64) + 10 * r) * pairs[r] for r in range(world)) / tot
    for rank, share, mt, grad in got:
        assert abs(share - (0.5 + rank) * pairs[rank] / tot) <= 1e-6
        assert abs(grad - pairs[rank] / tot) <= 1e-6
        assert torch.isfinite(mt).all()
        torch.testing.assert_close(mt, want_mt.float(), rtol=1e-6, atol=1e-6)


def test_balanced_groups_cover_every_group_once_and_balance_work():
    from invokerl_b200.distributed import balanced_groups

    b = rollout_batch(16, 8, 512, prompt_len=(16, 64), completion_len=(32, 448), seed=5)
    G, T = 8, 512
    for world in (1, 2, 3, 8):
        parts = balanced_groups(b.response_mask, G, world)
        assert sorted(g for p in parts for g in p) == list(range(16))
        assert parts == balanced_groups(b.response_mask, G, world)  # deterministic
        tok = b.response_mask.reshape(16, G * T).sum(1).tolist()
        load = [sum(G * T + 3 * tok[g] for g in p) for p in parts]
        contiguous = [sum(G * T + 3 * tok[g] for g in range(r * 16 // world, (r + 1) * 16 // world))
                      for r in range(world)]
        assert max(load) <= max(contiguous) + 1e-9


def test_balanced_shard_batch_rows_match_their_groups():
    from invokerl_b200.distributed import balanced_groups

    b = rollout_batch(6, 4, 64, prompt_len=(4, 20), completion_len=(8, 40), seed=9)
    parts = balanced_groups(b.response_mask, 4, 2)
    for r in range(2):
        loc = shard_batch(b, r, 2, balance=True)
        rows = [g * 4 + j for g in parts[r] for j in range(4)]
        assert torch.equal(loc.token_ids, b.token_ids[rows])
        assert torch.equal(loc.response_mask, b.response_mask[rows])
        assert torch.equal(loc.rewards, b.rewards[rows])
        assert loc.group_size == 4


# ---- PPO whitening moments over gloo ranks ----------------------------------------------------


def _moments_worker(rank, world, port, q, counts):
    import datetime

    from invokerl_b200.algorithms import PPO

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(100 + rank)
        x = 3.0 + 2.0 * torch.randn(max(counts) + 5, generator=g)
        m = torch.zeros_like(x, dtype=torch.bool)
        m[: counts[rank]] = True
        xm = x[m]
        n = xm.numel()
        # what ops.masked_moments returns on the device: [mean, unbiased std, count, enabled]
        w = torch.tensor([xm.mean() if n else 0.0, xm.std() if n > 1 else float("nan"), float(n),
                          1.0 if n > 1 else 0.0], dtype=torch.float32)
        out = PPO(row_sharded=True)._global_moments(w)
        alls = [torch.zeros(max(counts) + 5) for _ in counts]
        dist.all_gather(alls, x)
        if rank == 0:
            q.put((out, torch.cat([a[:c] for a, c in zip(alls, counts)])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("counts", [(37, 55), (1, 80), (0, 12), (1, 0)])
def test_ppo_whitening_moments_combine_over_ranks_gloo(counts):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_moments_worker, args=(r, world, port, q, counts)) for r in range(world)]
    for p in procs:
        p.start()
    out, allx = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n = allx.numel()
    assert float(out[2]) == n
    if n > 1:
        assert float(out[3]) == 1.0
        torch.testing.assert_close(out[0], allx.double().mean().float(), rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(out[1], allx.double().std().float(), rtol=1e-5, atol=1e-6)
    else:
        assert float(out[3]) == 0.0


@pytest.mark.parametrize("V,world", [(151936, 1), (151936, 2), (151936, 8), (151936, 3), (5000, 3),
                                     (1000, 7), (777, 8), (8, 4), (64, 8)])
def test_vocab_shard_bounds_cover_the_vocabulary(V, world):
    from invokerl_b200.vocab_parallel import shard_bounds

    bounds = [shard_bounds(V, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == V
    for (s0, e0), (s1, e1) in zip(bounds, bounds[1:]):
        assert e0 == s1
    for s, e in bounds:
        assert s % 8 == 0 and 0 <= s <= e <= V  # 16-byte aligned slices of a bf16 [V, H] weight
    sizes = [e - s for s, e in bounds]
    assert max(sizes) - min(sizes) <= 15
    if V >= 8 * world:
        assert min(sizes) > 0


def test_vocab_parallel_combine_restated():
    """The combine rule of the vocab-parallel forward: logsumexp over the slices' logsumexps and
    the owner's target logit give the unsharded log-prob (restated in torch on the CPU)."""
    from invokerl_b200.vocab_parallel import shard_bounds

    g = torch.Generator().manual_seed(0)
    N, V, P = 37, 1000, 3
    logits = 3 * torch.randn(N, V, generator=g, dtype=torch.float64)
    t = torch.randint(0, V, (N,), generator=g)
    want = torch.log_softmax(logits, dim=1).gather(1, t[:, None]).squeeze(1)
    lse_parts, t_parts = [], []
    for r in range(P):
        s, e = shard_bounds(V, P, r)
        lse_parts.append(torch.logsumexp(logits[:, s:e], dim=1))
        own = (t >= s) & (t < e)
        tl = torch.full((N,), float("-inf"), dtype=torch.float64)
        tl[own] = logits[own, t[own]]
        t_parts.append(tl)
    lse = torch.logsumexp(torch.stack(lse_parts), dim=0)
    got = torch.stack(t_parts).max(dim=0).values - lse
    torch.testing.assert_close(got, want, rtol=0, atol=1e-12)
