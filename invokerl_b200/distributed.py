"""Row sharding of the hot path across ranks (one process per GPU).

invokerl replicates every RolloutBatch on every rank (invokerl/distributed.py:236-302,
invokerl/trainer.py:131-140).  Here each rank takes whole prompt groups — G contiguous rows,
the layout of ``group_ids = arange(B/G).repeat_interleave(G)`` (trainer.py:317) — so group
advantages need no communication.  The only collectives of the path are the all-reduce of the
response-token count before the loss and of the metric sums after it (``algorithms.base``).
"""

from __future__ import annotations

import torch

from .algorithms.base import RolloutBatch


def group_shard_bounds(B: int, G: int, rank: int, world: int) -> tuple[int, int]:
    """Row range [start, end) of `rank`: whole groups, as even as possible, contiguous."""
    if G <= 0 or B % G:
        raise ValueError(f"B={B} is not a multiple of group_size={G}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    ngroups = B // G
    base, extra = divmod(ngroups, world)
    g0 = rank * base + min(rank, extra)
    g1 = g0 + base + (1 if rank < extra else 0)
    return g0 * G, g1 * G


def balanced_groups(response_mask: torch.Tensor, G: int, world: int, row_cost: float = 1.0,
                    token_cost: float = 3.0) -> list[list[int]]:
    """Whole groups per rank, balanced by estimated work instead of by count.

    A group costs `row_cost` per row (the LM-head forward runs every row) plus `token_cost` per
    response token (the backward runs only rows with a nonzero upstream gradient; 3 = its three
    GEMMs against the forward's one).  Groups are placed largest first on the least-loaded rank
    (ties: lower rank), then single moves and swaps off the most loaded rank are applied while
    they lower its load; each rank's groups are returned in increasing order.  Deterministic, so
    every rank computes the same assignment from the same masks."""
    B, T = response_mask.shape
    if G <= 0 or B % G:
        raise ValueError(f"B={B} is not a multiple of group_size={G}")
    ngroups = B // G
    tok = response_mask.reshape(ngroups, G * T).sum(dim=1).tolist()
    cost = [row_cost * G * T + token_cost * t for t in tok]
    order = sorted(range(ngroups), key=lambda g: (-cost[g], g))
    load = [0.0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for g in order:
        r = min(range(world), key=lambda q: (load[q], q))
        out[r].append(g)
        load[r] += cost[g]
    # Local search: move or swap a group between the most loaded rank and another while that lowers
    # the larger of the two loads.
    for _ in range(4 * ngroups):
        hi = max(range(world), key=lambda q: (load[q], -q))
        best = None
        for lo in range(world):
            if lo == hi:
                continue
            for g in out[hi]:
                cand = [(max(load[hi] - cost[g], load[lo] + cost[g]), g, None)]
                cand += [(max(load[hi] - cost[g] + cost[h], load[lo] - cost[h] + cost[g]), g, h) for h in out[lo]]
                for m, a, b in cand:
                    if m < load[hi] - 1e-9 and (best is None or m < best[0]):
                        best = (m, lo, a, b)
        if best is None:
            break
        _, lo, a, b = best
        out[hi].remove(a)
        out[lo].append(a)
        load[hi] -= cost[a]
        load[lo] += cost[a]
        if b is not None:
            out[lo].remove(b)
            out[hi].append(b)
            load[lo] -= cost[b]
            load[hi] += cost[b]
    return [sorted(x) for x in out]


def shard_rows(x, start: int, end: int, B: int):
    if isinstance(x, torch.Tensor) and x.dim() >= 1 and x.shape[0] == B:
        return x[start:end]
    return x


def shard_batch(batch: RolloutBatch, rank: int, world: int, balance: bool = False) -> RolloutBatch:
    """This rank's whole groups of `batch`: contiguous (views, no copies), or with balance=True the
    groups `balanced_groups` assigns to it (copies, in group order)."""
    B = batch.token_ids.shape[0]
    if balance:
        G = batch.group_size
        groups = balanced_groups(batch.response_mask, G, world)[rank]
        idx = torch.tensor([g * G + j for g in groups for j in range(G)], dtype=torch.long)

        def take(x):
            if isinstance(x, torch.Tensor) and x.dim() >= 1 and x.shape[0] == B:
                return x.index_select(0, idx.to(x.device))
            return x

        return RolloutBatch(
            token_ids=take(batch.token_ids), prompt_mask=take(batch.prompt_mask),
            response_mask=take(batch.response_mask), attention_mask=take(batch.attention_mask),
            rewards=take(batch.rewards), token_rewards=take(batch.token_rewards),
            old_log_probs=take(batch.old_log_probs), ref_log_probs=take(batch.ref_log_probs),
            group_ids=take(batch.group_ids), group_size=G, weight_version=batch.weight_version,
            extras={k: take(v) for k, v in batch.extras.items()},
        )
    s, e = group_shard_bounds(B, batch.group_size, rank, world)
    return RolloutBatch(
        token_ids=batch.token_ids[s:e],
        prompt_mask=batch.prompt_mask[s:e],
        response_mask=batch.response_mask[s:e],
        attention_mask=batch.attention_mask[s:e],
        rewards=batch.rewards[s:e],
        token_rewards=None if batch.token_rewards is None else batch.token_rewards[s:e],
        old_log_probs=batch.old_log_probs[s:e],
        ref_log_probs=batch.ref_log_probs[s:e],
        group_ids=None if batch.group_ids is None else batch.group_ids[s:e],
        group_size=batch.group_size,
        weight_version=batch.weight_version,
        extras={k: shard_rows(v, s, e, B) for k, v in batch.extras.items()},
    )


def scatter_batch(batch: RolloutBatch | None, src: int = 0, group=None,
                  device: torch.device | str | None = None, balance: bool = True) -> RolloutBatch:
    """Give every rank its whole prompt groups of the batch held by rank `src`.

    Replaces the replicate-everything `broadcast_batch` of invokerl/distributed.py:236-330.  Rank
    `src` chooses the groups of every rank -- by estimated work (`balanced_groups`, the assignment
    `shard_batch(..., balance=True)` makes) or, with balance=False, contiguous ranges -- and
    broadcasts that plan with the metadata (field shapes, dtypes, group size, extras layout) as a
    small object.  Then one all-to-all moves every row field at once: `src` packs each rank's rows
    of all fields into one byte block, and every rank receives only its own block, so each byte of
    the batch crosses the network once instead of world_size - 1 times.  A rank's rows come in the
    order of its groups.  Tensors whose leading dimension is B are sharded; other tensors and
    non-tensor extras are broadcast whole.  Collective over `group`."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    src_global = dist.get_global_rank(group, src) if group is not None else src
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"

    fields = ["token_ids", "prompt_mask", "response_mask", "attention_mask", "rewards", "token_rewards",
              "old_log_probs", "ref_log_probs", "group_ids"]
    if rank == src:
        B = batch.token_ids.shape[0]
        G = batch.group_size
        if balance:
            plan = balanced_groups(batch.response_mask, G, world)
        else:
            plan = []
            for r in range(world):
                s0, e0 = group_shard_bounds(B, G, r, world)
                plan.append(list(range(s0 // G, e0 // G)))
        meta = {"B": B, "G": G, "weight_version": batch.weight_version, "plan": plan, "rows": [], "extras": {},
                "extras_order": list(batch.extras)}
        for f in fields:
            t = getattr(batch, f)
            meta["rows"].append((f, None if t is None else (tuple(t.shape), t.dtype)))
        for k, v in batch.extras.items():
            if isinstance(v, torch.Tensor):
                if v.dim() >= 1 and v.shape[0] == B:
                    meta["rows"].append(("extras." + k, (tuple(v.shape), v.dtype)))
                else:
                    meta["extras"][k] = ("whole", tuple(v.shape), v.dtype)
            else:
                meta["extras"][k] = ("object", v, None)
        obj = [meta]
    else:
        obj = [None]
    dist.broadcast_object_list(obj, src=src_global, group=group)
    meta = obj[0]
    G, plan = meta["G"], meta["plan"]
    row_fields = [(name, m) for name, m in meta["rows"] if m is not None]

    def row_bytes(shape, dtype) -> int:
        n = 1
        for d in shape[1:]:
            n *= d
        return n * torch.empty((), dtype=dtype).element_size()

    def padded(n: int) -> int:  # keep every field's bytes 8-byte aligned inside a block
        return (n + 7) // 8 * 8

    def block_bytes(nrows: int) -> int:
        return sum(padded(nrows * row_bytes(*m)) for _, m in row_fields)

    rows_of = [len(p) * G for p in plan]
    if rank == src:
        def get(name):
            return batch.extras[name[7:]] if name.startswith("extras.") else getattr(batch, name)

        parts = []
        for r in range(world):
            idx = torch.tensor([g * G + j for g in plan[r] for j in range(G)], dtype=torch.long)
            for name, (shape, dtype) in row_fields:
                t = get(name)
                x = t.index_select(0, idx.to(t.device)).contiguous()
                b = x.view(torch.uint8).reshape(-1)
                pad = padded(b.numel()) - b.numel()
                parts.append(b.to(device))
                if pad:
                    parts.append(torch.zeros(pad, dtype=torch.uint8, device=device))
        send = torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=device)
        in_splits = [block_bytes(rows_of[r]) for r in range(world)]
    else:
        send = torch.empty(0, dtype=torch.uint8, device=device)
        in_splits = [0] * world
    mine = block_bytes(rows_of[rank])
    recv = torch.empty(mine, dtype=torch.uint8, device=device)
    out_splits = [mine if q == src else 0 for q in range(world)]
    dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)

    vals: dict = {f: None for f in fields}
    extras = {}
    off = 0
    nr = rows_of[rank]
    for name, (shape, dtype) in row_fields:
        nb = nr * row_bytes(shape, dtype)
        t = recv[off:off + nb].view(dtype).reshape((nr,) + tuple(shape[1:]))
        off += padded(nb)
        if name.startswith("extras."):
            extras[name[7:]] = t
        else:
            vals[name] = t
    for k, (kind, a, b) in meta["extras"].items():
        if kind == "object":
            extras[k] = a
        else:
            out = batch.extras[k].contiguous().to(device) if rank == src else torch.empty(a, dtype=b, device=device)
            dist.broadcast(out, src=src_global, group=group)
            extras[k] = out
    extras = {k: extras[k] for k in meta["extras_order"]}
    return RolloutBatch(**vals, group_size=G, weight_version=meta["weight_version"], extras=extras)
