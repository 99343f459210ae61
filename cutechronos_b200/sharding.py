"""Series-group sharding across ranks (one process per GPU).

Group attention couples only series with the same group id; every other op is
per series.  So a batch splits across ranks by whole groups, each rank runs
the forward on its shard with a full weight replica, and the (B_r, Q, H)
forecasts are gathered.  The only collective is that gather (NCCL on GPUs;
gloo in the CPU tests).
"""

from __future__ import annotations

import torch


def partition_groups(group_ids: torch.Tensor | None, B: int, world: int, tokens_per_series: int = 1):
    """Split series 0..B-1 into `world` shards of whole groups, balanced by
    series count (every series of a forward costs the same).  Returns a list of
    index tensors (int64), one per rank, each sorted; shards may be empty."""
    if group_ids is None:
        group_ids = torch.arange(B)
    gid = torch.as_tensor(group_ids).view(-1).cpu()
    if gid.numel() != B:
        raise ValueError("group_ids must have one entry per series")
    order, seen = [], {}
    for b, g in enumerate(gid.tolist()):
        if g not in seen:
            seen[g] = len(order)
            order.append([])
        order[seen[g]].append(b)
    loads = [0] * world
    shards = [[] for _ in range(world)]
    # largest groups first, each to the least-loaded rank (ties: lowest rank)
    for members in sorted(order, key=lambda m: -len(m)):
        r = min(range(world), key=lambda i: (loads[i], i))
        shards[r].extend(members)
        loads[r] += len(members) * tokens_per_series
    return [torch.tensor(sorted(s), dtype=torch.long) for s in shards]


def gather_forecasts(local: torch.Tensor, shards: list[torch.Tensor], group=None) -> torch.Tensor:
    """All-gather every rank's (B_r, Q, H) forecasts into the original (B, Q, H)
    order.  Shards are padded to the largest for the collective."""
    import torch.distributed as dist

    world = len(shards)
    Bmax = max(1, max(int(s.numel()) for s in shards))
    pad = torch.zeros((Bmax,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    buf = torch.cat(parts, dim=0)
    B = sum(int(s.numel()) for s in shards)
    out = torch.empty((B,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    for r, s in enumerate(shards):
        if s.numel():
            out[s.to(local.device)] = buf[r * Bmax: r * Bmax + s.numel()]
    return out
