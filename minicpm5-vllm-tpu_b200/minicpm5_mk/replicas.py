"""Independent full-weight replicas, one process per GPU (torch.distributed for the plumbing only).

Requests are whole sequences, so a batch shards into contiguous blocks of sequences with no
collective on the data path: each rank runs its block through its own engine (lm_head and argmax
included) and only the (bs,) int32 greedy ids are gathered at the end.  This replaces the reference's
2-core DP mode, which all-gathered last-token hidden rows (`plugin/minicpm5_mk/mk_jax.py:746-753`).
"""

from __future__ import annotations

from typing import Tuple

import torch


def shard_bounds(global_bs: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, count) of rank's contiguous block of sequences; the first global_bs % world ranks take
    one extra sequence."""
    if world < 1 or not 0 <= rank < world or global_bs < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(global_bs, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def gather_tokens(local: torch.Tensor, global_bs: int, group=None) -> torch.Tensor:
    """All ranks' greedy ids (int32, rank order) -> (global_bs,) on every rank.  Blocks are padded to the
    largest block so one all_gather serves uneven splits."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    cap = -(-global_bs // world)
    buf = torch.full((cap,), -1, dtype=torch.int32, device=local.device)
    buf[:local.numel()] = local.to(torch.int32)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    out = []
    for r, p in enumerate(parts):
        _, n = shard_bounds(global_bs, world, r)
        out.append(p[:n])
    return torch.cat(out)
