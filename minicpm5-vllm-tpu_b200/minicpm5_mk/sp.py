"""Sequence parallelism for batch-1 prefill: one sequence over `world` GPUs (one rank per GPU).

Counterpart of the reference's `core_forward_sp` (plugin/minicpm5_mk/mk_jax.py:440-489), which splits one
sequence over the two TensorCores of a TPU7x chip.  The sequence is cut into blocks; in every group of
2 * world consecutive blocks rank r owns block r and block 2 * world - 1 - r (the reference's
`sp_global_block`, plugin/minicpm5_mk/mk_attn.py:721-724, is the world = 2 case with 512-token blocks).
Early blocks carry little causal attention work and late ones much, so pairing block r with its mirror
balances the ranks.  Each rank runs the projections and MLPs on its own rows and attention for its own
queries; once per layer the ranks all-gather their K/V rows rank by rank (the reference's `unzigzag`
all-gather, mk_jax.py:467-469).

The device side is `mk_forward_sp` (C ABI); this module holds the same block arithmetic as the kernels
(`sp_pos` / `sp_row` in csrc/mk_common.cuh) and the all-gather callbacks the library calls:
  * `nccl_allgather(group)`: torch.distributed all_gather_into_tensor (NCCL over NVLink) on the
    library's stream;
  * `ThreadGroup`: ranks emulated as host threads on one GPU (each with its own stream and engine),
    the gather done with device copies after a host barrier.  No kernel waits on another, so this is
    safe on a single GPU; it is how the zig-zag path is tested without several GPUs.
"""

from __future__ import annotations

import threading
from typing import Callable, List, Optional

import torch

SP_MAX_BLOCK = 512  # the reference's SP_BQ


def sp_block(seq: int, world: int, n_q: int, n_kv: int) -> int:
    """Zig-zag block length (mk_sp_block): the largest of 512..64 with seq % (2 world blk) == 0 that holds
    whole attention query blocks (256 / G rows for G query heads per KV head); 0 if none."""
    if world < 1 or seq <= 0:
        return 0
    min_blk = max(64, 256 // (n_q // n_kv))
    b = SP_MAX_BLOCK
    while b >= min_blk:
        if seq % (2 * world * b) == 0:
            return b
        b //= 2
    return 0


def global_block(i: int, rank: int, world: int) -> int:
    """Sequence block of local block i on `rank` (sp_global_block of the reference for world = 2)."""
    k, j = divmod(i, 2)
    return 2 * world * k + (2 * world - 1 - rank if j else rank)


def sp_pos(row: int, blk: int, rank: int, world: int) -> int:
    """Sequence position of local row `row` (csrc sp_pos)."""
    return global_block(row // blk, rank, world) * blk + row % blk


def sp_row(pos: int, blk: int, world: int, rows_per_rank: int) -> int:
    """Row of sequence position `pos` in the rank-by-rank all-gathered buffer (csrc sp_row)."""
    b = pos // blk
    k, m = divmod(b, 2 * world)
    second = m >= world
    r = 2 * world - 1 - m if second else m
    return r * rows_per_rank + (2 * k + (1 if second else 0)) * blk + pos % blk


def local_positions(seq: int, blk: int, rank: int, world: int) -> torch.Tensor:
    """Positions of a rank's rows, in its storage order (int64 [seq / world])."""
    n = seq // world
    rows = torch.arange(n)
    i = rows // blk
    k, j = i // 2, i % 2
    b = 2 * world * k + torch.where(j == 1, 2 * world - 1 - rank, rank)
    return b * blk + rows % blk


# ------------------------------------------------------------------------------------ collectives
AllGather = Callable[[int, int, int, int], int]  # (send_ptr, recv_ptr, bytes_per_rank, stream) -> status


def _slice(buf: torch.Tensor, ptr: int, nbytes: int) -> torch.Tensor:
    """uint8 view of `nbytes` at device address `ptr` inside `buf` (a uint8 workspace tensor)."""
    off = ptr - buf.data_ptr()
    if off < 0 or off + nbytes > buf.numel():
        raise ValueError("minicpm5_mk: all-gather buffer outside the workspace")
    return buf[off:off + nbytes]


def nccl_allgather(group=None) -> Callable[[torch.Tensor], AllGather]:
    """All-gather through torch.distributed (NCCL): returns a factory taking the rank's workspace.

    torch's NCCL collectives order themselves against torch's current stream, so the gather runs with
    the stream the library passes made current: it then starts after the send rows are written and
    attention (issued after the callback returns) reads the receive rows only after it."""
    import torch.distributed as dist

    def bind(ws: torch.Tensor) -> AllGather:
        world = dist.get_world_size(group)

        def gather(send: int, recv: int, nbytes: int, stream: int) -> int:
            out, inp = _slice(ws, recv, nbytes * world), _slice(ws, send, nbytes)
            if ws.is_cuda and stream and stream != torch.cuda.current_stream(ws.device).cuda_stream:
                with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=ws.device)):
                    dist.all_gather_into_tensor(out, inp, group=group)
            else:
                dist.all_gather_into_tensor(out, inp, group=group)
            return 0

        return gather

    return bind


class ThreadGroup:
    """`world` ranks as host threads sharing one GPU.  Each rank calls `bind(rank, ws, stream)` for its
    callback; a gather waits (on the host) until every rank has reached it, then each rank's stream
    copies every rank's send rows into its own receive buffer after the sender's stream has produced
    them.  A rank that fails breaks the barrier, so the others raise instead of waiting forever."""

    def __init__(self, world: int, timeout_s: float = 120.0):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=timeout_s)
        self.send: List[Optional[torch.Tensor]] = [None] * world
        self.events: List[Optional[torch.cuda.Event]] = [None] * world

    def bind(self, rank: int, ws: torch.Tensor, stream: torch.cuda.Stream) -> AllGather:
        def gather(send: int, recv: int, nbytes: int, stream_ptr: int) -> int:
            ev = torch.cuda.Event()
            ev.record(stream)
            self.send[rank] = _slice(ws, send, nbytes)
            self.events[rank] = ev
            self.barrier.wait()  # every rank's send rows are enqueued
            out = _slice(ws, recv, nbytes * self.world)
            with torch.cuda.stream(stream):
                for r in range(self.world):
                    stream.wait_event(self.events[r])
                    out[r * nbytes:(r + 1) * nbytes].copy_(self.send[r], non_blocking=True)
            done = torch.cuda.Event()
            done.record(stream)
            self.barrier.wait()  # every rank has enqueued its copies (send rows may be reused after these)
            self.events[rank] = done
            self.barrier.wait()
            for r in range(self.world):  # no rank overwrites its send rows before all copies of them ran
                stream.wait_event(self.events[r])
            return 0

        return gather

    def abort(self) -> None:
        self.barrier.abort()
