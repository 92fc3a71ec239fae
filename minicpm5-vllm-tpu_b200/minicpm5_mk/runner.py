"""Host-side batch logic of the fast path (no vLLM import; unit-tested on CPU).

The reference decides per step whether a batch is a set of fresh, equal-length prefills it can run
as one megakernel program (`_mk_seq_ok`, `_eligible_batch`, `plugin/minicpm5_mk/model.py:131-169`)
and returns hidden rows laid out for vLLM's sampler (`scatter_last`, `plugin/minicpm5_mk/mk_jax.py:615-621`).
On the GPU vLLM runner the batch shape comes from the forward context's attention metadata
(`query_start_loc`, `seq_lens`).
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch


def mk_seq_ok(seq: int, max_seq: int) -> bool:
    """Lengths the fast path serves (`plugin/minicpm5_mk/model.py:131-136`): multiples of 128 up to
    1024, multiples of 1024 above, and at most max_seq."""
    if seq <= 0 or seq > max_seq:
        return False
    if seq <= 1024:
        return seq % 128 == 0
    return seq % 1024 == 0


def batch_from_lengths(query_lens: Sequence[int], seq_lens: Sequence[int], max_seq: int,
                       num_tokens: int) -> Tuple[Optional[Tuple[int, int]], str]:
    """(bs, seq) if every request is a fresh prefill (no cached context) of the same eligible length
    and the step holds exactly those tokens; else (None, reason)."""
    if not query_lens:
        return None, "empty"
    if len(query_lens) != len(seq_lens):
        return None, "metadata"
    if any(int(q) != int(s) for q, s in zip(query_lens, seq_lens)):
        return None, "not-fresh"
    s0 = int(query_lens[0])
    if any(int(q) != s0 for q in query_lens):
        return None, "unequal"
    if not mk_seq_ok(s0, max_seq):
        return None, "length"
    bs = len(query_lens)
    if bs * s0 > num_tokens:
        return None, "tokens"
    return (bs, s0), "ok"


def scatter_last(h: torch.Tensor, bs: int, seq: int, t_pad: int) -> torch.Tensor:
    """(bs, H) -> (t_pad, H) with h[b] at row b*seq + seq - 1 and zeros elsewhere
    (`scatter_last`, plugin/minicpm5_mk/mk_jax.py:615-621)."""
    out = torch.zeros((t_pad, h.shape[-1]), dtype=h.dtype, device=h.device)
    rows = torch.arange(bs, device=h.device) * seq + (seq - 1)
    out[rows] = h
    return out


class LastRowScatter:
    """`scatter_last` into one reused (rows, H) buffer instead of a fresh zero-filled tensor per step
    (805 MB for a 32 x 8192 step at H 1536).  Each call zeroes only the rows the previous call wrote, then
    writes this call's last-token rows, so the returned (t_pad, H) view holds zeros everywhere else, as
    `scatter_last` does.  The buffer grows (once) when a step has more tokens than it holds.  The view
    stays valid until the next call, which is all vLLM's runner needs: it gathers the sampled rows
    (`hidden_states[logits_indices]`) before the next forward."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None
        self.prev_rows: Optional[torch.Tensor] = None

    def __call__(self, h: torch.Tensor, bs: int, seq: int, t_pad: int) -> torch.Tensor:
        buf = self.buf
        if buf is None or buf.shape[0] < t_pad or buf.shape[1] != h.shape[-1] or buf.dtype != h.dtype \
                or buf.device != h.device:
            buf = self.buf = None
            buf = torch.zeros((t_pad, h.shape[-1]), dtype=h.dtype, device=h.device)
            self.buf, self.prev_rows = buf, None
        if self.prev_rows is not None:
            buf.index_fill_(0, self.prev_rows, 0)
        rows = torch.arange(bs, device=h.device) * seq + (seq - 1)
        buf.index_copy_(0, rows, h[:bs])
        self.prev_rows = rows
        return buf[:t_pad]
