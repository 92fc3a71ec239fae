"""`torch.ops.minicpm5_mk.forward`: the whole-model prefill-score op as a registered torch custom op.

The reference reaches its device program through one registered op, `jax_op("minicpm5_mk::forward",
mk_forward)` (`plugin/minicpm5_mk/model.py:57-66`), called from `_mk_call` (`model.py:737-753`) with the
ids, every weight tensor and the static sizes.  Here the weights are bound once to a library handle
(`MkEngine`, `mk_bind_weights`), so the op takes the ids, the engine's id in this process's registry
and (bs, seq), and returns what the library's `mk_forward` writes: the final-normed last-token hidden
rows (bs, H) bf16, the last-token logits (bs, V) f32 and the greedy ids (bs,) int32.

The op is registered for CUDA only: on any other device it raises (there is no CPU fallback).  Its fake
(meta) implementation gives torch.compile / FakeTensor tracing the output shapes, so a traced caller
sees an opaque op instead of graph-breaking on ctypes.
"""

from __future__ import annotations

import itertools
import threading
from typing import Dict, Tuple

import torch

_ENGINES: Dict[int, object] = {}
_IDS = itertools.count(1)
_LOCK = threading.Lock()


def register_engine(engine) -> int:
    """Make an `MkEngine` reachable from the op; returns its id (the op's `engine` argument)."""
    with _LOCK:
        i = next(_IDS)
        _ENGINES[i] = engine
    return i


def unregister_engine(engine_id: int) -> None:
    with _LOCK:
        _ENGINES.pop(int(engine_id), None)


def _engine(engine_id: int):
    try:
        return _ENGINES[int(engine_id)]
    except KeyError:
        raise RuntimeError(f"minicpm5_mk: no engine registered under id {engine_id}") from None


@torch.library.custom_op("minicpm5_mk::forward", mutates_args=(), device_types="cuda")
def forward(ids: torch.Tensor, engine: int, bs: int, seq: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """ids int32 [bs * seq] (sequence-major) on the engine's device -> (hidden, logits, top1)."""
    hid, lg, top1 = _engine(engine).forward(ids, bs, seq)
    return hid, lg, top1


@forward.register_fake
def _forward_fake(ids: torch.Tensor, engine: int, bs: int, seq: int):
    cfg = _engine(engine).cfg
    return (ids.new_empty((bs, cfg.hidden), dtype=torch.bfloat16),
            ids.new_empty((bs, cfg.vocab), dtype=torch.float32),
            ids.new_empty((bs,), dtype=torch.int32))
