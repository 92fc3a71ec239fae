"""Minimal numpy stand-in for the handful of jax calls made by the reference's
`benchmark/f32_golden.py` (jax is not installed in this image).

Used only by `tests/golden/make_golden.py` to run the reference's own `forward_one` on small
random-init models and record golden fixtures.  Every function keeps float32 arithmetic, like the
reference's `Precision.HIGHEST` f32 path.
"""
import types

import numpy as _np

from . import numpy  # noqa: F401  (jax.numpy)


class _Config:
    def update(self, *_a, **_k):
        return None


config = _Config()


def jit(fn=None, **_kw):
    if fn is None:
        return lambda f: f
    return fn


def _rsqrt(x):
    return (1.0 / _np.sqrt(x)).astype(_np.float32)


def _top_k(x, k):
    x = _np.asarray(x)
    idx = _np.argsort(-x, kind="stable")[:k]
    return x[idx], idx


class _Precision:
    HIGHEST = "highest"
    DEFAULT = "default"


lax = types.SimpleNamespace(rsqrt=_rsqrt, top_k=_top_k, Precision=_Precision)


def _softmax(x, axis=-1):
    x = _np.asarray(x, dtype=_np.float32)
    m = _np.max(x, axis=axis, keepdims=True)
    e = _np.exp(x - m)
    return (e / _np.sum(e, axis=axis, keepdims=True)).astype(_np.float32)


def _log_softmax(x, axis=-1):
    x = _np.asarray(x, dtype=_np.float32)
    m = _np.max(x, axis=axis, keepdims=True)
    s = x - m
    return (s - _np.log(_np.sum(_np.exp(s), axis=axis, keepdims=True))).astype(_np.float32)


def _silu(x):
    x = _np.asarray(x, dtype=_np.float32)
    return (x / (1.0 + _np.exp(-x))).astype(_np.float32)


nn = types.SimpleNamespace(softmax=_softmax, log_softmax=_log_softmax, silu=_silu)
