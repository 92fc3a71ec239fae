"""numpy stand-in for `jax.numpy` (see the package docstring)."""
import numpy as _np

float32 = _np.float32
int32 = _np.int32
bfloat16 = None
inf = _np.inf


def asarray(a, dtype=None):
    return _np.asarray(a, dtype=dtype)


def mean(x, axis=None, keepdims=False):
    return _np.mean(x, axis=axis, keepdims=keepdims, dtype=_np.float32)


def concatenate(xs, axis=0):
    return _np.concatenate(xs, axis=axis)


def einsum(eq, *ops, precision=None, preferred_element_type=None):
    return _np.einsum(eq, *[_np.asarray(o, dtype=_np.float32) for o in ops], optimize=True).astype(_np.float32)


def dot(a, b, precision=None, preferred_element_type=None):
    return _np.dot(_np.asarray(a, dtype=_np.float32), _np.asarray(b, dtype=_np.float32)).astype(_np.float32)


def arange(*a, **k):
    return _np.arange(*a, **k)


def where(c, a, b):
    return _np.where(c, a, b).astype(_np.float32)
