"""The allocation-free lm_head entry point (mk_lm_head_argmax_noalloc) against the regular one.

Some callers cannot allocate device memory when they call into the library -- a serving engine that has
reserved nearly the whole GPU for weights and KV cache, or a host runtime reaching the library through
a thin FFI with no access to the framework's allocator.  For them the library keeps the lm_head's argmax
partials in a fixed device array of its own.  This file checks, through the C ABI, that two calls in a
row give exactly the logits and greedy ids of mk_lm_head_argmax (which uses caller-provided scratch),
and that a batch above the fixed capacity is refused.  It is collected last so that a stop-at-first-
failure run has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ROWS = 64  # MK_LM_HEAD_NOALLOC_MAX_ROWS in include/minicpm5_mk.h


def _with_scratch(L, h, w, stream):
    bs, H = h.shape
    V = w.shape[0]
    P = L.mk_lm_head_parts()
    logits = torch.empty((bs, V), dtype=torch.float32, device=h.device)
    pv = torch.empty((bs, P), dtype=torch.float32, device=h.device)
    pi = torch.empty((bs, P), dtype=torch.int32, device=h.device)
    top1 = torch.empty((bs,), dtype=torch.int32, device=h.device)
    st = L.mk_lm_head_argmax(h.data_ptr(), bs, H, w.data_ptr(), V, logits.data_ptr(), pv.data_ptr(),
                             pi.data_ptr(), top1.data_ptr(), stream)
    assert st == 0, st
    return logits, top1


def _no_alloc(L, h, w, stream):
    bs, H = h.shape
    V = w.shape[0]
    logits = torch.full((bs, V), float("nan"), dtype=torch.float32, device=h.device)
    top1 = torch.full((bs,), -1, dtype=torch.int32, device=h.device)
    st = L.mk_lm_head_argmax_noalloc(h.data_ptr(), bs, H, w.data_ptr(), V, logits.data_ptr(),
                                     top1.data_ptr(), stream)
    assert st == 0, st
    return logits, top1


def test_no_alloc_lm_head_matches_scratch_version_on_two_calls():
    from minicpm5_mk import _lib

    assert torch.cuda.is_available()
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(2024)
    cases = [(MAX_ROWS, 1536, 73448), (3, 384, 1000)]  # two calls in a row, the first at full capacity
    for bs, H, V in cases:
        h = torch.randn((bs, H), generator=g, device=dev)
        w = (torch.randn((V, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        lg_ref, t_ref = _with_scratch(L, h, w, stream)
        lg, t = _no_alloc(L, h, w, stream)
        torch.cuda.synchronize()
        # same kernels, same inputs: identical results (tolerance of the other lm_head tests: exact ids)
        assert torch.equal(lg, lg_ref)
        assert torch.equal(t, t_ref)
        assert torch.equal(t.long(), torch.argmax(lg, dim=-1))
    e = ctypes.c_int32()
    assert L.mk_get_error(None, ctypes.byref(e)) == 0 and e.value == 0


def test_no_alloc_lm_head_rejects_batches_above_capacity():
    from minicpm5_mk import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    h = torch.zeros((MAX_ROWS + 1, 384), device=dev)
    w = torch.zeros((1000, 384), dtype=torch.bfloat16, device=dev)
    lg = torch.empty((MAX_ROWS + 1, 1000), device=dev)
    t = torch.empty((MAX_ROWS + 1,), dtype=torch.int32, device=dev)
    st = L.mk_lm_head_argmax_noalloc(h.data_ptr(), MAX_ROWS + 1, 384, w.data_ptr(), 1000, lg.data_ptr(),
                                     t.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert st == 9  # MK_ERR_TOO_LARGE
    assert L.mk_status_string(st) == b"request exceeds a fixed library capacity"
