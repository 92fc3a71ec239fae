"""The softmax's FMA-pipe exponential (`exp2_fma` in csrc/mk_attn_tc.cuh): range reduction to
x = j + f, f in [-0.5, 0.5], and a least-squares cubic for 2^f.  Replayed here in float32 with the
coefficients read from the header, against float64 2^x: the relative error must stay well below the
bf16 rounding (2^-9) that P gets right after."""
import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(__file__), "..", "minicpm5-vllm-tpu_b200", "csrc", "mk_attn_tc.cuh")


def _coefficients():
    src = open(HDR).read()
    body = src[src.index("float exp2_fma(float x)"):]
    body = body[:body.index("}")]
    c = [float(v) for v in re.findall(r"([0-9]\.[0-9]+)f", body)]
    assert len(c) == 4, c
    return [np.float32(v) for v in c]  # c3, c2, c1, c0 in Horner order


def _exp2_fma(x):
    c3, c2, c1, c0 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic)).astype(np.float32)
    p = ((c3 * f + c2) * f + c1) * f + c0  # float32 Horner (the kernel fuses each step; error is far smaller)
    bits = p.astype(np.float32).view(np.int32) + (t.view(np.int32) << 23)
    return bits.view(np.float32)


def test_exp2_fma_relative_error():
    x = np.linspace(-40.0, 8.0, 2_000_001, dtype=np.float32)
    got = _exp2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 1.2e-4, rel.max()  # the fit's 7.8e-5 plus float32 rounding; bf16 half-ulp is 2^-9


def test_exp2_fma_clamps_and_masks():
    got = _exp2_fma(np.array([-np.inf, -1e9, -125.0, -130.0], dtype=np.float32))
    assert np.all(got >= 0) and np.all(got < 1e-37), got
    assert np.all(np.isfinite(got))
