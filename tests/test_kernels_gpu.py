"""Per-kernel parity on a B200: each CUDA entry point of the C ABI against a plain PyTorch fp32
reference of the same op on the same (seeded) inputs."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from minicpm5_mk import _lib
    _lib.lib()
    return torch.device("cuda", 0)


def _gen(seed):
    return torch.Generator(device="cpu").manual_seed(seed)


def _rand(shape, seed, scale=1.0):
    return torch.randn(shape, generator=_gen(seed)) * scale


def _quant(w):
    from minicpm5_mk.mk_weights import quantize_per_out_channel
    return quantize_per_out_channel(w)


def _check_err():
    from minicpm5_mk import _lib
    import ctypes
    e = ctypes.c_int32()
    st = _lib.lib().mk_get_error(None, ctypes.byref(e))
    assert st == 0 and e.value == 0, (st, hex(e.value))


GEMM_CASES = [
    # M, K, N
    (8192, 1536, 1792),  # BASELINE's isolated QKV shape
    (128, 64, 256),
    (256, 128, 384),
    (300, 192, 256),
    (2048, 1536, 1920),
    (8192, 1536, 1536),
    (1000, 4096, 1536),
    (5, 1536, 1536),
]


@pytest.mark.parametrize("M,K,N", GEMM_CASES)
@pytest.mark.parametrize("mode", ["colscale", "rowscale", "resid", "resid32"])
def test_gemm_w8a16(dev, M, K, N, mode):
    from minicpm5_mk import ops, _lib
    a = _rand((M, K), 1 + M + K).to(torch.bfloat16)
    w8, s = _quant(_rand((N, K), 2 + N, 0.02))
    rstd = torch.rand((M,), generator=_gen(3)) + 0.5
    acc = a.float() @ w8.float().T
    ad, wd, sd, rd = a.to(dev), w8.to(dev), s.to(dev), rstd.to(dev)
    if mode == "colscale":
        out = ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_COLSCALE)
        ref = acc * s
    elif mode == "rowscale":
        out = ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_ROWSCALE, row_scale=rd)
        ref = acc * rstd[:, None] * s
    elif mode == "resid":
        x0 = _rand((M, N), 9).to(torch.bfloat16)
        out = x0.to(dev).clone()
        ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_RESID, resid_scale=0.3, out=out)
        ref = x0.float() + 0.3 * acc * s
    else:
        x0 = _rand((M, N), 9)
        x32 = x0.to(dev).clone()
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_RESID32, resid_scale=0.3, out=out, resid32=x32)
        ref = x0 + 0.3 * acc * s
        torch.cuda.synchronize()
        assert (x32.cpu() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-5
        assert torch.equal(out.cpu(), x32.cpu().to(torch.bfloat16))
    torch.cuda.synchronize()
    _check_err()
    got = out.float().cpu()
    tol = 1e-2 * ref.abs().max().item() + 1e-3
    err = (got - ref).abs().max().item()
    assert err <= tol, (err, tol)
    # bf16 output: almost every element within 1 bf16 ulp of the f32 reference
    rel = ((got - ref).abs() / (ref.abs() + 1e-3)).flatten()
    assert (rel > 1.6e-2).float().mean().item() < 1e-3


@pytest.mark.parametrize("M,K,N", [(8192, 1536, 1792), (300, 192, 256), (1000, 4096, 1536), (5, 1536, 1536)])
@pytest.mark.parametrize("mode", ["rowscale", "resid32", "swiglu"])
def test_gemm_bf16_weights(dev, M, K, N, mode):
    """The same GEMM with unquantised bf16 weights (weight_bits 16): the weight tiles are copied into the
    TMEM operand unchanged, against a plain PyTorch fp32 reference."""
    from minicpm5_mk import ops, _lib
    a = _rand((M, K), 101 + M).to(torch.bfloat16)
    w = _rand((N, K), 102 + N, 0.02).to(torch.bfloat16)
    s = torch.ones(N)
    rstd = torch.rand((M,), generator=_gen(103)) + 0.5
    acc = a.float() @ w.float().T
    ad, wd, sd, rd = a.to(dev), w.to(dev), s.to(dev), rstd.to(dev)
    if mode == "rowscale":
        out = ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_ROWSCALE, row_scale=rd)
        ref = acc * rstd[:, None]
    elif mode == "swiglu":
        out = ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_SWIGLU, row_scale=rd)
        g, u = acc[:, 0::2] * rstd[:, None], acc[:, 1::2] * rstd[:, None]
        ref = torch.nn.functional.silu(g) * u
    else:
        x0 = _rand((M, N), 104)
        x32 = x0.to(dev).clone()
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        ops.gemm_w8a16(ad, wd, sd, _lib.MK_GEMM_RESID32, resid_scale=0.3, out=out, resid32=x32)
        ref = x0 + 0.3 * acc
        torch.cuda.synchronize()
        assert (x32.cpu() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-5
    torch.cuda.synchronize()
    _check_err()
    got = out.float().cpu()
    assert (got - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


def _rope_pairs_ref(x, cos, sin, rope_cols, hd, pos):
    """Pair-ordered RoPE: columns (2j, 2j+1) of each head are the rotation pair (j, j + hd/2) at the
    angle index (column % hd) / 2 of position pos[m]."""
    out = x.clone()
    pj = (torch.arange(0, rope_cols, 2) % hd) // 2
    c, s = cos[pos][:, pj], sin[pos][:, pj]
    a, b = x[:, 0:rope_cols:2], x[:, 1:rope_cols:2]
    out[:, 0:rope_cols:2] = a * c - b * s
    out[:, 1:rope_cols:2] = b * c + a * s
    return out


def _close_bf16(got, ref, what):
    scale = ref.abs().max().item()
    err = (got - ref).abs()
    bad = err > 8e-3 * ref.abs() + 2e-3 * scale
    assert not bad.any(), (what, err.max().item(), scale, int(bad.sum()))


FUSED_CASES = [
    # M, K, N, head_dim, rope_cols, rope_seq, pos_base: the BASELINE isolated QKV shape (N 1792) with
    # hd-128 heads; the 1B QKV width (1920, hd 96: Q+K heads rotated, V not) at a ragged M of two
    # 4096-token sequences plus a tail; positions that wrap inside 32-token chunks (rope_seq 100)
    (8192, 1536, 1792, 128, 1536, 8192, 0),
    (8111, 1536, 1920, 96, 1728, 4096, 0),
    (333, 128, 256, 128, 256, 100, 7),
]


@pytest.mark.parametrize("M,K,N,hd,rope_cols,rope_seq,pos_base", FUSED_CASES)
def test_gemm_norm_rope_epilogue(dev, M, K, N, hd, rope_cols, rope_seq, pos_base):
    """The QKV projection's fused epilogue in isolation (mk_gemm_w8a16_fused, ROWSCALE): rstd from the
    per-(token, 128-channel tile) sums of squares, the per-channel scale, then RoPE on the pair-ordered
    Q/K columns (positions advanced by the angle-addition recurrence) -- against a plain PyTorch fp32
    reference on the same inputs."""
    from minicpm5_mk import ops, _lib
    from minicpm5_mk.mk_weights import rope_tables
    a = _rand((M, K), 71 + M).to(torch.bfloat16)
    w8, s = _quant(_rand((N, K), 72 + N, 0.02))
    npart = 12
    rowsq = torch.rand((M, npart), generator=_gen(73)) * 300.0 + 1.0
    eps = 1e-6
    rstd = torch.rsqrt(rowsq.sum(-1) / 1536.0 + eps)
    cos, sin = rope_tables(max(rope_seq + pos_base, 64), hd, 10000.0)
    acc = (a.float() @ w8.float().T) * rstd[:, None] * s
    pos = torch.arange(M) % rope_seq + pos_base
    ref = _rope_pairs_ref(acc, cos, sin, rope_cols, hd, pos)
    out = ops.gemm_w8a16(a.to(dev), w8.to(dev), s.to(dev), _lib.MK_GEMM_ROWSCALE, rowsq=rowsq.to(dev),
                         rowsq_np=npart, norm_dim=1536, eps=eps, rope=(cos.to(dev), sin.to(dev)),
                         rope_cols=rope_cols, head_dim=hd, rope_seq=rope_seq, rope_pos_base=pos_base)
    torch.cuda.synchronize()
    _check_err()
    _close_bf16(out.float().cpu(), ref, "norm+rope")


def test_gemm_swiglu_norm_epilogue(dev):
    """Gate/up with rstd taken from the sums-of-squares partials (the forward's fused post-attention
    RMSNorm) at a ragged M."""
    from minicpm5_mk import ops, _lib
    from minicpm5_mk.mk_weights import interleave_gu
    M, K, I = 1001, 1536, 4608
    a = _rand((M, K), 81).to(torch.bfloat16)
    g8, sg = _quant(_rand((I, K), 82, 0.05))
    u8, su = _quant(_rand((I, K), 83, 0.05))
    rowsq = torch.rand((M, 12), generator=_gen(84)) * 200.0 + 1.0
    rstd = torch.rsqrt(rowsq.sum(-1) / 1536.0 + 1e-6)
    g = (a.float() @ g8.float().T) * rstd[:, None] * sg
    u = (a.float() @ u8.float().T) * rstd[:, None] * su
    ref = torch.nn.functional.silu(g) * u
    out = ops.gemm_w8a16(a.to(dev), interleave_gu(g8, u8).to(dev), interleave_gu(sg, su).to(dev),
                         _lib.MK_GEMM_SWIGLU, rowsq=rowsq.to(dev), rowsq_np=12, norm_dim=1536, eps=1e-6)
    torch.cuda.synchronize()
    _check_err()
    got = out.float().cpu()
    assert (got - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("M,K", [(8111, 1536), (8192, 4608)])
def test_gemm_resid32_writes_norm_statistics(dev, M, K):
    """o_proj / down (RESID32) update the f32 residual and write each token's sum of squares per
    128-channel tile -- the statistics the next projection's RMSNorm reads."""
    from minicpm5_mk import ops, _lib
    N = 1536
    a = _rand((M, K), 91 + K).to(torch.bfloat16)
    w8, s = _quant(_rand((N, K), 92, 0.02))
    x0 = _rand((M, N), 93)
    ref = x0 + 0.29 * (a.float() @ w8.float().T) * s
    x32 = x0.to(dev).clone()
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    rowsq = torch.full((M, 16), -1.0, device=dev)  # 12 tiles written, the rest untouched
    ops.gemm_w8a16(a.to(dev), w8.to(dev), s.to(dev), _lib.MK_GEMM_RESID32, resid_scale=0.29, out=out,
                   resid32=x32, rowsq=rowsq)
    torch.cuda.synchronize()
    _check_err()
    x = x32.cpu()
    assert (x - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-5
    assert torch.equal(out.cpu(), x.to(torch.bfloat16))
    sq = rowsq.cpu()
    ref_sq = x.double().pow(2).reshape(M, N // 128, 128).sum(-1)
    assert torch.allclose(sq[:, :N // 128].double(), ref_sq, rtol=1e-5, atol=1e-4)
    assert torch.equal(sq[:, N // 128:], torch.full((M, 16 - N // 128), -1.0))


@pytest.mark.parametrize("M,K,I", [(256, 128, 128), (777, 384, 512), (4096, 1536, 4608)])
def test_gemm_swiglu(dev, M, K, I):
    from minicpm5_mk import ops, _lib
    from minicpm5_mk.mk_weights import interleave_gu
    a = _rand((M, K), 11).to(torch.bfloat16)
    g8, sg = _quant(_rand((I, K), 12, 0.05))
    u8, su = _quant(_rand((I, K), 13, 0.05))
    w8, s = interleave_gu(g8, u8), interleave_gu(sg, su)
    rstd = torch.rand((M,), generator=_gen(14)) + 0.5
    g = (a.float() @ g8.float().T) * rstd[:, None] * sg
    u = (a.float() @ u8.float().T) * rstd[:, None] * su
    ref = torch.nn.functional.silu(g) * u
    out = ops.gemm_w8a16(a.to(dev), w8.to(dev), s.to(dev), _lib.MK_GEMM_SWIGLU, row_scale=rstd.to(dev))
    torch.cuda.synchronize()
    _check_err()
    got = out.float().cpu()
    assert got.shape == (M, I)
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


def _attn_ref(qkv, bs, S, nq, nkv, hd, scale):
    q = qkv[:, :nq * hd].float().reshape(bs, S, nq, hd).permute(0, 2, 1, 3)
    k = qkv[:, nq * hd:(nq + nkv) * hd].float().reshape(bs, S, nkv, hd).permute(0, 2, 1, 3)
    v = qkv[:, (nq + nkv) * hd:].float().reshape(bs, S, nkv, hd).permute(0, 2, 1, 3)
    G = nq // nkv
    k = k.repeat_interleave(G, dim=1)
    v = v.repeat_interleave(G, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * scale
    mask = torch.ones(S, S, dtype=torch.bool).tril()
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v)
    return o.permute(0, 2, 1, 3).reshape(bs * S, nq * hd)


@pytest.mark.parametrize("bs,S,nq,nkv,hd", [
    (1, 128, 16, 2, 96), (2, 512, 16, 2, 96), (1, 384, 4, 1, 128), (2, 256, 4, 2, 96), (1, 256, 8, 8, 128),
    (1, 1024, 16, 2, 128), (3, 640, 16, 2, 96),
])
def test_attention_prefill(dev, bs, S, nq, nkv, hd):
    from minicpm5_mk import ops
    qkv = _rand((bs * S, (nq + 2 * nkv) * hd), 21 + S + hd).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    out = ops.attention_prefill(qkv.to(dev), bs, S, nq, nkv, hd, softmax_scale=scale)
    torch.cuda.synchronize()
    _check_err()
    ref = _attn_ref(qkv, bs, S, nq, nkv, hd, scale)
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 2.5e-2, err


@pytest.mark.parametrize("hd", [96, 128])
def test_attention_prefill_deterministic(dev, hd):
    """The same inputs give the same bits on every launch (a hand-off that read O before its last P V
    landed showed up only as a rare run-to-run difference)."""
    from minicpm5_mk import ops
    bs, S, nq, nkv = 4, 8192, 16, 2
    g = torch.Generator(device=dev).manual_seed(5 + hd)
    qkv = torch.randn((bs * S, (nq + 2 * nkv) * hd), generator=g, device=dev).to(torch.bfloat16)
    ref = ops.attention_prefill(qkv, bs, S, nq, nkv, hd, softmax_scale=hd ** -0.5).clone()
    for _ in range(30):
        out = ops.attention_prefill(qkv, bs, S, nq, nkv, hd, softmax_scale=hd ** -0.5)
        assert torch.equal(out, ref)
    _check_err()


@pytest.mark.parametrize("hd", [96, 128])
def test_attention_prefill_full_length(dev, hd):
    """BASELINE isolated-attention shape (seq 8192, 16 Q / 2 KV heads) against a plain PyTorch fp32
    reference evaluated on the GPU in 1024-query chunks."""
    from minicpm5_mk import ops
    S, nq, nkv = 8192, 16, 2
    g = torch.Generator(device=dev).manual_seed(77 + hd)
    qkv = torch.randn((S, (nq + 2 * nkv) * hd), generator=g, device=dev).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    out = ops.attention_prefill(qkv, 1, S, nq, nkv, hd, softmax_scale=scale)
    torch.cuda.synchronize()
    _check_err()
    q = qkv[:, :nq * hd].float().reshape(S, nq, hd)
    k = qkv[:, nq * hd:(nq + nkv) * hd].float().reshape(S, nkv, hd).repeat_interleave(nq // nkv, dim=1)
    v = qkv[:, (nq + nkv) * hd:].float().reshape(S, nkv, hd).repeat_interleave(nq // nkv, dim=1)
    worst = 0.0
    for q0 in range(0, S, 1024):
        q1 = q0 + 1024
        s = torch.einsum("qhd,khd->hqk", q[q0:q1], k[:q1]) * scale
        mask = torch.arange(q1, device=dev)[None, :] <= torch.arange(q0, q1, device=dev)[:, None]
        s = s.masked_fill(~mask[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v[:q1]).reshape(1024, nq * hd)
        worst = max(worst, (out[q0:q1].float() - o).abs().max().item())
    assert worst < 2.5e-2, worst


def test_rope(dev):
    from minicpm5_mk import ops
    from minicpm5_mk.mk_weights import rope_tables
    rows, nh, hd, S = 512, 6, 96, 256
    cos, sin = rope_tables(1024, hd, 10000.0)
    x = _rand((rows, nh * hd + 64), 31).to(torch.bfloat16)
    y = x.to(dev).clone()
    ops.rope_(y, nh, hd, cos.to(dev), sin.to(dev), S, col0=32)
    torch.cuda.synchronize()
    pos = torch.arange(rows) % S
    xf = x.float()[:, 32:32 + nh * hd].reshape(rows, nh, hd)
    h = hd // 2
    c, s_ = cos[pos][:, None, :], sin[pos][:, None, :]
    ref = torch.cat([xf[..., :h] * c - xf[..., h:] * s_, xf[..., h:] * c + xf[..., :h] * s_], -1).reshape(rows, -1)
    got = y.float().cpu()
    assert torch.equal(got[:, :32], x.float()[:, :32]) and torch.equal(got[:, 32 + nh * hd:], x.float()[:, 32 + nh * hd:])
    assert (got[:, 32:32 + nh * hd] - ref).abs().max().item() <= 2e-2


def test_rms_and_embed(dev):
    from minicpm5_mk import ops
    V, H, T = 1000, 384, 700
    E = _rand((V, H), 41, 0.02).to(torch.bfloat16)
    ids = torch.randint(0, V, (T,), generator=_gen(42), dtype=torch.int32)
    x32, xb = ops.embed(ids.to(dev), E.to(dev), 12.0)
    torch.cuda.synchronize()
    ref32 = E.float()[ids.long()] * 12.0
    assert torch.equal(x32.cpu(), ref32)
    assert torch.equal(xb.cpu(), ref32.to(torch.bfloat16))
    r = ops.rms_rstd(x32, 1e-6)
    refr = torch.rsqrt(ref32.pow(2).mean(-1) + 1e-6)
    assert torch.allclose(r.cpu(), refr, rtol=1e-5, atol=0)
    _check_err()


def test_embed_bad_id_is_reported(dev):
    from minicpm5_mk import ops, _lib
    import ctypes
    E = torch.ones((10, 64), dtype=torch.bfloat16, device=dev)
    ids = torch.tensor([1, 10, 3], dtype=torch.int32, device=dev)
    x32, xb = ops.embed(ids, E, 1.0)
    e = ctypes.c_int32()
    st = _lib.lib().mk_get_error(None, ctypes.byref(e))
    assert st == 7 and e.value == 0x300
    assert xb[1].abs().sum().item() == 0 and x32[1].abs().sum().item() == 0 and x32[0].sum().item() == 64
    _check_err()  # cleared


@pytest.mark.parametrize("bs,H,V", [(1, 1536, 73448), (3, 384, 1000), (11, 512, 2048), (32, 1536, 73448),
                                    (5, 2048, 130560), (2, 1536, 1001)])
def test_lm_head_argmax(dev, bs, H, V):
    from minicpm5_mk import ops
    h = _rand((bs, H), 51)
    W = _rand((V, H), 52, 0.02).to(torch.bfloat16)
    if V > 100:
        W[V - 7] = W[17]  # planted exact tie: lowest id must win
        h[0] = h[0].abs()
        W[17] = W[17].abs() + 0.05
        W[V - 7] = W[17]
    logits, top1 = ops.lm_head_argmax(h.to(dev), W.to(dev))
    torch.cuda.synchronize()
    ref = h @ W.float().T
    lg = logits.cpu()
    assert (lg - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())
    # argmax indexing is exact w.r.t. the kernel's own logits (ties -> lowest id)
    assert torch.equal(top1.cpu().long(), torch.argmax(lg, dim=-1))
    if V > 100:
        assert int(top1[0]) == 17


@pytest.mark.parametrize("bs,V,k", [(3, 73448, 20), (2, 1000, 64), (1, 130560, 1)])
def test_topk_logprobs(dev, bs, V, k):
    from minicpm5_mk import ops
    from oracle import golden
    lg = torch.randn((bs, V), generator=_gen(61)) * 3.0
    lg[0, 11] = lg[0, 5] = lg[0].max() + 1.0  # planted tie at the top: lower id first
    ids, lps = ops.topk_logprobs(lg.to(dev), k)
    torch.cuda.synchronize()
    ids, lps = ids.cpu(), lps.cpu()
    for b in range(bs):
        ref_ids, ref_lps = golden.topk_logprobs(lg[b], k)
        if b == 0:  # torch.topk leaves the order of equal values open
            assert ids[0, 0].item() == 5 and (k == 1 or ids[0, 1].item() == 11)
            ref_ids = [5, 11][:k] + ref_ids[2:] if k > 1 else [5]
        assert ids[b].tolist() == ref_ids, b
        assert max(abs(a - r) for a, r in zip(lps[b].tolist(), ref_lps)) < 2e-5
