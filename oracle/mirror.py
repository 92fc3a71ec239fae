"""CPU numerics mirror of the B200 path (TEST INFRASTRUCTURE ONLY -- see oracle/golden.py header).

The same forward as oracle/golden.py, but on the prepared int8 weight-only weights and with bf16
rounding at exactly the points where the CUDA kernels round: the residual stream stays f32 and its
bf16 copy feeds the projections; projection outputs (q/k/v, attention output, SiLU(g)*u) are stored
in bf16; RoPE is applied in f32 to the un-rounded q/k (pair-interleaved head layout of the prepared
weights) before that rounding; f32 accumulation; f32 scales applied in the GEMM epilogue; attention
probabilities rounded to bf16 before P @ V in the prefill kernel.  It lets the GPU parity tests use tolerances near bf16
resolution, separately from the accuracy of the design against the FP32 golden.

It follows the same reference steps as oracle/golden.py (benchmark/f32_golden.py:78-102) and the
reference's weight quantiser (plugin/minicpm5_mk/mk_weights.py:113-123) as restated in
minicpm5_mk/mk_weights.py (whose output it consumes).
"""

from __future__ import annotations

import math

import torch

F32 = torch.float32


def bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(F32)


def _deq(w8: torch.Tensor) -> torch.Tensor:
    return w8.to(F32)


def _rstd(x: torch.Tensor, eps: float) -> torch.Tensor:
    return torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)


def _rope_pairs(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE in the kernels' pair-interleaved head layout (columns 2j, 2j+1 = dims j, j + hd/2),
    applied in f32 to the un-rounded projection and rounded to bf16 once.
    x: (rows, heads, hd) f32; cos/sin: (rows, hd/2)."""
    a, b = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(x)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = b * c + a * s
    return bf(out)


def _deinterleave(t: torch.Tensor, block: int = 1):
    """Fused gate/up rows of the prepared weights (alternating rows) -> (gate, up)."""
    n2 = t.shape[0]
    v = t.reshape(n2 // (2 * block), 2, block, *t.shape[1:])
    return v[:, 0].reshape(n2 // 2, *t.shape[1:]), v[:, 1].reshape(n2 // 2, *t.shape[1:])


def _attn_prefill(q, k, v, G):
    """q: (S, nq, hd), k/v: (S, nkv, hd) bf16-valued; causal; P rounded to bf16 for P @ V."""
    S, nq, hd = q.shape
    out = torch.empty((S, nq * hd), dtype=F32)
    for q0 in range(0, S, 512):
        q1 = min(S, q0 + 512)
        qq = q[q0:q1]
        kk, vv = k[:q1], v[:q1]
        kr = kk.repeat_interleave(G, dim=1)
        vr = vv.repeat_interleave(G, dim=1)
        s = torch.einsum("qhd,khd->hqk", qq, kr)
        qi = torch.arange(q0, q1)[:, None]
        kj = torch.arange(q1)[None, :]
        s = torch.where((kj <= qi)[None], s, torch.tensor(-math.inf))
        m = s.amax(-1, keepdim=True)
        p = torch.exp(s - m)
        l = p.sum(-1, keepdim=True)
        o = torch.einsum("hqk,khd->qhd", bf(p), vr) / l.permute(1, 0, 2)
        out[q0:q1] = bf(o.reshape(q1 - q0, nq * hd))
    return out


@torch.no_grad()
def mirror_forward(ids: torch.Tensor, pw: dict, cfg):
    """ids: (bs, S) int. pw: prepared weights (minicpm5_mk.mk_weights.prepare_mk_weights, CPU).
    Returns (logits (bs, V) f32, hidden (bs, H) f32 final-normed rows)."""
    bs, S = ids.shape
    L, H, I = cfg.num_layers, cfg.hidden, cfg.inter
    nq, nkv, hd = cfg.n_q, cfg.n_kv, cfg.head_dim
    qd, kvd = nq * hd, nkv * hd
    G = nq // nkv
    r = cfg.residual_scale
    cos, sin = pw["rope_cos"][:S], pw["rope_sin"][:S]
    E = pw["embed"].to(F32)
    logits_all, hidden_all = [], []
    for b in range(bs):
        x = E[ids[b].long()] * cfg.scale_emb  # f32 residual stream
        for l in range(L - 1):
            Wqkv, sqkv = _deq(pw["w_qkv"][l]), pw["s_qkv"][l]
            qkv = (bf(x) @ Wqkv.T) * _rstd(x, cfg.eps) * sqkv
            q = _rope_pairs(qkv[:, :qd].reshape(S, nq, hd), cos, sin)
            k = _rope_pairs(qkv[:, qd:qd + kvd].reshape(S, nkv, hd), cos, sin)
            v = bf(qkv[:, qd + kvd:]).reshape(S, nkv, hd)
            a = _attn_prefill(q, k, v, G)
            x = x + r * ((a @ _deq(pw["w_o"][l]).T) * pw["s_o"][l])
            gu = (bf(x) @ _deq(pw["w_gu"][l]).T) * _rstd(x, cfg.eps) * pw["s_gu"][l]
            g, u = _deinterleave(gu.T)
            h = bf(torch.nn.functional.silu(g.T) * u.T)
            x = x + r * ((h @ _deq(pw["w_down"][l]).T) * pw["s_down"][l])
        l = L - 1
        Wqkv, sqkv = _deq(pw["w_qkv"][l]), pw["s_qkv"][l]
        rs = _rstd(x, cfg.eps)
        kv = (bf(x) @ Wqkv[qd:].T) * rs * sqkv[qd:]
        k = _rope_pairs(kv[:, :kvd].reshape(S, nkv, hd), cos, sin)
        v = bf(kv[:, kvd:]).reshape(S, nkv, hd)
        xl = x[-1:]
        ql = (bf(xl) @ Wqkv[:qd].T) * _rstd(xl, cfg.eps) * sqkv[:qd]
        ql = _rope_pairs(ql.reshape(1, nq, hd), cos[-1:], sin[-1:])[0]
        kr = k.repeat_interleave(G, dim=1)
        vr = v.repeat_interleave(G, dim=1)
        s = torch.einsum("hd,khd->hk", ql, kr)
        p = torch.softmax(s, dim=-1)
        al = bf(torch.einsum("hk,khd->hd", p, vr).reshape(1, qd))
        xl = xl + r * ((al @ _deq(pw["w_o"][l]).T) * pw["s_o"][l])
        gu = (bf(xl) @ _deq(pw["w_gu"][l]).T) * _rstd(xl, cfg.eps) * pw["s_gu"][l]
        g, u = _deinterleave(gu.T)
        h = bf(torch.nn.functional.silu(g.T) * u.T)
        xl = xl + r * ((h @ _deq(pw["w_down"][l]).T) * pw["s_down"][l])
        hn = xl * _rstd(xl, cfg.eps) * pw["final_norm"]
        logits_all.append((hn * cfg.logit_scale) @ pw["lm_head"].to(F32).T)
        hidden_all.append(hn)
    return torch.cat(logits_all, 0), torch.cat(hidden_all, 0)
