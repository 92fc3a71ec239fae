"""CPU oracle: restatement of the reference's full-FP32 golden forward.

TEST INFRASTRUCTURE ONLY.  Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s cpu_baseline /
`--impl reference` legs may import this module, and only as the checker or the timed CPU baseline.
The product path (the `minicpm5_mk` package and its CUDA library) never imports it.

What it restates: `benchmark/f32_golden.py` of the reference (MG-Cafe/minicpm5-vllm-tpu):

* `rope_tables` (f32_golden.py:45-50): inv_freq and angles in float64, cos/sin of [f, f] as f32.
* `rms` (f32_golden.py:53-54): x * rsqrt(mean(x^2) + eps) * w.
* `rot_half` (f32_golden.py:57-59): [-x2, x1].
* `_attn_chunk` (f32_golden.py:62-75): causal GQA, scores / sqrt(hd), -inf mask, f32 softmax,
  queries in chunks of 1024.  Keys beyond the chunk's last query are skipped here: they are fully
  masked in the reference, so the result is the same.
* `forward_one` (f32_golden.py:78-102): separate q/k/v matmuls, RoPE on q and k, residual adds,
  SiLU(gate) * up -> down, final RMSNorm on the last row, lm_head, log_softmax, top-k.
* lm_head = `lm_head.weight` or the tied embedding (f32_golden.py:122).

Additions (all default to 1.0, which gives exactly the reference golden): the three MiniCPM muP
scalars of the benchmark configs -- x = scale_emb * embed[ids]; x += residual_scale * branch;
logits = (logit_scale * h) @ lm_head^T.

Pinning: `tests/golden/make_golden.py` runs the reference's own `forward_one` (with a numpy
stand-in for the jax calls it makes) on small random-init models and commits its top-20 ids and
logprobs; `tests/test_oracle.py` checks this restatement against those fixtures.  The reference's
own golden dumps (`benchmark/ref/*.json`) pin the real HF checkpoints only, which are not available
offline.
"""

from __future__ import annotations

import math
from typing import Dict, List, Tuple

import numpy as np
import torch

F32 = torch.float32


def rope_tables(S: int, hd: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """f32_golden.py:45-50."""
    inv = 1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    t = np.arange(S, dtype=np.float64)
    f = np.einsum("i,j->ij", t, inv)
    e = np.concatenate([f, f], -1)
    return torch.from_numpy(np.cos(e).astype(np.float32)), torch.from_numpy(np.sin(e).astype(np.float32))


def rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """f32_golden.py:53-54."""
    return x * torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps) * w


def rot_half(x: torch.Tensor) -> torch.Tensor:
    """f32_golden.py:57-59."""
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def attn_chunk(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q0: int) -> torch.Tensor:
    """f32_golden.py:62-75. q: (Cq, nq, hd); k, v: (S, nkv, hd) -> (Cq, nq*hd)."""
    Cq, nq, hd = q.shape
    nkv = k.shape[1]
    g = nq // nkv
    kend = q0 + Cq  # keys past the last query are fully masked
    kk, vv = k[:kend], v[:kend]
    qg = q.reshape(Cq, nkv, g, hd)
    s = torch.einsum("qngd,knd->ngqk", qg, kk) / math.sqrt(hd)
    qi = q0 + torch.arange(Cq)[:, None]
    kj = torch.arange(kend)[None, :]
    s = torch.where((kj <= qi)[None, None], s, torch.tensor(-math.inf, dtype=F32))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("ngqk,knd->qngd", p, vv)
    return o.reshape(Cq, nq * hd)


def golden_weights(sd: Dict[str, torch.Tensor], cfg) -> dict:
    """HF-named tensors -> f32 matrices in x @ W form (f32_golden.py:119-134)."""
    put = lambda a: a.to(F32)  # noqa: E731
    emb = put(sd["model.embed_tokens.weight"])
    W = {"embed": emb, "norm": put(sd["model.norm.weight"]),
         "lm_head": put(sd["lm_head.weight"]).T if "lm_head.weight" in sd else emb.T, "layers": []}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        W["layers"].append({
            "in": put(sd[p + "input_layernorm.weight"]), "post": put(sd[p + "post_attention_layernorm.weight"]),
            "q": put(sd[p + "self_attn.q_proj.weight"]).T, "k": put(sd[p + "self_attn.k_proj.weight"]).T,
            "v": put(sd[p + "self_attn.v_proj.weight"]).T, "o": put(sd[p + "self_attn.o_proj.weight"]).T,
            "gate": put(sd[p + "mlp.gate_proj.weight"]).T, "up": put(sd[p + "mlp.up_proj.weight"]).T,
            "down": put(sd[p + "mlp.down_proj.weight"]).T,
        })
    return W


@torch.no_grad()
def forward_logits(ids: torch.Tensor, W: dict, cfg, layers: int | None = None,
                   last_only: bool = True) -> torch.Tensor:
    """f32_golden.forward_one up to the logits. ids: (S,) int. Returns last-token logits (V,) f32.

    With `layers` < cfg.num_layers only the first `layers` decoder layers run (timed CPU samples).
    With `last_only` the last layer computes K/V for every position but Q, attention, O and the MLP
    for the last position only -- the rows that feed the last-token logits are unchanged."""
    L = cfg.num_layers if layers is None else layers
    nq, nkv, hd, eps = cfg.n_q, cfg.n_kv, cfg.head_dim, cfg.eps
    S = int(ids.shape[0])
    cos, sin = rope_tables(S, hd, cfg.rope_theta)
    x = W["embed"][ids.long()] * cfg.scale_emb
    r = cfg.residual_scale
    for i in range(L):
        lw = W["layers"][i]
        last = last_only and i == L - 1
        xn = rms(x, lw["in"], eps)
        kk = (xn @ lw["k"]).reshape(S, nkv, hd)
        v = (xn @ lw["v"]).reshape(S, nkv, hd)
        kk = kk * cos[:, None, :] + rot_half(kk) * sin[:, None, :]
        if last:
            q = (xn[-1:] @ lw["q"]).reshape(1, nq, hd)
            q = q * cos[-1:, None, :] + rot_half(q) * sin[-1:, None, :]
            a = attn_chunk(q, kk, v, S - 1)
            x = x[-1:] + r * (a @ lw["o"])
        else:
            q = (xn @ lw["q"]).reshape(S, nq, hd)
            q = q * cos[:, None, :] + rot_half(q) * sin[:, None, :]
            a = torch.cat([attn_chunk(q[q0:q0 + 1024], kk, v, q0) for q0 in range(0, S, 1024)], 0)
            x = x + r * (a @ lw["o"])
        xn = rms(x, lw["post"], eps)
        gte = xn @ lw["gate"]
        up = xn @ lw["up"]
        x = x + r * ((torch.nn.functional.silu(gte) * up) @ lw["down"])
    h = rms(x[-1], W["norm"], eps)
    return (h * cfg.logit_scale) @ W["lm_head"]


def topk_logprobs(logits: torch.Tensor, k: int = 20) -> Tuple[List[int], List[float]]:
    """f32_golden.py:100-102 (log_softmax then top-k)."""
    lp = torch.log_softmax(logits.to(torch.float64), dim=-1)
    v, i = torch.topk(lp, k)
    return i.tolist(), v.tolist()


def argmax_first(logits: torch.Tensor) -> int:
    """Greedy token: the maximum logit, ties broken toward the lowest id (torch.argmax convention)."""
    m = logits.max()
    return int(torch.nonzero(logits == m)[0, 0])


def forward_one(ids: torch.Tensor, W: dict, cfg, k: int = 20) -> Tuple[List[int], List[float]]:
    """f32_golden.forward_one: (top-k ids, top-k logprobs) at the last position."""
    return topk_logprobs(forward_logits(ids, W, cfg), k)
