"""Load-time weight preparation: HF-named tensors -> the B200 kernels' HBM layout.

Follows the reference's `prepare_mk_weights` (`plugin/minicpm5_mk/mk_weights.py:126-265`) for
the parts this path keeps, re-laid-out for the tcgen05 GEMMs:

* 1/sqrt(head_dim) is folded into the Q rows before quantisation (`mk_weights.py:147`).
* The RMSNorm gains are folded into the weight columns (input channels) before quantisation, so the
  GEMM epilogue only applies the per-row rstd and the per-output-channel scale.
* int8 weight-only, per-output-channel: scale = max(amax_over_inputs(|W|) / 127, 1e-8),
  q = clamp(round_half_even(W / scale), -127, 127) (`_quantize_w`, `mk_weights.py:113-123`).
  No activation quantisation (the reference's W8A8 SmoothQuant calibration is not used).
  With `cfg.weight_bits == 16` the same layout is kept in bf16, unquantised, with unit scales.
* Every projection stays [out_features, in_features] (K contiguous = "K-major" B operand).
* gate/up are fused into one [2I, H] matrix with alternating rows ([g_0, u_0, g_1, u_1, ...],
  GU_BLOCK = 1): the GEMM keeps one weight row per TMEM lane, so gate and up of a channel sit in
  adjacent lanes and SiLU(g)*u takes one lane shuffle in the epilogue (same idea as the reference's
  chunk-interleaved `interleave_gu`, `plugin/minicpm5_mk/mk_mlp.py:148-158`, at a block of 1).
* All L layers are int8 (the reference keeps its last layer in bf16 because W8A8 hurt accuracy;
  weight-only int8 does not need that).
* RoPE tables: inv_freq = theta^(-2i/hd) and angles in float64, cos/sin stored as f32
  [max_seq, hd/2] (`benchmark/f32_golden.py:45-50`; the [f, f] duplication is implicit).
* RoPE is applied in the QKV GEMM epilogue.  To keep each rotation pair (i, i + hd/2) in adjacent
  output columns, the Q and K rows of every head are reordered to (0, hd/2, 1, hd/2 + 1, ...).
  Q and K use the same order, so Q.K (and the attention result) is unchanged; V keeps its order.
"""

from __future__ import annotations

import math
from typing import Dict, Iterable, Tuple

import numpy as np
import torch

from .mk_config import MkConfig

GU_BLOCK = 1
BF16 = torch.bfloat16
F32 = torch.float32


def quantize_per_out_channel(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """w: [out, in] float -> (int8 [out, in], f32 scale [out]).

    The divisor 127 is a tensor, not a Python scalar: torch's CUDA kernels turn division by a scalar into a
    multiplication by its reciprocal, which can differ from the division in the last bit; tensor / tensor
    divides exactly on every device, so a GPU preparation matches the CPU one bit for bit."""
    w = w.to(F32)
    amax = w.abs().amax(dim=1, keepdim=True)
    scale = torch.clamp(amax / torch.full((), 127.0, dtype=F32, device=w.device), min=1e-8)
    q = torch.clamp(torch.round(w / scale), -127, 127).to(torch.int8)
    return q.contiguous(), scale.squeeze(1).contiguous()


def rope_tables(max_seq: int, head_dim: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    t = np.arange(max_seq, dtype=np.float64)
    f = np.einsum("i,j->ij", t, inv)
    return torch.from_numpy(np.cos(f).astype(np.float32)), torch.from_numpy(np.sin(f).astype(np.float32))


def interleave_gu(gate: torch.Tensor, up: torch.Tensor, block: int = GU_BLOCK) -> torch.Tensor:
    """[I, ...] gate and up -> [2I, ...] with alternating blocks of `block` rows."""
    I = gate.shape[0]
    assert I % block == 0 and up.shape == gate.shape
    g = gate.reshape(I // block, block, *gate.shape[1:])
    u = up.reshape(I // block, block, *up.shape[1:])
    return torch.stack([g, u], dim=1).reshape(2 * I, *gate.shape[1:]).contiguous()


def deinterleave_gu(x: torch.Tensor, block: int = GU_BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    n2 = x.shape[0]
    v = x.reshape(n2 // (2 * block), 2, block, *x.shape[1:])
    return v[:, 0].reshape(n2 // 2, *x.shape[1:]), v[:, 1].reshape(n2 // 2, *x.shape[1:])


def rope_pair_order(head_dim: int) -> torch.Tensor:
    """Row order that makes rotation pairs adjacent: new row 2j <- j, new row 2j+1 <- j + hd/2."""
    half = head_dim // 2
    return torch.stack([torch.arange(half), torch.arange(half) + half], dim=1).reshape(-1)


def pair_heads(w: torch.Tensor, n_heads: int, head_dim: int) -> torch.Tensor:
    """Reorder the rows of every head of a [n_heads*head_dim, ...] projection into rope_pair_order."""
    perm = rope_pair_order(head_dim).to(w.device)
    return w.reshape(n_heads, head_dim, *w.shape[1:])[:, perm].reshape(w.shape)


def quantize_or_cast(w: torch.Tensor, weight_bits: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """int8 per output channel (weight_bits 8) or bf16 with unit scales (weight_bits 16)."""
    if weight_bits == 16:
        return w.to(BF16).contiguous(), torch.ones(w.shape[0], dtype=F32, device=w.device)
    return quantize_per_out_channel(w)


def prepare_layer(sd: Dict[str, torch.Tensor], cfg: MkConfig, i: int) -> Dict[str, torch.Tensor]:
    p = f"model.layers.{i}."
    quant = lambda w: quantize_or_cast(w, cfg.weight_bits)  # noqa: E731
    f = lambda n: sd[p + n].to(F32)  # noqa: E731
    g_in = f("input_layernorm.weight")
    g_post = f("post_attention_layernorm.weight")
    sm = 1.0 / math.sqrt(cfg.head_dim)
    wq = pair_heads(f("self_attn.q_proj.weight") * sm, cfg.n_q, cfg.head_dim)
    wk = pair_heads(f("self_attn.k_proj.weight"), cfg.n_kv, cfg.head_dim)
    wqkv = torch.cat([wq, wk, f("self_attn.v_proj.weight")], 0) * g_in[None, :]
    w_qkv, s_qkv = quant(wqkv)
    w_o, s_o = quant(f("self_attn.o_proj.weight"))
    wg = f("mlp.gate_proj.weight") * g_post[None, :]
    wu = f("mlp.up_proj.weight") * g_post[None, :]
    qg, sg = quant(wg)
    qu, su = quant(wu)
    w_gu = interleave_gu(qg, qu)
    s_gu = interleave_gu(sg, su)
    w_down, s_down = quant(f("mlp.down_proj.weight"))
    return dict(w_qkv=w_qkv, s_qkv=s_qkv, w_o=w_o, s_o=s_o, w_gu=w_gu, s_gu=s_gu, w_down=w_down, s_down=s_down)


LAYER_KEYS = ("w_qkv", "s_qkv", "w_o", "s_o", "w_gu", "s_gu", "w_down", "s_down")


def prepare_mk_weights(sd: Dict[str, torch.Tensor], cfg: MkConfig) -> Dict[str, torch.Tensor]:
    """HF-named CPU tensors -> CPU tensors in the kernels' layout (stacked over layers)."""
    cfg.check()
    per = [prepare_layer(sd, cfg, i) for i in range(cfg.num_layers)]
    out = {k: torch.stack([d[k] for d in per]).contiguous() for k in LAYER_KEYS}
    emb = sd["model.embed_tokens.weight"]
    out["embed"] = emb.to(BF16).contiguous()
    lm = sd.get("lm_head.weight", emb)
    out["lm_head"] = lm.to(BF16).contiguous()
    out["final_norm"] = sd["model.norm.weight"].to(F32).contiguous()
    c, s = rope_tables(cfg.max_seq, cfg.head_dim, cfg.rope_theta)
    out["rope_cos"], out["rope_sin"] = c.to(emb.device), s.to(emb.device)
    return out


def prepare_from_iter(weights: Iterable[Tuple[str, torch.Tensor]], cfg: MkConfig) -> Dict[str, torch.Tensor]:
    return prepare_mk_weights(dict(weights), cfg)
