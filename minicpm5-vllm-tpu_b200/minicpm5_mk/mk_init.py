"""Seeded random initialisation of a MiniCPM5-shaped checkpoint (HF tensor names, fp32, CPU).

No real checkpoint is available offline, so every benchmark and parity config uses random-init
weights: linear / embedding / lm_head weights ~ N(0, std) (std 0.02), RMSNorm gains 1.0.  Every
tensor has its own generator seeded from (seed, tensor name), so any single tensor (e.g. one layer)
can be regenerated independently and the CPU oracle and the GPU path see identical values.

Names and shapes follow the HF Llama layout read by `plugin/minicpm5_mk/model.py:34-39` and
`benchmark/f32_golden.py:124-134` ([out_features, in_features] for every projection).
"""

from __future__ import annotations

import zlib
from typing import Dict, Iterator, Tuple

import torch

from .mk_config import MkConfig

LAYER_WEIGHTS = (
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
    "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
)
LAYER_NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight")


def param_seed(seed: int, name: str) -> int:
    """Per-tensor generator seed: deterministic in (seed, name)."""
    return (int(seed) * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 62)


def param_shapes(cfg: MkConfig) -> Dict[str, Tuple[int, ...]]:
    H, I, hd = cfg.hidden, cfg.inter, cfg.head_dim
    shapes: Dict[str, Tuple[int, ...]] = {"model.embed_tokens.weight": (cfg.vocab, H), "model.norm.weight": (H,)}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = (H,)
        shapes[p + "post_attention_layernorm.weight"] = (H,)
        shapes[p + "self_attn.q_proj.weight"] = (cfg.n_q * hd, H)
        shapes[p + "self_attn.k_proj.weight"] = (cfg.n_kv * hd, H)
        shapes[p + "self_attn.v_proj.weight"] = (cfg.n_kv * hd, H)
        shapes[p + "self_attn.o_proj.weight"] = (H, cfg.n_q * hd)
        shapes[p + "mlp.gate_proj.weight"] = (I, H)
        shapes[p + "mlp.up_proj.weight"] = (I, H)
        shapes[p + "mlp.down_proj.weight"] = (H, I)
    if not cfg.tie_embeddings:
        shapes["lm_head.weight"] = (cfg.vocab, H)
    return shapes


def make_param(name: str, shape: Tuple[int, ...], seed: int = 1234, std: float = 0.02,
               device: str | torch.device = "cpu") -> torch.Tensor:
    """One tensor.  The CPU generator (default) is what the oracle and the parity tests use; a CUDA
    device draws from that device's generator (same seeds, different values) to set up benchmark
    replicas quickly."""
    if name.endswith("norm.weight"):
        return torch.ones(shape, dtype=torch.float32, device=device)
    g = torch.Generator(device=device).manual_seed(param_seed(seed, name))
    return torch.randn(shape, generator=g, dtype=torch.float32, device=device) * std


def iter_random_weights(cfg: MkConfig, seed: int = 1234, std: float = 0.02,
                        device: str | torch.device = "cpu") -> Iterator[Tuple[str, torch.Tensor]]:
    """(name, fp32 tensor) pairs in the order a checkpoint loader would yield them."""
    for name, shape in param_shapes(cfg).items():
        yield name, make_param(name, shape, seed, std, device)


def random_state_dict(cfg: MkConfig, seed: int = 1234, std: float = 0.02,
                      device: str | torch.device = "cpu") -> Dict[str, torch.Tensor]:
    return dict(iter_random_weights(cfg, seed, std, device))


def synthetic_ids(bs: int, seq: int, seed: int = 1234, lo: int = 1000, hi: int = 30000,
                  vocab: int | None = None) -> "torch.Tensor":
    """(bs, seq) int32 token ids uniform in [lo, min(hi, vocab)), numpy default_rng(seed)
    (the reference draws prompt ids from [1000, min(vocab, 30000)), `benchmark/run_benchmark.py:341-348`).
    Vocabularies no larger than lo (the tiny test models) draw from the whole [0, vocab)."""
    import numpy as np

    if vocab is not None:
        hi = min(hi, vocab)
        if lo >= hi:
            lo = 0
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.integers(lo, hi, size=(bs, seq), dtype=np.int64).astype(np.int32))
