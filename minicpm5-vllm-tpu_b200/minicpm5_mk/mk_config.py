"""Model configuration for the MiniCPM5 prefill-score path.

The reference reads its config from the HF checkpoint (`plugin/minicpm5_mk/model.py:561-567`):
num_layers, hidden, inter, n_q, n_kv, head_dim, eps, rope_theta.  On top of those the B200 path
carries the three MiniCPM muP scalars that the benchmark configs ask for (scale_emb, residual
scale, logit scale).  With all three at 1.0 the model is exactly the plain-Llama forward of
`benchmark/f32_golden.py:78-102`.

    x      = scale_emb * embed[ids]
    x     += residual_scale * branch(x)          (attention and MLP branches)
    logits = (logit_scale * h) @ lm_head^T       (logit_scale = 256 / hidden: "scaled by hidden/256"
                                                  read as divided by hidden/256, MiniCPM convention)
"""

from __future__ import annotations

import dataclasses
import math


@dataclasses.dataclass(frozen=True)
class MkConfig:
    num_layers: int
    hidden: int
    inter: int
    n_q: int
    n_kv: int
    head_dim: int
    vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-6
    scale_emb: float = 1.0
    residual_scale: float = 1.0
    logit_scale: float = 1.0
    max_seq: int = 8192
    tie_embeddings: bool = False
    # projection weights: 8 = int8 weight-only per output channel (the BASELINE configs), 16 = bf16
    weight_bits: int = 8

    @property
    def q_dim(self) -> int:
        return self.n_q * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim

    def replace(self, **kw) -> "MkConfig":
        return dataclasses.replace(self, **kw)

    def as_dict(self) -> dict:
        return dataclasses.asdict(self)

    def check(self) -> None:
        """Shape contract of the CUDA path (the C library rejects the same cases with MK_ERR_BAD_SHAPE)."""
        if self.head_dim not in (96, 128):
            raise ValueError(f"head_dim {self.head_dim} not in (96, 128)")
        if self.n_q % self.n_kv:
            raise ValueError("n_q must be a multiple of n_kv")
        if self.hidden % 128 or self.inter % 128 or self.q_dim % 128 or self.qkv_dim % 128:
            raise ValueError("hidden % 128, inter % 128, n_q*head_dim % 128 and qkv width % 128 must be 0")
        if (2 * self.n_kv * self.head_dim) % 128:
            raise ValueError("2*n_kv*head_dim must be a multiple of 128")
        if self.weight_bits not in (8, 16):
            raise ValueError(f"weight_bits {self.weight_bits} not in (8, 16)")


def minicpm_mup(num_layers: int, hidden: int) -> dict:
    """MiniCPM muP scalars: scale_emb 12, residual 1.4/sqrt(L), logits divided by hidden/256."""
    return dict(scale_emb=12.0, residual_scale=1.4 / math.sqrt(num_layers), logit_scale=256.0 / hidden)


# Primary graded configs: BASELINE configs with the plugin's intermediate sizes (4608 / 6144).
PRESETS: dict[str, MkConfig] = {
    "minicpm5-1b": MkConfig(num_layers=24, hidden=1536, inter=4608, n_q=16, n_kv=2, head_dim=96,
                            vocab=73448, rope_theta=10000.0, **minicpm_mup(24, 1536)),
    "minicpm5-1b-i4096": MkConfig(num_layers=24, hidden=1536, inter=4096, n_q=16, n_kv=2, head_dim=96,
                                  vocab=73448, rope_theta=10000.0, **minicpm_mup(24, 1536)),
    # Dimensions of the real MiniCPM5-1B checkpoint (plain Llama: no muP), results/v6e_minicpm5_1b.json.
    "minicpm5-1b-ckpt": MkConfig(num_layers=24, hidden=1536, inter=4608, n_q=16, n_kv=2, head_dim=128,
                                 vocab=130560, rope_theta=5000000.0),
    "minicpm5-2b": MkConfig(num_layers=42, hidden=2048, inter=6144, n_q=16, n_kv=2, head_dim=128,
                            vocab=73448, rope_theta=10000.0, **minicpm_mup(42, 2048)),
    # Small configs for parity tests (same code paths, hd 96 and 128).
    "tiny-hd96": MkConfig(num_layers=3, hidden=384, inter=512, n_q=4, n_kv=2, head_dim=96, vocab=1000,
                          **minicpm_mup(3, 384), max_seq=1024),
    "tiny-hd128": MkConfig(num_layers=2, hidden=512, inter=768, n_q=4, n_kv=1, head_dim=128, vocab=2048,
                           max_seq=1024),
}


def get_config(name: str) -> MkConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown config {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[name]


def rope_support(hf) -> tuple:
    """(rope_theta or None, problem or None) from a HF config's `rope_scaling` / `rope_parameters`
    (`plugin/minicpm5_mk/model.py:576-585`).  Newer configs keep rope_theta only inside
    `rope_parameters`; a theta there overrides the top-level field.  Any rope_type other than the
    plain one ("default", or none given) -- longrope, yarn, linear, dynamic ... -- is a problem: the
    kernels apply plain RoPE only."""
    rs = getattr(hf, "rope_scaling", None) or getattr(hf, "rope_parameters", None)
    if isinstance(rs, dict):
        rtype = rs.get("rope_type", rs.get("type", "default"))
        theta = float(rs["rope_theta"]) if rs.get("rope_theta") is not None else None
        if rtype not in (None, "default"):
            return theta, f"rope_scaling={rs} unsupported"
        return theta, None
    if rs:
        return None, f"rope_scaling={rs} unsupported"
    return None, None


def from_hf_config(hf, max_seq: int = 8192) -> MkConfig:
    """Config from a HF/vLLM `hf_config` (fields as read by `plugin/minicpm5_mk/model.py:561-567`).

    MiniCPM checkpoints carry `scale_emb`, `scale_depth` and `dim_model_base`; plain Llama ones do not,
    in which case the three scalars stay 1.0.  rope_theta comes from `rope_parameters` / `rope_scaling`
    when they hold one (`rope_support`); whether the rope type is supported is for the caller to check."""
    L = int(hf.num_hidden_layers)
    H = int(hf.hidden_size)
    n_q = int(hf.num_attention_heads)
    hd = int(getattr(hf, "head_dim", None) or H // n_q)
    theta, _ = rope_support(hf)
    if theta is None:
        theta = float(getattr(hf, "rope_theta", 10000.0) or 10000.0)
    scale_emb = float(getattr(hf, "scale_emb", 1.0) or 1.0)
    scale_depth = getattr(hf, "scale_depth", None)
    dim_base = getattr(hf, "dim_model_base", None)
    return MkConfig(
        num_layers=L, hidden=H, inter=int(hf.intermediate_size), n_q=n_q,
        n_kv=int(getattr(hf, "num_key_value_heads", n_q)), head_dim=hd, vocab=int(hf.vocab_size),
        rope_theta=theta, eps=float(hf.rms_norm_eps),
        scale_emb=scale_emb,
        residual_scale=(float(scale_depth) / math.sqrt(L)) if scale_depth is not None else 1.0,
        logit_scale=(float(dim_base) / H) if dim_base is not None else 1.0,
        max_seq=max_seq, tie_embeddings=bool(getattr(hf, "tie_word_embeddings", False)),
    )
