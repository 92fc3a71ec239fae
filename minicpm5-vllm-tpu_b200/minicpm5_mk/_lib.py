"""ctypes binding of the C ABI in include/minicpm5_mk.h (libminicpm5_mk.so, built in-tree).

There is no fallback: if the library is missing or a call fails, a RuntimeError is raised.
"""

from __future__ import annotations

import ctypes
import os

LIB_NAME = "libminicpm5_mk.so"
# MINICPM5_MK_LIB overrides the library path (a build kept elsewhere, e.g. for A/B timing of two builds)
LIB_PATH = os.environ.get("MINICPM5_MK_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# Every symbol declared in include/minicpm5_mk.h.
EXPORTED = (
    "mk_status_string", "mk_version", "mk_create", "mk_bind_weights", "mk_workspace_size", "mk_forward",
    "mk_get_error", "mk_destroy", "mk_gemm_w8a16", "mk_attention_prefill", "mk_rope", "mk_rms_rstd", "mk_embed",
    "mk_lm_head_parts", "mk_lm_head_argmax", "mk_launches_per_forward", "mk_lm_head_argmax_noalloc",
    "mk_topk_logprobs", "mk_forward_timed", "mk_sp_block", "mk_workspace_size_sp", "mk_forward_sp",
    "mk_gemm_w8a16_fused", "mk_set_sp_key_split",
)

MK_GEMM_ROWSCALE, MK_GEMM_RESID, MK_GEMM_SWIGLU, MK_GEMM_COLSCALE, MK_GEMM_RESID32 = 0, 1, 2, 3, 4

_i32, _f32, _vp, _sz = ctypes.c_int32, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class MkConfigC(ctypes.Structure):
    _fields_ = [("num_layers", _i32), ("hidden", _i32), ("inter", _i32), ("n_q", _i32), ("n_kv", _i32),
                ("head_dim", _i32), ("vocab", _i32), ("max_seq", _i32), ("eps", _f32), ("rope_theta", _f32),
                ("scale_emb", _f32), ("residual_scale", _f32), ("logit_scale", _f32), ("weight_bits", _i32)]


class MkWeightPtrsC(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("embed", "lm_head", "final_norm", "rope_cos", "rope_sin", "w_qkv", "s_qkv",
                                   "w_o", "s_o", "w_gu", "s_gu", "w_down", "s_down")]


class MkGemmFusionC(ctypes.Structure):
    _fields_ = [("rowsq", _vp), ("rowsq_ld", _i32), ("rowsq_np", _i32), ("norm_dim", _i32), ("eps", _f32),
                ("rope_cos", _vp), ("rope_sin", _vp), ("rope_cols", _i32), ("head_dim", _i32), ("rope_seq", _i32),
                ("rope_pos_base", _i32), ("weight_bits", _i32)]


MK_STAGE_NAMES = ("embed", "qkv", "attn", "o_proj", "gate_up", "down", "last_layer", "head", "kv_gather")

# int32 (*)(void* ctx, const void* d_send, void* d_recv, size_t bytes_per_rank, void* stream)
ALLGATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                ctypes.c_void_p)


class MkStageTimesC(ctypes.Structure):
    _fields_ = [("ms", _f32 * len(MK_STAGE_NAMES)), ("launches", _i32 * len(MK_STAGE_NAMES))]


class MkError(RuntimeError):
    def __init__(self, what: str, status: int):
        super().__init__(f"minicpm5_mk: {what} failed: {status_string(status)} ({status})")
        self.status = status


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"minicpm5_mk: CUDA library {LIB_PATH} is not built "
                               "(run `python -c 'import __graft_entry__ as g; g.build()'`)")
        L = ctypes.CDLL(LIB_PATH)
        L.mk_status_string.restype = ctypes.c_char_p
        L.mk_status_string.argtypes = [_i32]
        L.mk_version.restype = _i32
        L.mk_version.argtypes = []
        L.mk_create.argtypes = [ctypes.POINTER(MkConfigC), _i32, ctypes.POINTER(_vp)]
        L.mk_bind_weights.argtypes = [_vp, ctypes.POINTER(MkWeightPtrsC)]
        L.mk_workspace_size.argtypes = [_vp, _i32, _i32, ctypes.POINTER(_sz)]
        L.mk_forward.argtypes = [_vp, _vp, _i32, _i32, _vp, _sz, _vp, _vp, _vp, _vp]
        L.mk_forward_timed.argtypes = [_vp, _vp, _i32, _i32, _vp, _sz, _vp, _vp, _vp, _vp,
                                       ctypes.POINTER(MkStageTimesC)]
        L.mk_sp_block.restype = _i32
        L.mk_sp_block.argtypes = [_vp, _i32, _i32]
        L.mk_workspace_size_sp.argtypes = [_vp, _i32, _i32, ctypes.POINTER(_sz)]
        L.mk_set_sp_key_split.argtypes = [_vp, _i32]
        L.mk_forward_sp.argtypes = [_vp, _vp, _i32, _i32, _i32, ALLGATHER_FN, _vp, _vp, _sz, _vp, _vp, _vp, _vp,
                                    ctypes.POINTER(MkStageTimesC)]
        L.mk_get_error.argtypes = [_vp, ctypes.POINTER(_i32)]
        L.mk_destroy.restype = None
        L.mk_destroy.argtypes = [_vp]
        L.mk_gemm_w8a16.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _vp, _i32,
                                    _vp]
        L.mk_gemm_w8a16_fused.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _i32, _i32, _vp, _f32, _vp, _i32, _vp,
                                          _i32, ctypes.POINTER(MkGemmFusionC), _vp]
        L.mk_attention_prefill.argtypes = [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp,
                                           _i32, _vp]
        L.mk_rope.argtypes = [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i32, _i32, _vp]
        L.mk_rms_rstd.argtypes = [_vp, _i32, _i32, _i32, _f32, _vp, _vp]
        L.mk_embed.argtypes = [_vp, _i32, _vp, _i32, _i32, _f32, _vp, _vp, _vp]
        L.mk_lm_head_parts.restype = _i32
        L.mk_lm_head_parts.argtypes = []
        L.mk_lm_head_argmax.argtypes = [_vp, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _vp]
        L.mk_lm_head_argmax_noalloc.argtypes = [_vp, _i32, _i32, _vp, _i32, _vp, _vp, _vp]
        L.mk_topk_logprobs.argtypes = [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp]
        L.mk_launches_per_forward.restype = _i32
        L.mk_launches_per_forward.argtypes = [_vp, _i32, _i32]
        for name in EXPORTED:
            if name not in ("mk_status_string", "mk_version", "mk_destroy", "mk_lm_head_parts",
                            "mk_launches_per_forward"):
                getattr(L, name).restype = _i32
        _LIB = L
    return _LIB


def status_string(status: int) -> str:
    try:
        return lib().mk_status_string(int(status)).decode()
    except Exception:  # noqa: BLE001
        return f"status {status}"


def check(status: int, what: str) -> None:
    if status != 0:
        raise MkError(what, status)
