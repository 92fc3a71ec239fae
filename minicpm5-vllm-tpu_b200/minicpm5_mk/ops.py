"""torch-facing wrappers of the C ABI: the whole-model engine and the per-stage kernels.

Tensors are only plumbing here: device memory, the current CUDA stream and shapes.  All math runs
in libminicpm5_mk.so; nothing falls back to torch.
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from .mk_config import MkConfig


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"minicpm5_mk: {name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"minicpm5_mk: {name} must be contiguous")


WEIGHT_FIELDS = ("embed", "lm_head", "final_norm", "rope_cos", "rope_sin", "w_qkv", "s_qkv", "w_o", "s_o", "w_gu",
                 "s_gu", "w_down", "s_down")


class MkEngine:
    """One library handle on one device with its bound weights.

    `forward(ids, bs, seq)` is the counterpart of the reference op call in
    `MiniCPM5MegakernelForCausalLM._mk_call` (plugin/minicpm5_mk/model.py:737-753); it returns the
    final-normed last-token hidden rows (bs, H) bf16, the last-token logits (bs, V) f32 and the greedy
    token ids (bs,) int32."""

    def __init__(self, cfg: MkConfig, weights: Dict[str, torch.Tensor], device: torch.device | int | str = "cuda"):
        cfg.check()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        L = _lib.lib()
        c = _lib.MkConfigC(cfg.num_layers, cfg.hidden, cfg.inter, cfg.n_q, cfg.n_kv, cfg.head_dim, cfg.vocab,
                           cfg.max_seq, cfg.eps, cfg.rope_theta, cfg.scale_emb, cfg.residual_scale, cfg.logit_scale,
                           cfg.weight_bits)
        h = ctypes.c_void_p()
        _lib.check(L.mk_create(ctypes.byref(c), self.device.index, ctypes.byref(h)), "mk_create")
        self._h = h
        self.weights = {}
        wdt = torch.bfloat16 if cfg.weight_bits == 16 else torch.int8
        for k in ("w_qkv", "w_o", "w_gu", "w_down"):
            if weights[k].dtype != wdt:
                raise ValueError(f"minicpm5_mk: {k} is {weights[k].dtype}, weight_bits {cfg.weight_bits} wants {wdt}")
        for k in WEIGHT_FIELDS:
            t = weights[k]
            if t.device != self.device:
                t = t.to(self.device)
            _cuda(t, k)
            self.weights[k] = t
        wp = _lib.MkWeightPtrsC(*[self.weights[k].data_ptr() for k in WEIGHT_FIELDS])
        _lib.check(L.mk_bind_weights(self._h, ctypes.byref(wp)), "mk_bind_weights")
        self._ws: Optional[torch.Tensor] = None

    def workspace_bytes(self, bs: int, seq: int) -> int:
        n = ctypes.c_size_t()
        _lib.check(_lib.lib().mk_workspace_size(self._h, bs, seq, ctypes.byref(n)), "mk_workspace_size")
        return int(n.value)

    def _workspace(self, bs: int, seq: int) -> torch.Tensor:
        n = self.workspace_bytes(bs, seq)
        if self._ws is None or self._ws.numel() < n:
            self._ws = None
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, ids: torch.Tensor, bs: int, seq: int, *, hidden: bool = True, logits: bool = True,
                out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
                stage_times: Optional[dict] = None):
        """Prefill-score forward through `mk_forward`.  With a `stage_times` dict, the same launches run
        through `mk_forward_timed` (CUDA events between them, stream synchronised on return) and the dict
        receives {stage: {"ms": device ms, "launches": n}}."""
        _cuda(ids, "ids")
        if ids.dtype != torch.int32:
            raise ValueError("minicpm5_mk: ids must be int32")
        if ids.numel() < bs * seq:
            raise ValueError("minicpm5_mk: fewer ids than bs * seq")
        ws = self._workspace(bs, seq)
        if out is not None:
            hid, lg, top1 = out
        else:
            hid = torch.empty((bs, self.cfg.hidden), dtype=torch.bfloat16, device=self.device) if hidden else None
            lg = torch.empty((bs, self.cfg.vocab), dtype=torch.float32, device=self.device) if logits else None
            top1 = torch.empty((bs,), dtype=torch.int32, device=self.device)
        if stage_times is None:
            st = _lib.lib().mk_forward(self._h, ids.data_ptr(), bs, seq, ws.data_ptr(), ws.numel(), _ptr(hid),
                                       _ptr(lg), top1.data_ptr(), _stream(self.device))
            _lib.check(st, "mk_forward")
        else:
            t = _lib.MkStageTimesC()
            st = _lib.lib().mk_forward_timed(self._h, ids.data_ptr(), bs, seq, ws.data_ptr(), ws.numel(), _ptr(hid),
                                             _ptr(lg), top1.data_ptr(), _stream(self.device), ctypes.byref(t))
            _lib.check(st, "mk_forward_timed")
            stage_times.clear()
            for i, name in enumerate(_lib.MK_STAGE_NAMES):
                stage_times[name] = {"ms": float(t.ms[i]), "launches": int(t.launches[i])}
        return hid, lg, top1

    # ------------------------------------------------------------------ sequence parallelism
    def sp_block(self, seq: int, world: int) -> int:
        return int(_lib.lib().mk_sp_block(self._h, seq, world))

    def set_sp_key_split(self, enabled: bool) -> None:
        """mk_set_sp_key_split: let forward_sp cut long causal key ranges over several attention CTAs (the
        default); disabled, forward_sp is bit-identical to forward."""
        _lib.check(_lib.lib().mk_set_sp_key_split(self._h, 1 if enabled else 0), "mk_set_sp_key_split")

    def sp_workspace(self, seq: int, world: int) -> torch.Tensor:
        """The workspace mk_forward_sp uses (shared with `forward`'s): bind the all-gather callback to it."""
        n = ctypes.c_size_t()
        _lib.check(_lib.lib().mk_workspace_size_sp(self._h, seq, world, ctypes.byref(n)), "mk_workspace_size_sp")
        if self._ws is None or self._ws.numel() < n.value:
            self._ws = None
            self._ws = torch.empty(int(n.value), dtype=torch.uint8, device=self.device)
        return self._ws

    def forward_sp(self, ids: torch.Tensor, seq: int, rank: int, world: int, gather_for, *,
                   out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
                   stage_times: Optional[dict] = None):
        """Sequence-parallel forward of one sequence through `mk_forward_sp`.  `ids`: int32 [seq] (the whole
        sequence, on every rank).  `gather_for(workspace)` returns the all-gather the library calls,
        `gather(send_ptr, recv_ptr, bytes_per_rank, stream) -> 0`, over that uint8 workspace tensor
        (minicpm5_mk.sp.nccl_allgather / ThreadGroup build them).  Returns (hidden, logits, top1) as
        `forward` with bs = 1; they are written on rank 0 only."""
        _cuda(ids, "ids")
        if ids.dtype != torch.int32 or ids.numel() < seq:
            raise ValueError("minicpm5_mk: ids must be int32 with at least seq entries")
        ws = self.sp_workspace(seq, world)
        gather = gather_for(ws)
        if out is not None:
            hid, lg, top1 = out
        else:
            hid = torch.empty((1, self.cfg.hidden), dtype=torch.bfloat16, device=self.device)
            lg = torch.empty((1, self.cfg.vocab), dtype=torch.float32, device=self.device)
            top1 = torch.empty((1,), dtype=torch.int32, device=self.device)
        failure = []

        def cb(ctx, send, recv, nbytes, stream):
            try:
                return int(gather(int(send), int(recv), int(nbytes), int(stream or 0)))
            except BaseException as e:  # an exception must not cross the C frames
                failure.append(e)
                return 1

        fn = _lib.ALLGATHER_FN(cb)
        t = _lib.MkStageTimesC() if stage_times is not None else None
        st = _lib.lib().mk_forward_sp(self._h, ids.data_ptr(), seq, rank, world, fn, None, ws.data_ptr(), ws.numel(),
                                      _ptr(hid), _ptr(lg), top1.data_ptr(), _stream(self.device),
                                      ctypes.byref(t) if t is not None else None)
        if failure:
            raise RuntimeError("minicpm5_mk: sequence-parallel all-gather failed") from failure[0]
        _lib.check(st, "mk_forward_sp")
        if t is not None:
            stage_times.clear()
            for i, name in enumerate(_lib.MK_STAGE_NAMES):
                stage_times[name] = {"ms": float(t.ms[i]), "launches": int(t.launches[i])}
        return hid, lg, top1

    def launches_per_forward(self, bs: int, seq: int) -> int:
        return int(_lib.lib().mk_launches_per_forward(self._h, bs, seq))

    def check_device_error(self) -> int:
        e = ctypes.c_int32()
        st = _lib.lib().mk_get_error(self._h, ctypes.byref(e))
        _lib.check(st, f"device error word 0x{e.value:x}")
        return int(e.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().mk_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


# ----------------------------------------------------------------------------------- per-stage ops
def gemm_w8a16(a: torch.Tensor, w: torch.Tensor, col_scale: torch.Tensor, mode: int,
               row_scale: Optional[torch.Tensor] = None, resid_scale: float = 1.0,
               out: Optional[torch.Tensor] = None, resid32: Optional[torch.Tensor] = None, *,
               rowsq: Optional[torch.Tensor] = None, rowsq_np: int = 0, norm_dim: int = 0, eps: float = 0.0,
               rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, rope_cols: int = 0, head_dim: int = 0,
               rope_seq: int = 1, rope_pos_base: int = 0) -> torch.Tensor:
    """acc = a @ w^T (a bf16 [M, K], w int8 or bf16 [N, K]) with the epilogue `mode` (see _lib.MK_GEMM_*).
    RESID32 updates the f32 residual `resid32` in place and writes its bf16 copy to `out`.

    The keyword arguments are the forward's fused epilogue work (mk_gemm_w8a16_fused): `rowsq` f32 [M, np]
    per-(token, 128-channel tile) sums of squares, read into rstd by ROWSCALE / SWIGLU when rowsq_np > 0 and
    written by RESID32; `rope` = (cos, sin) tables rotating the pair-ordered columns [0, rope_cols)."""
    for t, n in ((a, "a"), (w, "w"), (col_scale, "col_scale")):
        _cuda(t, n)
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        width = N // 2 if mode == _lib.MK_GEMM_SWIGLU else N
        out = torch.empty((M, width), dtype=torch.bfloat16, device=a.device)
    args = (a.data_ptr(), M, K, a.stride(0), w.data_ptr(), col_scale.data_ptr(), N, mode, _ptr(row_scale),
            float(resid_scale), out.data_ptr(), out.stride(0), _ptr(resid32),
            resid32.stride(0) if resid32 is not None else 0)
    if w.dtype not in (torch.int8, torch.bfloat16):
        raise ValueError("minicpm5_mk: GEMM weights must be int8 or bf16")
    if rowsq is None and rope is None and w.dtype == torch.int8:
        st = _lib.lib().mk_gemm_w8a16(*args, _stream(a.device))
        _lib.check(st, "mk_gemm_w8a16")
        return out
    fu = _lib.MkGemmFusionC()
    fu.weight_bits = 16 if w.dtype == torch.bfloat16 else 8
    if rowsq is not None:
        _cuda(rowsq, "rowsq")
        fu.rowsq, fu.rowsq_ld, fu.rowsq_np, fu.norm_dim, fu.eps = rowsq.data_ptr(), rowsq.stride(0), rowsq_np, \
            norm_dim, eps
    if rope is not None:
        _cuda(rope[0], "rope_cos")
        _cuda(rope[1], "rope_sin")
        fu.rope_cos, fu.rope_sin = rope[0].data_ptr(), rope[1].data_ptr()
        fu.rope_cols, fu.head_dim, fu.rope_seq, fu.rope_pos_base = rope_cols, head_dim, rope_seq, rope_pos_base
    st = _lib.lib().mk_gemm_w8a16_fused(*args, ctypes.byref(fu), _stream(a.device))
    _lib.check(st, "mk_gemm_w8a16_fused")
    return out


def attention_prefill(qkv: torch.Tensor, bs: int, seq: int, n_q: int, n_kv: int, head_dim: int,
                      q_col: int = 0, k_col: Optional[int] = None, v_col: Optional[int] = None,
                      softmax_scale: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _cuda(qkv, "qkv")
    k_col = n_q * head_dim if k_col is None else k_col
    v_col = k_col + n_kv * head_dim if v_col is None else v_col
    if out is None:
        out = torch.empty((bs * seq, n_q * head_dim), dtype=torch.bfloat16, device=qkv.device)
    st = _lib.lib().mk_attention_prefill(qkv.data_ptr(), bs, seq, n_q, n_kv, head_dim, qkv.stride(0), q_col, k_col,
                                         v_col, float(softmax_scale), out.data_ptr(), out.stride(0),
                                         _stream(qkv.device))
    _lib.check(st, "mk_attention_prefill")
    return out


def rope_(x: torch.Tensor, n_heads: int, head_dim: int, cos: torch.Tensor, sin: torch.Tensor, seq: int,
          col0: int = 0, pos_base: int = 0) -> torch.Tensor:
    _cuda(cos, "cos")
    st = _lib.lib().mk_rope(x.data_ptr(), x.shape[0], x.stride(0), col0, n_heads, head_dim, cos.data_ptr(),
                            sin.data_ptr(), seq, pos_base, _stream(x.device))
    _lib.check(st, "mk_rope")
    return x


def rms_rstd(x: torch.Tensor, eps: float) -> torch.Tensor:
    """x: f32 [T, H] residual stream."""
    if x.dtype != torch.float32:
        raise ValueError("minicpm5_mk: rms_rstd expects the f32 residual stream")
    out = torch.empty((x.shape[0],), dtype=torch.float32, device=x.device)
    st = _lib.lib().mk_rms_rstd(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), float(eps), out.data_ptr(),
                                _stream(x.device))
    _lib.check(st, "mk_rms_rstd")
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, scale: float):
    """Returns (x32 f32 [T, H], xb bf16 [T, H])."""
    _cuda(ids, "ids")
    _cuda(table, "embed")
    x32 = torch.empty((ids.numel(), table.shape[1]), dtype=torch.float32, device=ids.device)
    xb = torch.empty((ids.numel(), table.shape[1]), dtype=torch.bfloat16, device=ids.device)
    st = _lib.lib().mk_embed(ids.data_ptr(), ids.numel(), table.data_ptr(), table.shape[0], table.shape[1],
                             float(scale), x32.data_ptr(), xb.data_ptr(), _stream(ids.device))
    _lib.check(st, "mk_embed")
    return x32, xb


def lm_head_argmax(h: torch.Tensor, w: torch.Tensor):
    _cuda(h, "h")
    _cuda(w, "lm_head")
    bs, H = h.shape
    V = w.shape[0]
    P = _lib.lib().mk_lm_head_parts()
    logits = torch.empty((bs, V), dtype=torch.float32, device=h.device)
    pv = torch.empty((bs, P), dtype=torch.float32, device=h.device)
    pi = torch.empty((bs, P), dtype=torch.int32, device=h.device)
    top1 = torch.empty((bs,), dtype=torch.int32, device=h.device)
    st = _lib.lib().mk_lm_head_argmax(h.data_ptr(), bs, H, w.data_ptr(), V, logits.data_ptr(), pv.data_ptr(),
                                      pi.data_ptr(), top1.data_ptr(), _stream(h.device))
    _lib.check(st, "mk_lm_head_argmax")
    return logits, top1


def topk_logprobs(logits: torch.Tensor, k: int = 20):
    """Top-k log-probabilities of each row of f32 logits [bs, V] on the GPU (mk_topk_logprobs):
    (ids int32 [bs, k], logprobs f32 [bs, k]), descending, equal logits -> lower id first.
    The golden's log_softmax + top-k (benchmark/f32_golden.py:100-102)."""
    _cuda(logits, "logits")
    if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-major f32 [bs, V] tensor")
    bs, V = logits.shape
    ids = torch.empty((bs, k), dtype=torch.int32, device=logits.device)
    lps = torch.empty((bs, k), dtype=torch.float32, device=logits.device)
    st = _lib.lib().mk_topk_logprobs(logits.data_ptr(), bs, V, logits.stride(0), k, ids.data_ptr(), lps.data_ptr(),
                                     _stream(logits.device))
    _lib.check(st, "mk_topk_logprobs")
    return ids, lps
