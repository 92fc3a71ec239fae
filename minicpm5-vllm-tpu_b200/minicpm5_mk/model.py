"""MiniCPM5MegakernelForCausalLM: a vLLM LlamaForCausalLM whose prefill-only scoring steps run the whole
MiniCPM5 forward on the B200 sm_100a kernels (libminicpm5_mk.so through the C ABI).

Reference: `plugin/minicpm5_mk/model.py:554-795`.  Same class name, constructor, `load_weights` and
`forward` contract; every other step (decode, chunked or partial prefill, unequal lengths) runs vLLM's
stock Llama path, so generation stays correct.  A fast-path step calls the registered op
`torch.ops.minicpm5_mk.forward` (minicpm5_mk/torch_op.py, the counterpart of the reference's
`jax_op("minicpm5_mk::forward", ...)`), returns the final-normed hidden rows of each sequence's last token
at that token's position (the rest zero, in one reused buffer), and `compute_logits` hands vLLM's sampler
the library's own last-token logits, so vLLM's lm_head GEMM does not run again for those rows.

Env knobs (reference names, `plugin/minicpm5_mk/model.py:24-32`): MINICPM5_MK_ENABLE ("0" = stock only),
MINICPM5_MK_FREE_STOCK ("1" = drop stock decoder-layer weights, no fallback), MINICPM5_MK_STATUS_DIR,
MINICPM5_MK_LOG_EVERY.
"""

from __future__ import annotations

import json
import os
import time
from collections.abc import Iterable

import torch
from vllm.logger import init_logger
from vllm.model_executor.models.llama import LlamaForCausalLM

from minicpm5_mk import ARCH
from minicpm5_mk.runner import LastRowScatter, batch_from_lengths

logger = init_logger("vllm.minicpm5_mk")

ENV_ENABLE = "MINICPM5_MK_ENABLE"
ENV_FREE_STOCK = "MINICPM5_MK_FREE_STOCK"
ENV_LOG_EVERY = "MINICPM5_MK_LOG_EVERY"
ENV_STATUS_DIR = "MINICPM5_MK_STATUS_DIR"

_WEIGHT_SUFFIXES = (
    "input_layernorm.weight", "post_attention_layernorm.weight",
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
    "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
)


def _batch_from_forward_context(num_tokens: int, max_seq: int):
    """(bs, seq) of the current vLLM step from the attention metadata, or (None, reason)."""
    try:
        from vllm.forward_context import get_forward_context, is_forward_context_available

        if not is_forward_context_available():
            return None, "no-context"
        md = get_forward_context().attn_metadata
    except Exception:  # noqa: BLE001
        return None, "no-context"
    if isinstance(md, list) or not md:
        return None, "dummy"
    m = next(iter(md.values()))
    qsl = getattr(m, "query_start_loc", None)
    sl = getattr(m, "seq_lens", None)
    if qsl is None or sl is None:
        return None, "metadata"
    q = qsl.tolist()
    query_lens = [q[i + 1] - q[i] for i in range(len(q) - 1)]
    return batch_from_lengths(query_lens, sl.tolist()[:len(query_lens)], max_seq, num_tokens)


class MiniCPM5MegakernelForCausalLM(LlamaForCausalLM):
    """LlamaForCausalLM + whole-model B200 megakernel path for prefill-only (max_tokens=1) steps."""

    def __init__(self, *, vllm_config, prefix: str = "", **kwargs):
        super().__init__(vllm_config=vllm_config, prefix=prefix, **kwargs)
        from minicpm5_mk.mk_config import from_hf_config, rope_support

        hf = vllm_config.model_config.hf_config
        self._mk_max_seq = int(vllm_config.model_config.max_model_len)
        self._mk_cfg = from_hf_config(hf, max_seq=max(self._mk_max_seq, 128))
        self._mk_enabled = os.environ.get(ENV_ENABLE, "1") != "0"
        self._mk_engine = None
        self._mk_engine_id = None
        self._mk_scatter = LastRowScatter()
        self._mk_step = None  # (bs, logits) of the forward just served, for compute_logits
        self._mk_entered = False  # forward ran since the last compute_logits (not a CUDA-graph replay)
        self._mk_counts = {"mk": 0, "stock": 0}
        self._mk_log_every = int(os.environ.get(ENV_LOG_EVERY, "0"))
        _, rope_problem = rope_support(hf)  # rope_theta itself is already taken by from_hf_config
        if rope_problem:
            logger.warning("minicpm5_mk: %s; fast path disabled", rope_problem)
            self._mk_enabled = False
        if vllm_config.parallel_config.pipeline_parallel_size != 1 or \
                vllm_config.parallel_config.tensor_parallel_size != 1:
            logger.warning("minicpm5_mk: the fast path runs one full replica per GPU (TP=PP=1); disabled")
            self._mk_enabled = False
        try:
            self._mk_cfg.check()
        except ValueError as e:
            logger.warning("minicpm5_mk: %s; fast path disabled", e)
            self._mk_enabled = False

    # ------------------------------------------------------------------ weights
    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        if not self._mk_enabled:
            return super().load_weights(weights)
        stash: dict[str, torch.Tensor] = {}

        def tee():
            for name, t in weights:
                if (name.startswith("model.layers.") and name.endswith(_WEIGHT_SUFFIXES)) or name in (
                        "model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"):
                    stash[name] = t.detach()
                yield name, t

        loaded = super().load_weights(tee())
        try:
            self._mk_build(stash)
        except Exception:
            if os.environ.get(ENV_FREE_STOCK, "0") == "1":
                logger.exception("minicpm5_mk: build failed and MINICPM5_MK_FREE_STOCK=1")
                raise
            logger.exception("minicpm5_mk: build failed; using the stock path only")
            self._mk_engine = None
        return loaded

    def _mk_build(self, stash: dict[str, torch.Tensor]) -> None:
        from minicpm5_mk import mk_weights, torch_op
        from minicpm5_mk.ops import MkEngine

        t0 = time.perf_counter()
        device = self.lm_head.weight.device
        sd = {k: v.to(device=device, dtype=torch.float32) for k, v in stash.items()}
        pw = mk_weights.prepare_mk_weights(sd, self._mk_cfg)
        del sd
        self._mk_engine = MkEngine(self._mk_cfg, pw, device)
        self._mk_engine_id = torch_op.register_engine(self._mk_engine)
        self._mk_build_s = time.perf_counter() - t0
        logger.info("minicpm5_mk: B200 megakernel ready in %.1fs", self._mk_build_s)
        if os.environ.get(ENV_FREE_STOCK, "0") == "1":
            for layer in self.model.layers:
                for p in layer.parameters():
                    p.data = torch.empty((0,), dtype=p.dtype, device=p.device)
            self._mk_stock_freed = True
        self._mk_status = {"arch": ARCH, "stock_freed": bool(getattr(self, "_mk_stock_freed", False)),
                           "build_s": round(self._mk_build_s, 3), "shapes": {}}
        self._mk_write_status()

    def _mk_write_status(self) -> None:
        d = os.environ.get(ENV_STATUS_DIR)
        if not d or not getattr(self, "_mk_status", None):
            return
        try:
            os.makedirs(d, exist_ok=True)
            path = os.path.join(d, "minicpm5_mk_status_rank0.json")
            with open(path + ".tmp", "w") as f:
                json.dump(self._mk_status, f, indent=1)
            os.replace(path + ".tmp", path)
        except Exception as e:  # noqa: BLE001
            logger.warning("minicpm5_mk: could not write status file: %r", e)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids, positions, intermediate_tensors=None, inputs_embeds=None):
        self._mk_step = None
        self._mk_entered = True
        reason = "disabled"
        from minicpm5_mk.engine_hooks import in_runner_step

        if torch.cuda.is_current_stream_capturing():
            # CUDA-graph capture of a dummy batch (decode sizes): never the fast path, whose batch shape
            # is decided per step on the host
            reason = "capture"
        elif in_runner_step() is False:
            reason = "dummy"  # profile run / CUDA-graph warm-up: not a scheduler step
        elif (self._mk_engine is not None and input_ids is not None and inputs_embeds is None
                and intermediate_tensors is None):
            batch, reason = _batch_from_forward_context(int(input_ids.shape[0]), self._mk_max_seq)
            if batch is not None:
                bs, seq = batch
                self._mk_counts["mk"] += 1
                key = f"mk:{bs}x{seq}"
                if getattr(self, "_mk_status", None) is not None:
                    shp = self._mk_status["shapes"].setdefault(key, {"mode": "replica", "steps": 0})
                    shp["steps"] += 1
                    self._mk_write_status()  # only with MINICPM5_MK_STATUS_DIR set: one small file per step
                ids = input_ids[:bs * seq].to(torch.int32).contiguous()
                # the registered op (torch.ops.minicpm5_mk.forward -> mk_forward through the C ABI):
                # final-normed last-token rows, their logits and greedy ids
                hid, lg, _ = torch.ops.minicpm5_mk.forward(ids, self._mk_engine_id, bs, seq)
                self._mk_step = (bs, lg)
                return self._mk_scatter(hid, bs, seq, int(input_ids.shape[0]))
        self._mk_counts["stock"] += 1
        st = getattr(self, "_mk_status", None)
        if st is not None and reason != "capture":  # why steps take the stock path
            reasons = st.setdefault("stock_reasons", {})
            reasons[reason] = reasons.get(reason, 0) + 1
            if reasons[reason] == 1:
                self._mk_write_status()
        if getattr(self, "_mk_stock_freed", False):
            if reason in ("dummy", "capture"):
                return torch.zeros((input_ids.shape[0], self._mk_cfg.hidden), dtype=torch.bfloat16,
                                   device=input_ids.device)
            raise RuntimeError(f"minicpm5_mk: stock path needed ({reason}) but stock weights were freed")
        return super().forward(input_ids, positions, intermediate_tensors, inputs_embeds)

    def compute_logits(self, hidden_states, *args, **kwargs):
        """Logits of the sampled rows.  After a fast-path step these are the library's own last-token logits
        (lm_head on the last rows only, computed inside `mk_forward`; the logit scale applied), so vLLM's
        lm_head GEMM does not run again; vLLM's sampler then takes the greedy token from them.  Any other
        step uses the inherited LlamaForCausalLM.compute_logits
        (`vllm:model_executor/models/llama.py:577-582`)."""
        step, self._mk_step = self._mk_step, None
        entered, self._mk_entered = self._mk_entered, False
        if step is not None and hidden_states.shape[0] == step[0]:
            return step[1]
        if not entered and getattr(self, "_mk_stock_freed", False):
            # the step never entered `forward`: a replayed CUDA graph (decode), which with the stock
            # weights freed holds the zeros captured for a dummy batch
            raise RuntimeError("minicpm5_mk: a step ran without the fast path but stock weights were freed")
        return super().compute_logits(hidden_states, *args, **kwargs)
