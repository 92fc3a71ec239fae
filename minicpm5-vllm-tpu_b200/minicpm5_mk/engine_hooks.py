"""vLLM engine hooks for max_tokens=1 scoring batches (host side; the counterparts of the reference's
engine patches, plugin/minicpm5_mk/__init__.py:154-244).

* KV-cache allocation skip (TTVLLM_SKIP_KV_ALLOC_MT1, default on): a fresh, full, max_tokens=1 prefill
  that the megakernel path serves never reads its KV cache, so the scheduler need not hand it blocks.
  Safe only when no stock step can run for this model (MINICPM5_MK_FREE_STOCK=1: an ineligible step
  raises instead of running stock attention without KV), the engine in this process serves the
  megakernel architecture, and the request is a fast-path shape.
* Single-step scheduling (TTVLLM_SINGLE_STEP_MT1, default on): with a batch queue deeper than one,
  vLLM would split a waiting set of max_tokens=1 requests over several overlapped steps; when they all
  fit into one step they are scheduled as one (so a 32 x 8192 batch is one megakernel call).

* Step marker: GPUModelRunner.execute_model is wrapped so the model's forward knows whether it runs in a
  real step or in a dummy run (profile, CUDA-graph warm-up / capture); see RUNNER_STEP.

The predicates are plain functions of the request / scheduler fields, unit-tested on CPU; `install`
wraps the engine classes it is given (vLLM's by default) once.
"""

from __future__ import annotations

import os
from typing import Iterable

from . import ARCH, sampling_fast_ok

ENV_SKIP_KV = "TTVLLM_SKIP_KV_ALLOC_MT1"
ENV_SINGLE_STEP = "TTVLLM_SINGLE_STEP_MT1"

# Whether the engine core of this process serves ARCH (set when an EngineCore is constructed).
ENGINE_SERVES_ARCH = {"active": False, "logged": False}

# Real scheduler steps in progress in this process (GPUModelRunner.execute_model), and whether the marker
# is installed.  The model's forward also runs outside real steps -- the profile run, CUDA-graph warm-up
# and capture -- on dummy batches whose attention metadata can look like any shape; the reference tells
# them apart the same way, by its runner hook setting the step's batch (plugin/minicpm5_mk/model.py:755-794,
# reason "dummy").
RUNNER_STEP = {"depth": 0, "installed": False}


def in_runner_step():
    """True inside a real step, False in a dummy run, None when the marker is not installed."""
    if not RUNNER_STEP["installed"]:
        return None
    return RUNNER_STEP["depth"] > 0


def install_step_marker(runner_cls) -> None:
    if getattr(runner_cls, "_minicpm5_step_marked", False):
        return
    orig = runner_cls.execute_model

    def execute_model(self, *args, **kwargs):
        RUNNER_STEP["depth"] += 1
        try:
            return orig(self, *args, **kwargs)
        finally:
            RUNNER_STEP["depth"] -= 1

    runner_cls.execute_model = execute_model
    runner_cls._minicpm5_step_marked = True
    RUNNER_STEP["installed"] = True


def fast_path_length(seq: int) -> bool:
    """Prompt lengths the fast path takes (plugin/minicpm5_mk/__init__.py:191): multiples of 128 up to
    1024, multiples of 1024 above."""
    return seq > 0 and ((seq <= 1024 and seq % 128 == 0) or seq % 1024 == 0)


def kv_skip_eligible(request, num_new_tokens: int, serves_arch: bool, env=os.environ) -> bool:
    """True iff allocate_slots may hand `request` no KV blocks (plugin/minicpm5_mk/__init__.py:180-195)."""
    sp = getattr(request, "sampling_params", None)
    return bool(
        serves_arch
        and env.get("MINICPM5_MK_ENABLE", "1") != "0"
        and env.get("MINICPM5_MK_FREE_STOCK", "0") == "1"
        and request.num_computed_tokens == 0
        and sp is not None
        and sp.max_tokens == 1
        and num_new_tokens == request.num_prompt_tokens
        and sampling_fast_ok(sp)
        and fast_path_length(request.num_prompt_tokens))


def single_step_eligible(batch_queue, batch_queue_size: int, running: Iterable, waiting: Iterable,
                         max_running: int, max_scheduled_tokens: int) -> bool:
    """True iff the waiting requests are all max_tokens=1, nothing is running or queued, and they fit in
    one step (plugin/minicpm5_mk/__init__.py:213-233)."""
    if batch_queue is None or len(batch_queue) or batch_queue_size <= 1:
        return False
    waiting = list(waiting)
    if list(running) or not waiting or len(waiting) > max_running:
        return False
    tot = 0
    for r in waiting:
        sp = getattr(r, "sampling_params", None)
        if sp is None or sp.max_tokens != 1:
            return False
        tot += r.num_prompt_tokens
    return 0 < tot <= max_scheduled_tokens


def _archs(vllm_config) -> list:
    mc = vllm_config.model_config
    return list(getattr(mc, "architectures", None) or []) + list(getattr(mc.hf_config, "architectures", None) or [])


def install_kv_skip(kv_cache_manager_cls, engine_core_cls) -> None:
    if not getattr(engine_core_cls, "_minicpm5_arch_hooked", False):
        orig_init = engine_core_cls.__init__

        def __init__(self, vllm_config, *args, **kwargs):
            try:
                ENGINE_SERVES_ARCH["active"] = ARCH in _archs(vllm_config)
            except Exception:  # noqa: BLE001 - an unexpected config shape disables the skip
                ENGINE_SERVES_ARCH["active"] = False
            return orig_init(self, vllm_config, *args, **kwargs)

        engine_core_cls.__init__ = __init__
        engine_core_cls._minicpm5_arch_hooked = True
    if not getattr(kv_cache_manager_cls, "_minicpm5_mt1_hooked", False):
        orig_alloc = kv_cache_manager_cls.allocate_slots

        def allocate_slots(self, request, num_new_tokens, *args, **kwargs):
            if kv_skip_eligible(request, num_new_tokens, ENGINE_SERVES_ARCH["active"]):
                if not ENGINE_SERVES_ARCH["logged"]:
                    ENGINE_SERVES_ARCH["logged"] = True
                    print("[minicpm5_mk] KV-cache allocation skipped for fast-path max_tokens=1 requests "
                          "(MINICPM5_MK_FREE_STOCK=1)", flush=True)
                return self.empty_kv_cache_blocks
            return orig_alloc(self, request, num_new_tokens, *args, **kwargs)

        kv_cache_manager_cls.allocate_slots = allocate_slots
        kv_cache_manager_cls._minicpm5_mt1_hooked = True


def install_single_step(engine_core_cls) -> None:
    if getattr(engine_core_cls, "_minicpm5_single_step_hooked", False):
        return
    orig_step = engine_core_cls.step_with_batch_queue

    def step_with_batch_queue(self):
        s = self.scheduler
        if single_step_eligible(self.batch_queue, self.batch_queue_size, s.running, s.waiting,
                                s.max_num_running_reqs, s.max_num_scheduled_tokens):
            saved = self.batch_queue_size
            self.batch_queue_size = 1
            try:
                return orig_step(self)
            finally:
                self.batch_queue_size = saved
        return orig_step(self)

    engine_core_cls.step_with_batch_queue = step_with_batch_queue
    engine_core_cls._minicpm5_single_step_hooked = True


def install(env=os.environ) -> None:
    """Install the enabled hooks on vLLM's engine classes (no-op where vLLM lacks them)."""
    try:
        from vllm.v1.core.kv_cache_manager import KVCacheManager
        from vllm.v1.engine.core import EngineCore
    except Exception:  # noqa: BLE001 - a vLLM without the v1 engine: nothing to hook
        return
    if env.get(ENV_SKIP_KV, "1") == "1" and hasattr(KVCacheManager, "allocate_slots"):
        install_kv_skip(KVCacheManager, EngineCore)
    if env.get(ENV_SINGLE_STEP, "1") == "1" and hasattr(EngineCore, "step_with_batch_queue"):
        install_single_step(EngineCore)
    try:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except Exception:  # noqa: BLE001 - no GPU runner in this vLLM: forward falls back to its metadata checks
        return
    if hasattr(GPUModelRunner, "execute_model"):
        install_step_marker(GPUModelRunner)
