"""The vLLM engine hooks for max_tokens=1 scoring batches (minicpm5_mk/engine_hooks.py), on fake engine
classes: KV-cache allocation skip and single-step scheduling, with the reference's conditions
(plugin/minicpm5_mk/__init__.py:154-244)."""
from collections import deque
from types import SimpleNamespace

from minicpm5_mk import engine_hooks as eh

FREE = {"MINICPM5_MK_FREE_STOCK": "1"}


def _sp(max_tokens=1, **kw):
    return SimpleNamespace(max_tokens=max_tokens, prompt_logprobs=None, presence_penalty=0.0, frequency_penalty=0.0,
                           repetition_penalty=1.0, min_p=0.0, logit_bias=None, allowed_token_ids=None, bad_words=None,
                           structured_outputs=None, logits_processors=None, **kw)


def _req(n=8192, computed=0, sp=None):
    return SimpleNamespace(num_prompt_tokens=n, num_computed_tokens=computed, sampling_params=sp or _sp())


def test_kv_skip_conditions():
    assert eh.kv_skip_eligible(_req(), 8192, True, FREE)
    assert not eh.kv_skip_eligible(_req(), 8192, True, {})                      # stock fallback possible
    assert not eh.kv_skip_eligible(_req(), 8192, False, FREE)                   # engine serves another arch
    assert not eh.kv_skip_eligible(_req(), 8192, True, dict(FREE, MINICPM5_MK_ENABLE="0"))
    assert not eh.kv_skip_eligible(_req(computed=128), 8064, True, FREE)        # not fresh
    assert not eh.kv_skip_eligible(_req(), 4096, True, FREE)                    # chunked prefill
    assert not eh.kv_skip_eligible(_req(sp=_sp(max_tokens=2)), 8192, True, FREE)
    p = _sp()
    p.presence_penalty = 0.5
    assert not eh.kv_skip_eligible(_req(sp=p), 8192, True, FREE)               # sampling the fast path lacks
    assert eh.kv_skip_eligible(_req(n=384), 384, True, FREE)
    assert not eh.kv_skip_eligible(_req(n=1536), 1536, True, FREE)             # not a fast-path length


def test_single_step_conditions():
    w = [_req(), _req()]
    assert eh.single_step_eligible(deque(), 2, [], w, 32, 262144)
    assert not eh.single_step_eligible(deque(), 1, [], w, 32, 262144)           # no batch queue depth
    assert not eh.single_step_eligible(deque([0]), 2, [], w, 32, 262144)        # queue busy
    assert not eh.single_step_eligible(deque(), 2, [w[0]], w, 32, 262144)       # something running
    assert not eh.single_step_eligible(deque(), 2, [], w, 1, 262144)            # too many requests
    assert not eh.single_step_eligible(deque(), 2, [], w, 32, 8192)             # does not fit one step
    assert not eh.single_step_eligible(deque(), 2, [], [_req(sp=_sp(max_tokens=4))], 32, 262144)
    assert not eh.single_step_eligible(None, 2, [], w, 32, 262144)


def test_installed_hooks_on_fake_engine(monkeypatch):
    monkeypatch.setenv("MINICPM5_MK_FREE_STOCK", "1")

    class Mgr:
        empty_kv_cache_blocks = "EMPTY"

        def allocate_slots(self, request, num_new_tokens, *a, **k):
            return "BLOCKS"

    class Core:
        def __init__(self, vllm_config):
            self.batch_queue = deque(maxlen=2)
            self.batch_queue_size = 2
            self.scheduler = SimpleNamespace(running=[], waiting=[_req()], max_num_running_reqs=32,
                                             max_num_scheduled_tokens=262144)
            self.seen = []

        def step_with_batch_queue(self):
            self.seen.append(self.batch_queue_size)
            return "STEP"

    eh.install_kv_skip(Mgr, Core)
    eh.install_single_step(Core)
    eh.install_kv_skip(Mgr, Core)  # idempotent
    cfg = SimpleNamespace(model_config=SimpleNamespace(architectures=["MiniCPM5MegakernelForCausalLM"],
                                                       hf_config=SimpleNamespace(architectures=[])))
    core = Core(cfg)
    assert eh.ENGINE_SERVES_ARCH["active"]
    assert Mgr().allocate_slots(_req(), 8192) == "EMPTY"
    assert Mgr().allocate_slots(_req(), 4096) == "BLOCKS"
    assert core.step_with_batch_queue() == "STEP" and core.seen == [1] and core.batch_queue_size == 2
    core.scheduler.waiting = [_req(sp=_sp(max_tokens=3))]
    core.step_with_batch_queue()
    assert core.seen == [1, 2]
    other = SimpleNamespace(model_config=SimpleNamespace(architectures=["LlamaForCausalLM"],
                                                         hf_config=SimpleNamespace(architectures=[])))
    Core(other)
    assert not eh.ENGINE_SERVES_ARCH["active"]
    assert Mgr().allocate_slots(_req(), 8192) == "BLOCKS"


def test_step_marker_tells_real_steps_from_dummy_runs():
    """Forward calls inside the runner's execute_model are real steps; the profile run and CUDA-graph
    warm-up call the model outside it (the reference's "dummy" reason)."""
    seen = []

    class FakeRunner:
        def execute_model(self, scheduler_output):
            seen.append(eh.in_runner_step())
            return "out"

        def dummy_run(self):
            seen.append(eh.in_runner_step())

    saved = dict(eh.RUNNER_STEP)
    try:
        eh.RUNNER_STEP.update(depth=0, installed=False)
        assert eh.in_runner_step() is None
        eh.install_step_marker(FakeRunner)
        eh.install_step_marker(FakeRunner)  # once only
        r = FakeRunner()
        r.dummy_run()
        assert r.execute_model(None) == "out"
        r.dummy_run()
        assert seen == [False, True, False]
        assert eh.RUNNER_STEP["depth"] == 0
    finally:
        eh.RUNNER_STEP.update(saved)
