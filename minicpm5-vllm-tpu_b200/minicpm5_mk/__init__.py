"""vLLM general plugin registering MiniCPM5MegakernelForCausalLM (B200 / sm_100a megakernel path).

Same entry point, architecture string and eligibility predicate as the reference plugin
(`plugin/minicpm5_mk/__init__.py:4-42`, `plugin/pyproject.toml:16-17`):

    [project.entry-points."vllm.general_plugins"]  minicpm5_mk = "minicpm5_mk:register"
    LLM(model, hf_overrides={"architectures": ["MiniCPM5MegakernelForCausalLM"]})
"""

ARCH = "MiniCPM5MegakernelForCausalLM"


def sampling_fast_ok(sp) -> bool:
    """True iff a request's SamplingParams only use features the megakernel fast path implements
    (`plugin/minicpm5_mk/__init__.py:10-32`): no prompt logprobs, penalties, min_p, logit bias, allowed
    or bad words, structured output or custom logits processors."""
    if sp is None:
        return False
    g = getattr
    if g(sp, "prompt_logprobs", None) is not None:
        return False
    if (g(sp, "presence_penalty", 0.0) or 0.0) != 0.0 or (g(sp, "frequency_penalty", 0.0) or 0.0) != 0.0:
        return False
    if (g(sp, "repetition_penalty", 1.0) or 1.0) != 1.0 or (g(sp, "min_p", 0.0) or 0.0) != 0.0:
        return False
    if g(sp, "logit_bias", None) or g(sp, "allowed_token_ids", None) or g(sp, "bad_words", None):
        return False
    if g(sp, "structured_outputs", None) is not None or g(sp, "guided_decoding", None) is not None:
        return False
    if g(sp, "logits_processors", None):
        return False
    return True


def register() -> None:
    """Entry point for the `vllm.general_plugins` group (runs in every vLLM process)."""
    from vllm import ModelRegistry

    if ARCH not in ModelRegistry.get_supported_archs():
        ModelRegistry.register_model(ARCH, "minicpm5_mk.model:MiniCPM5MegakernelForCausalLM")
    # engine hooks for max_tokens=1 scoring batches (plugin/minicpm5_mk/__init__.py:154-244)
    from .engine_hooks import install

    install()
