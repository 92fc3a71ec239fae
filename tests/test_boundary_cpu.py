"""The drop-in boundary on CPU: plugin entry point, eligibility predicate, batch detection and the
row layout handed back to vLLM (no GPU, no kernel calls)."""
import importlib.metadata as md
import types

import pytest
import torch

from minicpm5_mk import ARCH, sampling_fast_ok
from minicpm5_mk.runner import batch_from_lengths, mk_seq_ok, scatter_last


def test_entry_point_is_discoverable():
    eps = md.entry_points(group="vllm.general_plugins")
    names = {e.name: e.value for e in eps}
    assert names.get("minicpm5_mk") == "minicpm5_mk:register"
    assert ARCH == "MiniCPM5MegakernelForCausalLM"


def _sp(**kw):
    base = dict(prompt_logprobs=None, presence_penalty=0.0, frequency_penalty=0.0, repetition_penalty=1.0,
                min_p=0.0, logit_bias=None, allowed_token_ids=None, bad_words=None, structured_outputs=None,
                logits_processors=None, max_tokens=1, temperature=0.0)
    base.update(kw)
    return types.SimpleNamespace(**base)


@pytest.mark.parametrize("kw,ok", [
    ({}, True), ({"prompt_logprobs": 5}, False), ({"presence_penalty": 0.5}, False),
    ({"repetition_penalty": 1.1}, False), ({"min_p": 0.1}, False), ({"logit_bias": {1: 2.0}}, False),
    ({"allowed_token_ids": [1]}, False), ({"bad_words": ["x"]}, False), ({"structured_outputs": object()}, False),
    ({"logits_processors": [abs]}, False), ({"temperature": 0.7}, True),
])
def test_sampling_fast_ok(kw, ok):
    assert sampling_fast_ok(_sp(**kw)) is ok
    assert sampling_fast_ok(None) is False


def test_seq_ok_matches_reference_rule():
    # plugin/minicpm5_mk/model.py:131-136
    assert mk_seq_ok(128, 8192) and mk_seq_ok(1024, 8192) and mk_seq_ok(8192, 8192)
    assert not mk_seq_ok(100, 8192) and not mk_seq_ok(1152, 8192) and not mk_seq_ok(9216, 8192)
    assert mk_seq_ok(2048, 8192) and not mk_seq_ok(0, 8192)


def test_batch_from_lengths():
    assert batch_from_lengths([8192] * 4, [8192] * 4, 8192, 32768) == ((4, 8192), "ok")
    assert batch_from_lengths([8192, 4096], [8192, 4096], 8192, 12288)[0] is None
    assert batch_from_lengths([1], [8193], 8192, 1)[1] == "not-fresh"       # decode step
    assert batch_from_lengths([100], [100], 8192, 100)[1] == "length"
    assert batch_from_lengths([], [], 8192, 0)[1] == "empty"
    assert batch_from_lengths([1024] * 2, [1024] * 2, 8192, 1024)[1] == "tokens"


def test_scatter_last_layout():
    h = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    out = scatter_last(h, 2, 4, 10)
    assert out.shape == (10, 3)
    assert torch.equal(out[3], h[0]) and torch.equal(out[7], h[1])
    assert out.abs().sum() == h.abs().sum()


@pytest.mark.slow
def test_model_class_subclasses_vllm_llama():
    from vllm.model_executor.models.llama import LlamaForCausalLM
    from minicpm5_mk.model import MiniCPM5MegakernelForCausalLM
    assert issubclass(MiniCPM5MegakernelForCausalLM, LlamaForCausalLM)


def test_last_row_scatter_reuses_one_buffer():
    """The reused buffer gives exactly scatter_last's layout step after step (shapes shrinking and
    growing), zeroing the rows of the previous step."""
    from minicpm5_mk.runner import LastRowScatter
    sc = LastRowScatter()
    g = torch.Generator().manual_seed(0)
    ptr, cap = None, 0
    for bs, seq, t_pad in [(2, 4, 10), (3, 2, 8), (1, 8, 8), (2, 4, 9), (4, 4, 20), (1, 4, 4), (2, 8, 16)]:
        h = torch.randn((bs, 6), generator=g).to(torch.bfloat16)
        out = sc(h, bs, seq, t_pad)
        assert torch.equal(out, scatter_last(h, bs, seq, t_pad)), (bs, seq, t_pad)
        if t_pad <= cap:
            assert sc.buf.data_ptr() == ptr  # no new allocation while the buffer is large enough
        ptr, cap = sc.buf.data_ptr(), sc.buf.shape[0]
