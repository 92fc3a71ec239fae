"""Scoring a checkpoint offline on a B200: load a Hugging Face checkpoint directory
(minicpm5_mk.checkpoint), dump the gate sets' top-20 log-probs in the reference's layout and score them
with the reference's gate (restated in oracle/gate.py).

* Always: the seeded tiny model of a committed golden fixture, written as a checkpoint, against the
  reference's own forward_one dump of it.
* With MINICPM5_CHECKPOINT (a MiniCPM5 checkpoint directory) and MINICPM5_REF_LOGPROBS (the matching
  benchmark/ref/*_logprobs.json of the reference): the real model against the reference's golden.  The
  checkpoints are not part of this repository, so this case is skipped unless both are supplied."""
import json
import os

import pytest
import torch

from ckpt_util import write_checkpoint
from minicpm5_mk import checkpoint, mk_weights
from minicpm5_mk.mk_config import PRESETS
from minicpm5_mk.mk_init import random_state_dict

pytestmark = pytest.mark.gpu


def _engine_from(path, max_seq):
    from minicpm5_mk.ops import MkEngine
    cfg, sd = checkpoint.load_hf_checkpoint(path, device="cuda:0", max_seq=max_seq)
    return MkEngine(cfg, mk_weights.prepare_mk_weights(sd, cfg), "cuda:0")


def test_fixture_checkpoint_passes_reference_gate(golden_dir, tmp_path):
    from oracle.gate import compare_gate
    fx = json.load(open(os.path.join(golden_dir, "golden_f32_tiny96_s256.json")))
    cfg = PRESETS[fx["preset"]].replace(**fx["overrides"])
    write_checkpoint(str(tmp_path), cfg, random_state_dict(cfg, seed=fx["seed"]))
    eng = _engine_from(str(tmp_path), cfg.max_seq)
    ids = fx["prompt_token_ids"]
    sets = [{"batch_size": len(ids), "seq_len": len(ids[0]), "prompt_token_ids": ids}]
    cand = checkpoint.gate_results(eng, sets, k=20)
    ref = [{"batch_size": len(ids), "seq_len": len(ids[0]), "seqs": fx["seqs"]}]
    rep = compare_gate(ref, cand)
    assert rep["gate_v2"] == "PASS", rep
    assert rep["top1_agreement"] == 1.0 and rep["top1_agreement_nolp"] == 1.0
    for s in cand[0]["seqs"]:
        assert s["sampled"] == s["sampled_nolp"] == s["top_ids"][0]


@pytest.mark.skipif(not (os.environ.get("MINICPM5_CHECKPOINT") and os.environ.get("MINICPM5_REF_LOGPROBS")),
                    reason="real checkpoint not supplied (MINICPM5_CHECKPOINT, MINICPM5_REF_LOGPROBS)")
def test_real_checkpoint_passes_reference_gate():
    from oracle.gate import compare_gate
    ref = json.load(open(os.environ["MINICPM5_REF_LOGPROBS"]))
    eng = _engine_from(os.environ["MINICPM5_CHECKPOINT"], max(s["seq_len"] for s in ref["inputs"]))
    cand = checkpoint.gate_results(eng, ref["inputs"], k=int(ref.get("k", 20)))
    rep = compare_gate(ref["results"], cand)
    assert rep["gate_v2"] == "PASS", rep


@pytest.mark.parametrize("preset,layers,wbits", [("minicpm5-1b", 2, 8), ("minicpm5-2b", 1, 8), ("tiny-hd96", None, 16)])
def test_device_weight_preparation_matches_cpu(preset, layers, wbits):
    """prepare_mk_weights on the GPU (what the vLLM class and load_hf_checkpoint(device='cuda') run) gives
    bit-identical int8 weights and scales to the CPU run whose quantiser is pinned against the reference's
    `_quantize_w` (plugin/minicpm5_mk/mk_weights.py:113-123; tests/test_oracle.py), and identical bf16
    weights for weight_bits 16."""
    import time
    cfg = PRESETS[preset].replace(weight_bits=wbits)
    if layers:
        cfg = cfg.replace(num_layers=layers)
    sd = random_state_dict(cfg, seed=99)
    cpu = mk_weights.prepare_mk_weights(sd, cfg)
    sd_dev = {k: v.to("cuda:0") for k, v in sd.items()}
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dev = mk_weights.prepare_mk_weights(sd_dev, cfg)
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert set(cpu) == set(dev)
    for k in cpu:
        assert dev[k].is_cuda, k
        assert cpu[k].dtype == dev[k].dtype, k
        assert torch.equal(cpu[k], dev[k].cpu()), k
    print(f"{preset} x{cfg.num_layers} layers: device preparation {took:.3f} s")
