"""Whole-model parity on a B200: mk_forward through the C ABI against
  * the CPU numerics mirror (oracle/mirror.py): same design, tight tolerance;
  * the FP32 golden restatement (oracle/golden.py): the accuracy bar -- identical top-1,
    last-token logits cosine >= 0.999 and max-abs error <= 2e-2 x logit range."""
import json
import os

import pytest
import torch

from minicpm5_mk.mk_config import PRESETS
from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
from minicpm5_mk import mk_weights

pytestmark = pytest.mark.gpu

COS_MIN = 0.999
MAXABS_FRAC = 2e-2


def _engine(cfg, sd):
    from minicpm5_mk.ops import MkEngine
    pw = mk_weights.prepare_mk_weights(sd, cfg)
    return MkEngine(cfg, pw, "cuda:0"), pw


def _assert_bar(ref, got, what):
    cos = torch.nn.functional.cosine_similarity(ref.double(), got.double(), dim=0).item()
    rng = (ref.max() - ref.min()).item()
    mad = (ref - got).abs().max().item()
    assert cos >= COS_MIN, (what, cos)
    assert mad <= MAXABS_FRAC * rng, (what, mad, rng)
    return cos, mad / rng


@pytest.mark.parametrize("preset,bs,S", [("tiny-hd96", 2, 256), ("tiny-hd128", 1, 384), ("tiny-hd96", 3, 1024)])
def test_forward_tiny(preset, bs, S):
    from oracle import golden, mirror
    cfg = PRESETS[preset]
    sd = random_state_dict(cfg, seed=1234)
    eng, pw = _engine(cfg, sd)
    ids = synthetic_ids(bs, S, seed=7, vocab=cfg.vocab)
    hid, lg, top1 = eng.forward(ids.reshape(-1).contiguous().cuda(), bs, S)
    torch.cuda.synchronize()
    assert eng.check_device_error() == 0
    lg, top1, hid = lg.cpu(), top1.cpu(), hid.float().cpu()
    lm, hm = mirror.mirror_forward(ids, pw, cfg)
    W = golden.golden_weights(sd, cfg)
    for b in range(bs):
        # design mirror: bf16-resolution agreement
        cos = torch.nn.functional.cosine_similarity(lm[b].double(), lg[b].double(), dim=0).item()
        assert cos > 0.99995, cos
        assert (hm[b] - hid[b]).abs().max().item() < 0.05 * hm[b].abs().max().item()
        # FP32 golden: the accuracy bar
        lgold = golden.forward_logits(ids[b], W, cfg)
        _assert_bar(lgold, lg[b], f"{preset} seq {b}")
        assert int(top1[b]) == golden.argmax_first(lgold)
        # argmax indexing exact w.r.t. the returned logits
        assert int(top1[b]) == int(torch.argmax(lg[b]))


def test_forward_batch_invariance():
    """Same sequence alone and inside a batch gives the same logits (the reference checks batch
    invariance of top-1, benchmark/run_benchmark.py:716-727)."""
    cfg = PRESETS["tiny-hd96"]
    eng, _ = _engine(cfg, random_state_dict(cfg, seed=1234))
    ids = synthetic_ids(4, 256, seed=9, vocab=cfg.vocab)
    _, lg4, t4 = eng.forward(ids.reshape(-1).contiguous().cuda(), 4, 256)
    _, lg1, t1 = eng.forward(ids[2].contiguous().cuda(), 1, 256)
    torch.cuda.synchronize()
    assert torch.equal(lg4[2].cpu(), lg1[0].cpu())
    assert int(t4[2]) == int(t1[0])


def test_forward_timed_matches_forward():
    """mk_forward_timed runs the same launches as mk_forward (bit-identical outputs), counts every launch
    once and charges positive device time to each stage."""
    cfg = PRESETS["tiny-hd96"]
    eng, _ = _engine(cfg, random_state_dict(cfg, seed=1234))
    bs, S = 2, 256
    ids = synthetic_ids(bs, S, seed=11, vocab=cfg.vocab).reshape(-1).contiguous().cuda()
    h0, l0, t0 = eng.forward(ids, bs, S)
    stages = {}
    h1, l1, t1 = eng.forward(ids, bs, S, stage_times=stages)
    torch.cuda.synchronize()
    assert torch.equal(h0, h1) and torch.equal(l0, l1) and torch.equal(t0, t1)
    assert sum(v["launches"] for v in stages.values()) == eng.launches_per_forward(bs, S)
    L = cfg.num_layers
    for name in ("qkv", "attn", "o_proj", "gate_up", "down"):
        assert stages[name]["launches"] == L - 1, (name, stages[name])
    assert stages["last_layer"]["launches"] == 7
    assert stages["kv_gather"] == {"ms": 0.0, "launches": 0}  # sequence-parallel only
    assert all(v["ms"] > 0 for k, v in stages.items() if k != "kv_gather"), stages


def test_forward_1b_s1024_vs_golden():
    from oracle import golden
    cfg = PRESETS["minicpm5-1b"]
    sd = random_state_dict(cfg, seed=1234)
    eng, _ = _engine(cfg, sd)
    ids = synthetic_ids(1, 1024, seed=1234)
    _, lg, top1 = eng.forward(ids.reshape(-1).contiguous().cuda(), 1, 1024)
    torch.cuda.synchronize()
    assert eng.check_device_error() == 0
    W = golden.golden_weights(sd, cfg)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    lgold = golden.forward_logits(ids[0], W, cfg)
    _assert_bar(lgold, lg[0].cpu(), "1b s1024")
    assert int(top1[0]) == golden.argmax_first(lgold)


def test_forward_1b_s8192_vs_committed_golden(golden_dir):
    """Full BASELINE config 1 shape (1 x 8192, 24 layers) against the committed FP32 golden fixture
    (tests/golden/make_golden_1b.py)."""
    path = os.path.join(golden_dir, "golden_1b_s8192.json")
    fx = json.load(open(path))
    cfg = PRESETS[fx["preset"]]
    sd = random_state_dict(cfg, seed=fx["seed"])
    eng, _ = _engine(cfg, sd)
    ids = torch.tensor(fx["prompt_token_ids"], dtype=torch.int32)
    _, lg, top1 = eng.forward(ids.reshape(-1).contiguous().cuda(), 1, ids.shape[1])
    torch.cuda.synchronize()
    assert eng.check_device_error() == 0
    lg = lg[0].cpu()
    assert int(top1[0]) == fx["top1"]
    sel = torch.tensor(fx["probe_ids"])
    ref = torch.tensor(fx["probe_logits"])
    got = lg[sel]
    cos = torch.nn.functional.cosine_similarity(ref.double(), got.double(), dim=0).item()
    assert cos >= COS_MIN, cos
    assert (ref - got).abs().max().item() <= MAXABS_FRAC * fx["logit_range"]
    assert abs((lg.max() - lg.min()).item() - fx["logit_range"]) <= MAXABS_FRAC * fx["logit_range"]


@pytest.mark.parametrize("name", ["tiny96_s256", "tiny128_s384"])
def test_forward_topk_passes_reference_gate(golden_dir, name):
    """GPU forward + GPU top-20 log-probs scored against the reference's own forward_one top-20 dump
    with the reference's gate (restated in oracle/gate.py, pinned on its reports): gate v2 PASS and
    top-1 agreement 1.0."""
    from minicpm5_mk import ops
    from oracle.gate import compare_gate
    fx = json.load(open(os.path.join(golden_dir, f"golden_f32_{name}.json")))
    cfg = PRESETS[fx["preset"]].replace(**fx["overrides"])
    eng, _ = _engine(cfg, random_state_dict(cfg, seed=fx["seed"]))
    ids = torch.tensor(fx["prompt_token_ids"], dtype=torch.int32)
    bs, S = ids.shape
    _, lg, top1 = eng.forward(ids.reshape(-1).contiguous().cuda(), bs, S)
    tid, tlp = ops.topk_logprobs(lg, 20)
    torch.cuda.synchronize()
    cand = [{"top_ids": tid[b].tolist(), "top_logprobs": tlp[b].tolist()} for b in range(bs)]
    ref = [{"batch_size": bs, "seq_len": S, "seqs": fx["seqs"]}]
    rep = compare_gate(ref, [{"batch_size": bs, "seq_len": S, "seqs": cand}])
    assert rep["gate_v2"] == "PASS", rep
    assert rep["top1_agreement"] == 1.0
    assert all(int(top1[b]) == cand[b]["top_ids"][0] for b in range(bs))
