"""CPU oracle checks: the restatement of the reference's FP32 golden path against fixtures made by
running the reference's own code (tests/golden/make_golden.py)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import golden
from minicpm5_mk.mk_config import PRESETS
from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
from minicpm5_mk import mk_weights


@pytest.mark.parametrize("name", ["tiny96_s256", "tiny96_s1152", "tiny128_s384"])
def test_oracle_matches_reference_f32_golden(golden_dir, name):
    fx = json.load(open(os.path.join(golden_dir, f"golden_f32_{name}.json")))
    cfg = PRESETS[fx["preset"]].replace(**fx["overrides"])
    sd = random_state_dict(cfg, seed=fx["seed"])
    W = golden.golden_weights(sd, cfg)
    ids = torch.tensor(fx["prompt_token_ids"], dtype=torch.int32)
    for b, ref in enumerate(fx["seqs"]):
        tid, tlp = golden.forward_one(ids[b], W, cfg, k=20)
        assert tid[0] == ref["top_ids"][0]
        rmap = dict(zip(ref["top_ids"], ref["top_logprobs"]))
        common = [t for t in tid if t in rmap]
        assert len(common) >= 18
        cmap = dict(zip(tid, tlp))
        err = max(abs(cmap[t] - rmap[t]) for t in common)
        assert err < 2e-4, err


def test_ids_are_reproducible():
    a = synthetic_ids(2, 64, seed=1234)
    b = synthetic_ids(2, 64, seed=1234)
    assert torch.equal(a, b)
    assert int(a.min()) >= 1000 and int(a.max()) < 30000


def test_quantizer_matches_reference(golden_dir):
    z = np.load(os.path.join(golden_dir, "quantize_w.npz"))
    for i in range(3):
        w = torch.from_numpy(z[f"w{i}"])           # reference layout [in, out]
        q, s = mk_weights.quantize_per_out_channel(w.T)  # ours: [out, in]
        assert np.array_equal(q.T.numpy(), z[f"q{i}"])
        assert np.array_equal(s.numpy(), z[f"s{i}"])


def test_gu_interleave_roundtrip():
    g = torch.arange(512 * 3).reshape(512, 3)
    u = -g
    x = mk_weights.interleave_gu(g, u)
    assert torch.equal(x[0::2], g) and torch.equal(x[1::2], u)  # row 2i = gate i, row 2i+1 = up i
    g2, u2 = mk_weights.deinterleave_gu(x)
    assert torch.equal(g2, g) and torch.equal(u2, u)
    x64 = mk_weights.interleave_gu(g, u, block=64)
    assert torch.equal(x64[:64], g[:64]) and torch.equal(x64[64:128], u[:64])
    g2, u2 = mk_weights.deinterleave_gu(x64, block=64)
    assert torch.equal(g2, g) and torch.equal(u2, u)


def test_rope_table_matches_golden_formula():
    cfg = PRESETS["tiny-hd96"]
    c, s = mk_weights.rope_tables(300, cfg.head_dim, cfg.rope_theta)
    gc, gs = golden.rope_tables(300, cfg.head_dim, cfg.rope_theta)
    half = cfg.head_dim // 2
    assert torch.equal(c, gc[:, :half]) and torch.equal(c, gc[:, half:])
    assert torch.equal(s, gs[:, :half])


@pytest.mark.parametrize("preset,S", [("tiny-hd96", 256), ("tiny-hd128", 384)])
def test_mirror_tracks_golden(preset, S):
    """The int8 weight-only / bf16-activation design stays within the accuracy bar of the FP32 golden."""
    from oracle import mirror
    cfg = PRESETS[preset]
    sd = random_state_dict(cfg, seed=1234)
    pw = mk_weights.prepare_mk_weights(sd, cfg)
    W = golden.golden_weights(sd, cfg)
    ids = synthetic_ids(2, S, seed=3, vocab=cfg.vocab)
    lg_m, _ = mirror.mirror_forward(ids, pw, cfg)
    for b in range(2):
        lg_g = golden.forward_logits(ids[b], W, cfg)
        cos = torch.nn.functional.cosine_similarity(lg_g, lg_m[b], dim=0).item()
        rng = (lg_g.max() - lg_g.min()).item()
        assert cos >= 0.999, cos
        assert (lg_g - lg_m[b]).abs().max().item() <= 2e-2 * rng


def test_design_meets_accuracy_bar_1b_s1024():
    """The numerics design (int8 weight-only, f32 residual stream, bf16 activations), evaluated by the
    CPU mirror on the full 1B config at 1024 tokens, meets the accuracy bar against the FP32 golden."""
    from oracle import mirror
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    cfg = PRESETS["minicpm5-1b"]
    sd = random_state_dict(cfg, seed=1234)
    pw = mk_weights.prepare_mk_weights(sd, cfg)
    ids = synthetic_ids(1, 1024, seed=1234)
    lg_m, _ = mirror.mirror_forward(ids, pw, cfg)
    lg_g = golden.forward_logits(ids[0], golden.golden_weights(sd, cfg), cfg)
    cos = torch.nn.functional.cosine_similarity(lg_g.double(), lg_m[0].double(), dim=0).item()
    rng = (lg_g.max() - lg_g.min()).item()
    assert cos >= 0.999
    assert (lg_g - lg_m[0]).abs().max().item() <= 2e-2 * rng
    assert golden.argmax_first(lg_g) == golden.argmax_first(lg_m[0])


def test_gate_scorer_matches_reference_reports(golden_dir):
    """oracle/gate.py against the reference's own compare_gate reports (PASS, JUDGE and FAIL verdicts,
    with and without a no-logprobs sampled token): every field identical."""
    from oracle.gate import compare_gate
    cases = json.load(open(os.path.join(golden_dir, "gate_cases.json")))
    verdicts = set()
    for c in cases:
        assert compare_gate(c["ref"], c["cand"]) == c["report"]
        verdicts.add(c["report"]["gate_v2"])
    assert verdicts == {"PASS", "JUDGE", "FAIL"}
