"""Generate the committed golden fixtures under tests/golden/ from the reference's own code.

Run in the build container (it reads the reference sources, which do not exist on the GPU box):

    python tests/golden/make_golden.py --reference <reference checkout>

1. `f32_golden.forward_one` (benchmark/f32_golden.py:78-102) of the reference, executed with the
   numpy stand-in for jax under tests/golden/jax_shim, on small seeded random-init models
   (muP scalars off: the reference golden is plain Llama).  Records the top-20 ids/logprobs and the
   gate inputs.  -> golden_f32_<name>.json
2. `_quantize_w` (plugin/minicpm5_mk/mk_weights.py:113-123) of the reference on seeded matrices.
   -> quantize_w.npz
3. `compare_gate` (benchmark/gate.py:16-121) of the reference on synthetic top-20 dumps.
   -> gate_cases.json
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "minicpm5-vllm-tpu_b200"))

from minicpm5_mk.mk_config import PRESETS  # noqa: E402
from minicpm5_mk.mk_init import random_state_dict, synthetic_ids  # noqa: E402

# (fixture name, preset, overrides, seq_len, batch of prompts)
F32_CASES = [
    ("tiny96_s256", "tiny-hd96", dict(scale_emb=1.0, residual_scale=1.0, logit_scale=1.0), 256, 2),
    ("tiny96_s1152", "tiny-hd96", dict(scale_emb=1.0, residual_scale=1.0, logit_scale=1.0), 1152, 1),
    ("tiny128_s384", "tiny-hd128", dict(), 384, 2),
]


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_f32(ref_root):
    sys.path.insert(0, os.path.join(HERE, "jax_shim"))
    f32g = _load(os.path.join(ref_root, "benchmark", "f32_golden.py"), "ref_f32_golden")
    for name, preset, over, S, nb in F32_CASES:
        cfg = PRESETS[preset].replace(**over)
        sd = random_state_dict(cfg, seed=1234)
        sdn = {k: v.numpy() for k, v in sd.items()}
        put = lambda a: np.asarray(a, np.float32)  # noqa: E731  (f32_golden.py:118)
        W = {"embed": put(sdn["model.embed_tokens.weight"]), "norm": put(sdn["model.norm.weight"]),
             "lm_head": put(sdn["lm_head.weight"].T if "lm_head.weight" in sdn else sdn["model.embed_tokens.weight"].T),
             "layers": []}
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            W["layers"].append({
                "in": put(sdn[p + "input_layernorm.weight"]), "post": put(sdn[p + "post_attention_layernorm.weight"]),
                "q": put(sdn[p + "self_attn.q_proj.weight"].T), "k": put(sdn[p + "self_attn.k_proj.weight"].T),
                "v": put(sdn[p + "self_attn.v_proj.weight"].T), "o": put(sdn[p + "self_attn.o_proj.weight"].T),
                "gate": put(sdn[p + "mlp.gate_proj.weight"].T), "up": put(sdn[p + "mlp.up_proj.weight"].T),
                "down": put(sdn[p + "mlp.down_proj.weight"].T),
            })
        rcfg = dict(L=cfg.num_layers, nq=cfg.n_q, nkv=cfg.n_kv, hd=cfg.head_dim, eps=cfg.eps, theta=cfg.rope_theta)
        cos, sin = f32g.rope_tables(S + 64, cfg.head_dim, cfg.rope_theta)
        ids = synthetic_ids(nb, S, seed=20261027, vocab=cfg.vocab).numpy()
        seqs = []
        for b in range(nb):
            tid, tlp = f32g.forward_one(ids[b].astype(np.int32), W, rcfg, cos, sin, k=20)
            seqs.append({"top_ids": [int(t) for t in tid], "top_logprobs": [float(v) for v in tlp]})
        out = {"generator": "reference benchmark/f32_golden.py forward_one via tests/golden/jax_shim",
               "preset": preset, "overrides": over, "seed": 1234, "ids_seed": 20261027,
               "config": cfg.as_dict(), "prompt_token_ids": ids.tolist(), "seqs": seqs}
        with open(os.path.join(HERE, f"golden_f32_{name}.json"), "w") as f:
            json.dump(out, f)
        print(f"[golden] {name}: top1={[s['top_ids'][0] for s in seqs]}")


def make_quant(ref_root):
    mkw = _load(os.path.join(ref_root, "plugin", "minicpm5_mk", "mk_weights.py"), "ref_mk_weights")
    g = torch.Generator().manual_seed(7)
    cases = {}
    for i, (k, n) in enumerate([(64, 48), (384, 128), (257, 31)]):
        w = torch.randn((k, n), generator=g) * 0.02  # reference layout [in, out]
        if i == 2:
            w[:, 3] = 0.0  # all-zero channel: scale clamps to 1e-8
            w[5, 7] = 0.5  # outlier
            w[:, 9] = torch.linspace(-1, 1, k)
        q, s = mkw._quantize_w(w, "int8", 1.0)
        cases[f"w{i}"] = w.numpy()
        cases[f"q{i}"] = q.numpy()
        cases[f"s{i}"] = s.numpy()
    np.savez(os.path.join(HERE, "quantize_w.npz"), **cases)
    print("[golden] quantize_w.npz")


def make_gate(ref_root):
    gate = _load(os.path.join(ref_root, "benchmark", "gate.py"), "ref_gate")
    rng = np.random.default_rng(5)
    cases = []
    # noise levels 0.02..0.08 (PASS), 0.17 (JUDGE), then 0.25 and 1.0 (FAIL); the last two cases
    # also carry a no-logprobs sampled token
    for c, noise_scale in enumerate((0.02, 0.04, 0.06, 0.08, 0.17, 0.25, 1.0)):
        ref_sets, cand_sets = [], []
        for bs in (1, 2):
            rs, cs = [], []
            for _ in range(bs):
                logits = rng.normal(size=200) * (1.0 + c)
                noise = rng.normal(size=200) * noise_scale
                lr = logits - np.log(np.exp(logits).sum())
                lc = (logits + noise) - np.log(np.exp(logits + noise).sum())
                ir = np.argsort(-lr)[:20]
                ic = np.argsort(-lc)[:20]
                rs.append({"top_ids": ir.tolist(), "top_logprobs": lr[ir].tolist()})
                cand = {"top_ids": ic.tolist(), "top_logprobs": lc[ic].tolist()}
                if c >= 5:
                    cand["sampled_nolp"] = int(ic[0] if rng.random() < 0.5 else ic[1])
                cs.append(cand)
            ref_sets.append({"batch_size": bs, "seq_len": 64, "seqs": rs})
            cand_sets.append({"batch_size": bs, "seq_len": 64, "seqs": cs})
        cases.append({"ref": ref_sets, "cand": cand_sets, "report": gate.compare_gate(ref_sets, cand_sets)})
    with open(os.path.join(HERE, "gate_cases.json"), "w") as f:
        json.dump(cases, f)
    print("[golden] gate_cases.json")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default="f32,quant,gate")
    a = ap.parse_args()
    only = set(a.only.split(","))
    if "f32" in only:
        make_f32(a.reference)
    if "quant" in only:
        make_quant(a.reference)
    if "gate" in only:
        make_gate(a.reference)


if __name__ == "__main__":
    main()
