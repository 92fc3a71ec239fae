"""Golden fixtures for the parity configs beyond the primary 1B one, computed by the CPU oracle
(oracle/golden.py, pinned to the reference's f32_golden.forward_one by tests/test_oracle.py).

* `ckpt_gate`: the real MiniCPM5-1B checkpoint's dimensions (preset `minicpm5-1b-ckpt`: head_dim 128,
  intermediate 4608, vocab 130,560, rope theta 5e6, no muP -- exactly `f32_golden.forward_one`),
  random-init seed 1234, on the reference's own gate prompts (tests/golden/gate_prompts_1b.npz: one
  1 x 8192 and one 4 x 8192 set, ids 0 .. 129,072 with the BOS id 0).
* `2b`: the MiniCPM5-2B primary config (42 layers, hidden 2048, head_dim 128, intermediate 6144,
  vocab 73,448, muP), random-init seed 1234, 1 x 8192 ids uniform in [1000, 30000) (seed 1234).

Each sequence's full last-token logits are stored as float16 (their rounding, at most 2^-11 of a
logit's magnitude, is far below the accuracy bar the tests apply), with the float64 log-softmax top-20
and the greedy id taken from the float32 logits.

    python tests/golden/make_golden_configs.py [ckpt_gate|2b ...]   (about 2 + 6 minutes per sequence
                                                                    on 8 cores)
"""
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minicpm5-vllm-tpu_b200"))

from oracle import golden  # noqa: E402
from minicpm5_mk.mk_config import PRESETS  # noqa: E402
from minicpm5_mk.mk_init import random_state_dict, synthetic_ids  # noqa: E402


def _sets(name):
    if name == "ckpt_gate":
        z = np.load(os.path.join(HERE, "gate_prompts_1b.npz"))
        return "minicpm5-1b-ckpt", [torch.from_numpy(z["set0"]), torch.from_numpy(z["set1"])], "gate_prompts_1b.npz"
    if name == "2b":
        return "minicpm5-2b", [synthetic_ids(1, 8192, seed=1234)], "synthetic_ids(1, 8192, seed=1234)"
    raise SystemExit(f"unknown case {name}")


def make(name):
    preset, sets, source = _sets(name)
    cfg = PRESETS[preset]
    t0 = time.time()
    W = golden.golden_weights(random_state_dict(cfg, seed=1234), cfg)
    arrays, meta = {}, {"generator": "oracle/golden.py forward_logits (FP32)", "preset": preset, "seed": 1234,
                        "prompts": source, "sets": []}
    for si, ids in enumerate(sets):
        rows = []
        for b in range(ids.shape[0]):
            t1 = time.time()
            lg = golden.forward_logits(ids[b], W, cfg)
            tid, tlp = golden.topk_logprobs(lg, 20)
            arrays[f"logits_{si}_{b}"] = lg.numpy().astype(np.float16)
            rows.append({"top1": golden.argmax_first(lg), "top_ids": tid, "top_logprobs": tlp,
                         "logit_range": float(lg.max() - lg.min()), "cpu_seconds": round(time.time() - t1, 1)})
            print(f"{name} set {si} seq {b}: top1 {rows[-1]['top1']} range {rows[-1]['logit_range']:.4f} "
                  f"{rows[-1]['cpu_seconds']}s", flush=True)
        meta["sets"].append({"batch_size": int(ids.shape[0]), "seq_len": int(ids.shape[1]), "seqs": rows})
        if name == "2b":
            arrays[f"ids_{si}"] = ids.numpy()
    meta["cpu_threads"] = torch.get_num_threads()
    meta["total_seconds"] = round(time.time() - t0, 1)
    np.savez_compressed(os.path.join(HERE, f"golden_{name}_logits.npz"), **arrays)
    with open(os.path.join(HERE, f"golden_{name}.json"), "w") as f:
        json.dump(meta, f)


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    for name in sys.argv[1:] or ["ckpt_gate", "2b"]:
        make(name)


if __name__ == "__main__":
    main()
