"""Golden fixture for the full BASELINE config-1 shape: MiniCPM5-1B (primary config: head_dim 96,
intermediate 4608, vocab 73448, muP on), random-init seed 1234, batch 1 x 8192 ids uniform in
[1000, 30000) (seed 1234), computed by the CPU oracle (oracle/golden.py, itself pinned to the
reference's f32_golden.forward_one by tests/test_oracle.py).

    python tests/golden/make_golden_1b.py      (about a minute per layer batch on 8 cores)
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


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = PRESETS["minicpm5-1b"]
    t0 = time.time()
    sd = random_state_dict(cfg, seed=1234)
    W = golden.golden_weights(sd, cfg)
    ids = synthetic_ids(1, 8192, seed=1234)
    t1 = time.time()
    lg = golden.forward_logits(ids[0], W, cfg)
    t2 = time.time()
    tid, tlp = golden.topk_logprobs(lg, 20)
    np.savez_compressed(os.path.join(HERE, "golden_1b_s8192_logits.npz"), logits=lg.numpy())
    rng = np.random.default_rng(0)
    probe = sorted(set(tid) | set(rng.choice(cfg.vocab, 236, replace=False).tolist()))
    out = {"generator": "oracle/golden.py forward_logits (FP32)", "preset": "minicpm5-1b", "seed": 1234,
           "ids_seed": 1234, "prompt_token_ids": ids.tolist(), "top1": golden.argmax_first(lg),
           "top_ids": tid, "top_logprobs": tlp, "probe_ids": probe, "probe_logits": lg[probe].tolist(),
           "logit_range": float(lg.max() - lg.min()), "cpu_seconds": round(t2 - t1, 1),
           "cpu_threads": torch.get_num_threads()}
    with open(os.path.join(HERE, "golden_1b_s8192.json"), "w") as f:
        json.dump(out, f)
    print(f"init {t1 - t0:.1f}s forward {t2 - t1:.1f}s top1 {out['top1']} range {out['logit_range']:.4f}")


if __name__ == "__main__":
    main()
