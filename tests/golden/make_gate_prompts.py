"""Extract the reference's own gate prompts into a committed fixture.

The reference scores every candidate on the same gate prompt sets, stored beside its FP32 goldens
(`benchmark/ref/fp32_8192_1b_golden_logprobs.json` -> "inputs": a 1 x 8192 and a 4 x 8192 set of seeded
prompt texts tokenised to 8192 ids, gate seed 20261027, `make_gate_inputs`,
`benchmark/run_benchmark.py:471-479`).  Their ids span
the real MiniCPM5 vocabulary (0 .. 130,559) and start with the BOS id 0, so they are the reference's
edge-case inputs for the embedding gather and the whole forward.  The logprobs in that file belong to
the real checkpoint, which is not available offline; only the prompt ids are taken.

    python tests/golden/make_gate_prompts.py <reference checkout>

writes tests/golden/gate_prompts_1b.npz with arrays set0 (1, 8192) and set1 (4, 8192), int32.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    src = os.path.join(sys.argv[1], "benchmark", "ref", "fp32_8192_1b_golden_logprobs.json")
    d = json.load(open(src))
    arrays = {}
    for i, s in enumerate(d["inputs"]):
        ids = np.asarray(s["prompt_token_ids"], dtype=np.int32)
        assert ids.shape == (s["batch_size"], s["seq_len"]), ids.shape
        arrays[f"set{i}"] = ids
    arrays["gate_seed"] = np.asarray([d["gate_seed"]], dtype=np.int64)
    out = os.path.join(HERE, "gate_prompts_1b.npz")
    np.savez_compressed(out, **arrays)
    print(out, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
