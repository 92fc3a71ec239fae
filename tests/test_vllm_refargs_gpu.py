"""The drop-in at the reference's own engine arguments and shapes, on a B200.

The reference builds `LLM(..., max_model_len=8256, max_num_batched_tokens=262144, max_num_seqs=32,
block_size=256, gpu_memory_utilization=0.5)` without `enforce_eager`, with VLLM_ENABLE_V1_MULTIPROCESSING=0
and MINICPM5_MK_FREE_STOCK=1 (examples/minimal_vllm_inference.py:10-19, 90-103), and times
`generate(..., SamplingParams(max_tokens=1, temperature=0))` at 1 x 8192 and 32 x 8192
(benchmark/run_benchmark.py:368-466).  `bench.py --vllm-e2e` does the same on a random-init checkpoint of
the MiniCPM5-1B primary config; this test runs it with a few timed calls and checks that
  * every greedy token equals the library's own (MkEngine on the same checkpoint),
  * only the megakernel path served the two shapes (the plugin's status file, as the reference's verifier
    requires, benchmark/verify_results.py:301-314), and
  * each 32 x 8192 generate call was one forward (single-step scheduling of the whole batch)."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_vllm_generate_reference_engine_args():
    pytest.importorskip("vllm")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "minicpm5-vllm-tpu_b200"), ROOT,
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--vllm-e2e", "--vllm-runs", "3",
                        "--vllm-runs-batch", "1"], env=env, capture_output=True, text=True, timeout=2400)
    if r.returncode != 0:
        tb = r.stderr.rfind("RuntimeError: vllm child")
        pytest.fail(r.stderr[tb:tb + 8000] if tb >= 0 else r.stderr[-8000:], pytrace=False)
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    for key in ("1x8192", "32x8192"):
        assert line[key]["tokens_match_direct"], line
    st = line["status"]
    assert st and st["stock_freed"], st
    shapes = st["shapes"]
    assert set(shapes) == {"mk:1x8192", "mk:32x8192"}, shapes
    assert shapes["mk:1x8192"]["steps"] == 5 + 3
    assert shapes["mk:32x8192"]["steps"] == 2 + 1  # one forward per generate call
    assert set(st.get("stock_reasons", {})) <= {"dummy"}, st
