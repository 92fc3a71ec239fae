"""The drop-in contract on a B200: `vllm.LLM(..., hf_overrides={"architectures":
["MiniCPM5MegakernelForCausalLM"]}).generate(prompts, SamplingParams(max_tokens=1, temperature=0))`
loads the plugin through its `vllm.general_plugins` entry point, serves the fresh equal-length prefill
step on the megakernel path, and returns the same greedy tokens as vLLM's own Llama path and as the FP32
golden (the reference's drop-in claim, `README.md:255`, `plugin/minicpm5_mk/model.py:554-795`).

Each engine runs in its own child process (tests/vllm_drop_in_child.py)."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _child(what, mdir, timeout):
    env = dict(os.environ)
    # the package dir carries the plugin's dist-info (entry point `vllm.general_plugins`)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "minicpm5-vllm-tpu_b200"), ROOT,
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, os.path.join(HERE, "vllm_drop_in_child.py"), what, mdir], env=env,
                       capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, (what, r.stdout[-2000:], r.stderr[-4000:])
    return json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1]), r.stdout + r.stderr


def test_vllm_generate_drop_in(tmp_path):
    pytest.importorskip("vllm")
    mdir = str(tmp_path / "tiny_llama")
    made, _ = _child("make", mdir, 300)
    fast, _ = _child("mk", mdir, 600)
    stock, _ = _child("stock", mdir, 600)
    assert fast["tokens"] == made["golden_top1"], (fast, made)
    assert stock["tokens"] == made["golden_top1"], (stock, made)
    served = fast["status"]["shapes"]
    assert served and all(k.startswith("mk:") for k in served), fast["status"]


def test_vllm_generate_kv_cache_skip(tmp_path):
    """With no stock fallback (MINICPM5_MK_FREE_STOCK=1) the scheduler hands the max_tokens=1 prefills no
    KV-cache blocks (engine hook of plugin/minicpm5_mk/__init__.py:154-205) and the tokens stay the golden's."""
    pytest.importorskip("vllm")
    mdir = str(tmp_path / "tiny_llama")
    made, _ = _child("make", mdir, 300)
    free, log = _child("mkfree", mdir, 600)
    assert free["tokens"] == made["golden_top1"], (free, made)
    assert "KV-cache allocation skipped" in log
    served = free["status"]["shapes"]
    assert served and all(k.startswith("mk:") for k in served), free["status"]
