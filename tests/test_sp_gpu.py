"""Sequence-parallel forward (mk_forward_sp) on a B200.

The zig-zag ranks run as host threads on one GPU (minicpm5_mk.sp.ThreadGroup: one engine and stream
per rank, the per-layer K/V all-gather done by device copies after a host barrier), so the full
multi-rank data path is exercised without several GPUs.  With the key split off, every row's arithmetic
is the same as in the single-GPU forward (same GEMM K order, same key-tile order in attention, RoPE
chunks on the same positions), so the results must be bit-identical to mk_forward at bs = 1.  With two
or more GPUs the same check runs over NCCL, one process per GPU (tests/sp_nccl_child.py).  With the key
split on (the default; it splits the tiny configs at 2 and 4 ranks and the 1B config at 4 and 8), a
rank's long causal key ranges are cut over several attention CTAs and merged by a second kernel; the
logits then agree with mk_forward to float rounding, and the greedy id is the same."""
import os
import subprocess
import sys
import threading

import pytest
import torch

from minicpm5_mk import mk_weights, sp
from minicpm5_mk.mk_config import PRESETS, get_config
from minicpm5_mk.mk_init import random_state_dict, synthetic_ids

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _engines(cfg, world, key_split=False, init_device="cuda"):
    from minicpm5_mk.ops import MkEngine
    pw = mk_weights.prepare_mk_weights(random_state_dict(cfg, seed=1234, device=init_device), cfg)
    base = MkEngine(cfg, pw, "cuda:0")
    engines = [MkEngine(cfg, base.weights, "cuda:0") for _ in range(world)]
    for e in engines:
        e.set_sp_key_split(key_split)
    return base, engines


def _metrics(ref, got):
    a, b = ref.double().flatten(), got.double().flatten()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    return cos, (a - b).abs().max().item() / (a.max() - a.min()).item()


def _assert_close_logits(l0, l1, what):
    """Key-split sequence parallelism against the one-GPU forward.  Each key range takes its exponentials
    against its own running max, so the bf16 rounding of P (the tensor-core operand of P V) falls
    differently than in one pass; over 24 layers that moves the logits by a few tenths of a percent of
    their range, an order below the int8 weights' own error against the FP32 golden."""
    cos, mad = _metrics(l0, l1)
    assert cos > 0.9999 and mad <= 1e-2, f"{what}: cos {cos:.7f} max-abs {mad:.2e} of the range"


def _run_threads(engines, ids, seq, world):
    tg = sp.ThreadGroup(world)
    outs, errs = [None] * world, []
    streams = [torch.cuda.Stream() for _ in range(world)]
    torch.cuda.synchronize()

    def rank_main(r):
        try:
            with torch.cuda.stream(streams[r]):
                outs[r] = engines[r].forward_sp(ids, seq, r, world, lambda ws: tg.bind(r, ws, streams[r]))
        except BaseException as e:  # noqa: BLE001
            errs.append(e)
            tg.abort()

    th = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    torch.cuda.synchronize()
    if errs:
        raise errs[0]
    return outs[0]


@pytest.mark.parametrize("preset,seq,world", [("tiny-hd96", 1024, 2), ("tiny-hd96", 1024, 4),
                                              ("tiny-hd128", 1024, 2)])
def test_sp_threads_bit_identical_tiny(preset, seq, world):
    cfg = PRESETS[preset]
    base, engines = _engines(cfg, world)
    assert base.sp_block(seq, world) == sp.sp_block(seq, world, cfg.n_q, cfg.n_kv) > 0
    ids = synthetic_ids(1, seq, seed=21, vocab=cfg.vocab).reshape(-1).contiguous().cuda()
    h0, l0, t0 = base.forward(ids, 1, seq)
    h1, l1, t1 = _run_threads(engines, ids, seq, world)
    assert torch.equal(t0, t1)
    assert torch.equal(l0, l1)
    assert torch.equal(h0, h1)
    for e in engines:
        assert e.check_device_error() == 0


@pytest.mark.parametrize("world", [2, 8])
def test_sp_threads_bit_identical_1b_s8192(world):
    """The BASELINE config at the 2- and 8-GPU layouts (8 ranks: 1024 rows each, 64 attention CTAs)."""
    cfg = get_config("minicpm5-1b").replace(max_seq=8192)
    base, engines = _engines(cfg, world)
    ids = synthetic_ids(1, 8192, seed=1234).reshape(-1).contiguous().cuda()
    h0, l0, t0 = base.forward(ids, 1, 8192)
    h1, l1, t1 = _run_threads(engines, ids, 8192, world)
    assert torch.equal(t0, t1)
    assert torch.equal(l0, l1)
    assert torch.equal(h0, h1)


@pytest.mark.parametrize("preset,seq,world", [("tiny-hd96", 1024, 2), ("tiny-hd96", 1024, 4),
                                              ("tiny-hd128", 1024, 2)])
def test_sp_threads_key_split_tiny(preset, seq, world):
    cfg = PRESETS[preset]
    base, engines = _engines(cfg, world, key_split=True)
    ids = synthetic_ids(1, seq, seed=21, vocab=cfg.vocab).reshape(-1).contiguous().cuda()
    h0, l0, t0 = base.forward(ids, 1, seq)
    h1, l1, t1 = _run_threads(engines, ids, seq, world)
    assert torch.equal(t0, t1)
    _assert_close_logits(l0, l1, f"{preset} world {world}")
    for e in engines:
        assert e.check_device_error() == 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sp_threads_key_split_1b_s8192(golden_dir, world):
    """The default sequence-parallel path at the 2-, 4- and 8-GPU layouts of the BASELINE config on the
    committed 1 x 8192 FP32 golden's prompt and weights: the golden's greedy id, the int8 accuracy bounds
    of the one-GPU forward's own test over the whole vocabulary, close to that forward, and the same bits
    when run twice (the ranges are merged in a fixed order)."""
    import json
    import numpy as np
    fx = json.load(open(os.path.join(golden_dir, "golden_1b_s8192.json")))
    ref = torch.from_numpy(np.load(os.path.join(golden_dir, "golden_1b_s8192_logits.npz"))["logits"])
    cfg = PRESETS[fx["preset"]].replace(max_seq=8192)
    assert fx["seed"] == 1234
    base, engines = _engines(cfg, world, key_split=True, init_device="cpu")  # the golden's weights
    ids = torch.tensor(fx["prompt_token_ids"], dtype=torch.int32).reshape(-1).contiguous().cuda()
    h0, l0, t0 = base.forward(ids, 1, 8192)
    h1, l1, t1 = _run_threads(engines, ids, 8192, world)
    l1, t1 = l1.clone(), t1.clone()
    h2, l2, t2 = _run_threads(engines, ids, 8192, world)
    assert torch.equal(t1, t2) and torch.equal(l1, l2)
    assert int(t1[0]) == int(t0[0]) == fx["top1"]
    _assert_close_logits(l0, l1, f"1b world {world}")
    cos, mad = _metrics(ref, l1[0].cpu())
    assert cos >= 0.997 and mad <= 4e-2, (cos, mad)
    for e in engines:
        assert e.check_device_error() == 0


def test_sp_stage_times_and_errors():
    cfg = PRESETS["tiny-hd96"]
    base, _ = _engines(cfg, 1)
    ids = synthetic_ids(1, 1024, seed=3, vocab=cfg.vocab).reshape(-1).contiguous().cuda()
    def local(ws):  # world 1: the gather is a copy
        def gather(send, recv, nbytes, s):
            sp._slice(ws, recv, nbytes).copy_(sp._slice(ws, send, nbytes))
            return 0
        return gather

    stages = {}
    h1, l1, t1 = base.forward_sp(ids, 1024, 0, 1, local, stage_times=stages)
    h0, l0, t0 = base.forward(ids, 1, 1024)
    torch.cuda.synchronize()
    assert torch.equal(l0, l1)
    assert stages["attn"]["launches"] == cfg.num_layers - 1 and stages["kv_gather"]["ms"] > 0
    with pytest.raises(RuntimeError):  # a failing collective surfaces as an error, not a hang
        base.forward_sp(ids, 1024, 0, 1, lambda ws: lambda *a: 1 / 0)
    from minicpm5_mk._lib import MkError
    with pytest.raises(MkError):
        base.forward_sp(ids, 1024, 1, 1, local)  # rank outside the world
    with pytest.raises(MkError):
        base.forward_sp(ids, 1024, 0, 16, local)  # no zig-zag block fits


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs on one node")
def test_sp_nccl_two_gpus_bit_identical():
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([os.path.dirname(HERE),
                                                       os.path.join(os.path.dirname(HERE), "minicpm5-vllm-tpu_b200")]),
               NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29561", os.path.join(HERE, "sp_nccl_child.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "SP_NCCL_OK" in r.stdout
