"""Benchmark of the MiniCPM5 prefill-score path on B200 (one process per GPU, independent replicas).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mk|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Workload (BASELINE metric "prefill tok/s (MiniCPM5-1B 32x8192, 1/2/4/8 B200); p50 ms at 1x8192"):
MiniCPM5-1B primary config (24 layers, H 1536, 16Q/2KV, head_dim 96, I 4608, vocab 73448, muP),
random-init weights, int8 weight-only linears, bf16 activations, a global batch of 32 sequences x
8192 synthetic token ids (uniform in [1000, 30000), seed 1234, a fresh draw per step) sharded
evenly over the N ranks (each rank holds a full weight replica; no collective on the data path).
One step = one prefill-score forward of the rank's sequences returning one greedy token each.

value  : whole-job tokens/s, ids already resident in HBM, device-timed with CUDA events, max over
         ranks.  Every step's working set (weights + activations) is far larger than L2.
e2e    : the same through MkEngine.forward with the ids copied from pinned host memory each step
         and the greedy ids read back to the host each step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minicpm5-vllm-tpu_b200"))

import torch  # noqa: E402

METRIC = "prefill tok/s (MiniCPM5-1B 32x8192, 1/2/4/8 B200); p50 ms at 1x8192"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mk", choices=["mk", "reference"])
    ap.add_argument("--config", default="minicpm5-1b")
    ap.add_argument("--global-bs", type=int, default=32)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--latency-runs", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sp", action="store_true", help="skip the sequence-parallel 1 x seq latency (N > 1)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--kernel", default=None, choices=["gemm_swiglu", "gemm_qkv", "gemm_o", "gemm_kv", "gemm_down", "attn"],
                    help="time one isolated kernel of the forward (profiling driver) instead of the bench")
    ap.add_argument("--kernel-bs", type=int, default=4, help="sequences of --seq tokens for --kernel")
    ap.add_argument("--kernel-iters", type=int, default=3)
    ap.add_argument("--isolated", action="store_true",
                    help="time the isolated-kernel configuration (GEMMs at M=8192, attention at S=8192) and print "
                         "one JSON line per kernel instead of the bench")
    return ap.parse_args()


def run_kernel(a):
    """Isolated launches of one forward kernel at the bench shapes (1 warm-up + --kernel-iters timed),
    on random inputs; used as the small-case driver for ncu captures."""
    from minicpm5_mk import _lib, ops
    from minicpm5_mk.mk_config import get_config
    from minicpm5_mk.mk_weights import quantize_per_out_channel

    cfg = get_config(a.config)
    dev = torch.device("cuda", 0)
    T = a.kernel_bs * a.seq
    g = torch.Generator(device=dev).manual_seed(3)
    H, I = cfg.hidden, cfg.inter
    if a.kernel.startswith("gemm"):
        N, K, mode = {"gemm_swiglu": (2 * I, H, _lib.MK_GEMM_SWIGLU), "gemm_qkv": (cfg.qkv_dim, H, _lib.MK_GEMM_ROWSCALE),
                      "gemm_o": (H, cfg.q_dim, _lib.MK_GEMM_RESID32), "gemm_kv": (2 * cfg.kv_dim, H, _lib.MK_GEMM_ROWSCALE),
                      "gemm_down": (H, I, _lib.MK_GEMM_RESID32)}[a.kernel]
        x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
        w8, s = quantize_per_out_channel(torch.randn((N, K), generator=g, device=dev) * 0.02)
        rstd = torch.ones((T,), device=dev)
        out = torch.zeros((T, N // 2 if mode == _lib.MK_GEMM_SWIGLU else N), dtype=torch.bfloat16, device=dev)
        x32 = torch.zeros((T, N), dtype=torch.float32, device=dev) if mode == _lib.MK_GEMM_RESID32 else None
        fn = lambda: ops.gemm_w8a16(x, w8, s, mode, row_scale=rstd, resid_scale=0.3, out=out,  # noqa: E731
                                    resid32=x32)
        flops = 2.0 * T * N * K
    else:
        qkv = torch.randn((T, cfg.qkv_dim), generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty((T, cfg.q_dim), dtype=torch.bfloat16, device=dev)
        fn = lambda: ops.attention_prefill(qkv, a.kernel_bs, a.seq, cfg.n_q, cfg.n_kv, cfg.head_dim,  # noqa: E731
                                           softmax_scale=cfg.head_dim ** -0.5, out=out)
        flops = 2.0 * a.seq * a.seq * cfg.head_dim * cfg.n_q * a.kernel_bs
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.kernel_iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.kernel_iters
    print(json.dumps({"kernel": a.kernel, "tokens": T, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}))


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def _flops_per_seq(cfg, S):
    """Skip-aware algorithmic FLOPs of one S-token prefill-score (layers 0..L-2 in full, layer L-1 as
    K/V projection for every position + Q/O/MLP/attention for the last token, last-token lm_head).
    Same terms as the reference's verify formula (benchmark/verify_results.py:131-140)."""
    H, I, L, hd, nq, nkv, V = cfg.hidden, cfg.inter, cfg.num_layers, cfg.head_dim, cfg.n_q, cfg.n_kv, cfg.vocab
    lin_tok = 2 * (H * (nq + 2 * nkv) * hd + nq * hd * H + 2 * H * I + I * H)
    attn_seq = 2 * S * S * hd * nq  # causal: (QK^T + PV) halved
    full = (L - 1) * (S * lin_tok + attn_seq)
    last = 2 * S * H * 2 * nkv * hd + lin_tok - 2 * H * 2 * nkv * hd + 4 * S * hd * nq
    head = 2 * H * V
    return full + last + head


def _clock_sampler(gpu_index):
    try:
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        return subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except Exception:  # noqa: BLE001
        return None


def _clock_summary(proc):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except Exception:  # noqa: BLE001
        proc.kill()
        return None
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            mx = float(f[2])
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower().startswith("active"):
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def _traffic_per_launch(kernel):
    """dram bytes per launch of `kernel` at the bench workload, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith(kernel + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def cpu_sample(cfg, S, target_s, threads):
    """Time the CPU FP32 oracle (restatement of the reference's f32_golden path) on a bounded sample:
    decoder layers of one S-token sequence run one at a time until ~target_s of CPU time, then
    extrapolated to the full model.  Returns (tok/s, sample description)."""
    from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
    from oracle import golden

    torch.set_num_threads(threads)
    c1 = cfg.replace(num_layers=1, vocab=min(cfg.vocab, 4096))
    sd = random_state_dict(c1, seed=1234)
    W = golden.golden_weights(sd, c1)
    ids = synthetic_ids(1, S, seed=1234, vocab=c1.vocab)[0]
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        golden.forward_logits(ids, W, c1, last_only=False)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start >= target_s or len(times) >= cfg.num_layers:
            break
    per_layer = statistics.median(times)
    total = per_layer * cfg.num_layers
    return S / total, (f"1 x {S} tokens through {len(times)} full decoder layer(s) of the FP32 oracle "
                       f"(median {per_layer:.2f} s/layer), extrapolated x{cfg.num_layers} layers")


def run_reference(a, rank, world):
    """--impl reference: the reference's CPU FP32 path (oracle port of benchmark/f32_golden.py) on the
    host cores; rank 0 only."""
    if rank != 0:
        return
    from minicpm5_mk.mk_config import get_config

    cfg = get_config(a.config)
    threads = os.cpu_count() or 1
    vals = []
    desc = ""
    for i in range(a.warmup + a.steps):
        v, desc = cpu_sample(cfg, a.seq, target_s=0.0, threads=threads)  # one layer per step
        if i >= a.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(a.seq / value * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{a.config} 1x{a.seq} prefill-score, CPU FP32 oracle (one layer per step, "
                                   f"extrapolated)", "seq_len": a.seq, "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_isolated(a):
    """The isolated-kernel configuration: int8 weight-only GEMMs at M=8192 (K=1536, N=1792 QKV /
    1536 o_proj / 8192 gate+up; K=4096, N=1536 down) with their forward epilogues, and causal GQA
    attention at S=8192 with 16 Q / 2 KV heads, head_dim 96 and 128, batch 1 and 8.  Inputs and
    weights ~N(0,1), weights quantised per output channel.  CUDA-event time of each launch (1 warm-up,
    --kernel-iters timed), with L2 flushed before every timed launch (a 256 MB buffer is rewritten)."""
    from minicpm5_mk import _lib, ops
    from minicpm5_mk.mk_weights import quantize_per_out_channel

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234)
    peak = _peaks()[0]["bf16_tflops"]

    flush = torch.empty((64 * 1024 * 1024,), dtype=torch.float32, device=dev)  # 256 MB > L2

    def timeit(fn):
        fn()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(a.kernel_iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        return total / a.kernel_iters

    M = 8192
    for name, N, K, mode in (("gemm_qkv", 1792, 1536, _lib.MK_GEMM_ROWSCALE), ("gemm_o_proj", 1536, 1536, _lib.MK_GEMM_RESID32),
                             ("gemm_gate_up", 8192, 1536, _lib.MK_GEMM_SWIGLU), ("gemm_down", 1536, 4096, _lib.MK_GEMM_RESID32)):
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        w8, s = quantize_per_out_channel(torch.randn((N, K), generator=g, device=dev))
        rstd = torch.ones((M,), device=dev)
        out = torch.empty((M, N // 2 if mode == _lib.MK_GEMM_SWIGLU else N), dtype=torch.bfloat16, device=dev)
        x32 = torch.zeros((M, N), dtype=torch.float32, device=dev) if mode == _lib.MK_GEMM_RESID32 else None
        ms = timeit(lambda: ops.gemm_w8a16(x, w8, s, mode, row_scale=rstd, resid_scale=0.3, out=out, resid32=x32))
        tf = 2.0 * M * N * K / ms / 1e9
        print(json.dumps({"kernel": name, "M": M, "N": N, "K": K, "ms": round(ms, 4), "tflops": round(tf, 1),
                          "frac_of_measured_peak": round(tf / peak, 4)}))
    for hd in (96, 128):
        for bs in (1, 8):
            S, nq, nkv = 8192, 16, 2
            qkv = torch.randn((bs * S, (nq + 2 * nkv) * hd), generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty((bs * S, nq * hd), dtype=torch.bfloat16, device=dev)
            ms = timeit(lambda: ops.attention_prefill(qkv, bs, S, nq, nkv, hd, softmax_scale=hd ** -0.5, out=out))
            tf = 2.0 * S * S * hd * nq * bs / ms / 1e9
            print(json.dumps({"kernel": "attention", "batch": bs, "seq": S, "heads": f"{nq}q/{nkv}kv", "head_dim": hd,
                              "ms": round(ms, 4), "tflops": round(tf, 1), "frac_of_measured_peak": round(tf / peak, 4)}))


def main():
    a = _args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    if a.kernel:
        run_kernel(a)
        return
    if a.isolated:
        run_isolated(a)
        return
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from minicpm5_mk import mk_weights, ops
    from minicpm5_mk.mk_config import get_config
    from minicpm5_mk.mk_init import random_state_dict, synthetic_ids

    from minicpm5_mk.replicas import shard_bounds

    cfg = get_config(a.config).replace(max_seq=max(a.seq, 8192))
    _, bs = shard_bounds(a.global_bs, world, rank)  # this replica's block of sequences
    if bs == 0:
        raise SystemExit(f"global batch {a.global_bs} leaves rank {rank} without sequences")
    S = a.seq
    T = bs * S

    # Full weight replica on this GPU (random-init from the device generator, prepared on device).
    sd = random_state_dict(cfg, seed=1234, device=dev)
    pw = mk_weights.prepare_mk_weights(sd, cfg)
    del sd
    torch.cuda.empty_cache()
    eng = ops.MkEngine(cfg, pw, dev)
    del pw

    nbat = a.warmup + a.steps
    ids_host = [synthetic_ids(bs, S, seed=1234 + 1000 * rank + i).reshape(-1).contiguous().pin_memory()
                for i in range(nbat)]
    ids_dev = [t.to(dev) for t in ids_host]
    hid = torch.empty((bs, cfg.hidden), dtype=torch.bfloat16, device=dev)
    lg = torch.empty((bs, cfg.vocab), dtype=torch.float32, device=dev)
    top1 = torch.empty((bs,), dtype=torch.int32, device=dev)
    out = (hid, lg, top1)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------------------------------------------------------- device-timed throughput
    for i in range(a.warmup):
        eng.forward(ids_dev[i], bs, S, out=out)
    torch.cuda.synchronize()
    eng.check_device_error()
    clk = _clock_sampler(local)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(a.steps):
        eng.forward(ids_dev[a.warmup + i], bs, S, out=out)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = _clock_summary(clk)
    dev_ms = ev0.elapsed_time(ev1) / a.steps
    step_ms = max_over_ranks(dev_ms)
    err = eng.check_device_error()
    total_tokens = a.global_bs * S
    value = total_tokens / (step_ms / 1e3)

    # ---------------------------------------------------------------- per-stage device time inside a step
    # One more forward right after the timed region, in the same clock and power state, through
    # mk_forward_timed: the same launches with CUDA events between them.
    stages = {}
    eng.forward(ids_dev[a.warmup], bs, S, out=out, stage_times=stages)

    # ---------------------------------------------------------------- end to end (host buffers)
    e2e = None
    if not a.no_e2e:
        ids_buf = torch.empty((T,), dtype=torch.int32, device=dev)
        top1_host = torch.empty((bs,), dtype=torch.int32).pin_memory()
        for i in range(min(2, a.warmup)):
            ids_buf.copy_(ids_host[i], non_blocking=True)
            eng.forward(ids_buf, bs, S, out=out)
            top1_host.copy_(top1, non_blocking=True)
            stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(a.steps):
            ids_buf.copy_(ids_host[a.warmup + i], non_blocking=True)
            eng.forward(ids_buf, bs, S, out=out)
            top1_host.copy_(top1, non_blocking=True)
            stream.synchronize()
            _ = top1_host.tolist()  # the host reads each step's result
        e1.record(stream)
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - t0) * 1e3 / a.steps
        e2e_ms = max_over_ranks(max(wall_ms, e0.elapsed_time(e1) / a.steps))
        e2e = {"value": round(total_tokens / (e2e_ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(e2e_ms, 3),
               "h2d_bytes_per_step": int(a.global_bs * S * 4), "d2h_bytes_per_step": int(a.global_bs * 4),
               "api": "minicpm5_mk.ops.MkEngine.forward -> mk_forward (C ABI)"}

    # ---------------------------------------------------------------- latency at 1 x 8192
    lat = None
    if rank == 0 and a.latency_runs > 0:
        one = ids_dev[0][:S].contiguous()
        o1 = (hid[:1], lg[:1], top1[:1])
        for _ in range(5):
            eng.forward(one, 1, S, out=o1)
        torch.cuda.synchronize()
        ts = []
        for _ in range(a.latency_runs):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            eng.forward(one, 1, S, out=o1)
            s1.record(stream)
            s1.synchronize()
            ts.append(s0.elapsed_time(s1))
        ts.sort()

        def pct(p):
            k = (len(ts) - 1) * p / 100.0
            lo = int(k)
            hi = min(lo + 1, len(ts) - 1)
            return ts[lo] + (ts[hi] - ts[lo]) * (k - lo)

        lat = {"p50_ms": round(pct(50), 3), "p99_ms": round(pct(99), 3), "runs": len(ts), "warmup": 5,
               "timing": "device (CUDA events)"}
    barrier()

    # ---------------------------------------------------------------- latency at 1 x seq, sequence parallel
    # One sequence over all N ranks (zig-zag blocks, per-layer K/V all-gather over NCCL): every rank runs
    # every step; a run's latency is the maximum over ranks of its device time.
    lat_sp = None
    if world > 1 and not a.no_sp and a.latency_runs > 0 and eng.sp_block(S, world) > 0:
        from minicpm5_mk import sp as mk_sp
        one_sp = synthetic_ids(1, S, seed=1234).reshape(-1).contiguous().to(dev)  # the same sequence on every rank
        gather = mk_sp.nccl_allgather()
        o1 = (hid[:1], lg[:1], top1[:1])
        for _ in range(5):
            eng.forward_sp(one_sp, S, rank, world, gather, out=o1)
        torch.cuda.synchronize()
        barrier()
        ts_sp = []
        for _ in range(a.latency_runs):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            eng.forward_sp(one_sp, S, rank, world, gather, out=o1)
            s1.record(stream)
            s1.synchronize()
            ts_sp.append(s0.elapsed_time(s1))
        t = torch.tensor(ts_sp, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ts_sp = sorted(t.tolist())
        sp_stages = {}
        eng.forward_sp(one_sp, S, rank, world, gather, out=o1, stage_times=sp_stages)
        barrier()

        def pct_sp(p):
            k = (len(ts_sp) - 1) * p / 100.0
            lo = int(k)
            hi = min(lo + 1, len(ts_sp) - 1)
            return ts_sp[lo] + (ts_sp[hi] - ts_sp[lo]) * (k - lo)

        lat_sp = {"p50_ms": round(pct_sp(50), 3), "p99_ms": round(pct_sp(99), 3), "runs": len(ts_sp), "warmup": 5,
                  "ranks": world, "block": eng.sp_block(S, world),
                  "timing": "device (CUDA events), max over ranks per run",
                  "api": "minicpm5_mk.ops.MkEngine.forward_sp -> mk_forward_sp (C ABI) + NCCL all-gather",
                  "stages_rank0_ms": {k: round(v["ms"], 3) for k, v in sp_stages.items()}}

    # ---------------------------------------------------------------- roofline of the dominant kernels
    # In-step figures: each stage's device time inside the forward just after the timed region (a long,
    # power-capped step), against the sustained GEMM peak.  Alone figures: the two largest kernels timed
    # by themselves (3 back-to-back launches on the same inputs), against the burst peak.
    peaks, peak_kind = _peaks()
    H, I, hd = cfg.hidden, cfg.inter, cfg.head_dim
    flops_per_launch = {"qkv": 2.0 * T * H * cfg.qkv_dim, "attn": 2.0 * S * S * hd * cfg.n_q * bs,
                        "o_proj": 2.0 * T * cfg.q_dim * H, "gate_up": 2.0 * T * H * 2 * I, "down": 2.0 * T * I * H}
    stage_total = sum(v["ms"] for v in stages.values())
    peak_sus = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    in_step = {}
    for name, fl in flops_per_launch.items():
        v = stages[name]
        ms = v["ms"] / max(1, v["launches"])
        in_step[name] = {"ms_per_launch": round(ms, 4), "achieved": round(fl / ms / 1e9, 1),
                         "frac": round(fl / ms / 1e9 / peak_sus, 4), "share_of_step": round(v["ms"] / stage_total, 3)}
    for name in ("embed", "last_layer", "head"):
        in_step[name] = {"ms": round(stages[name]["ms"], 4), "launches": stages[name]["launches"],
                         "share_of_step": round(stages[name]["ms"] / stage_total, 3)}

    alone = {}
    if rank == 0:
        g = torch.Generator(device=dev).manual_seed(5)
        x = (torch.randn((T, cfg.hidden), generator=g, device=dev) * 0.5).to(torch.bfloat16)
        rstd = torch.ones((T,), device=dev)
        w_gu, s_gu = eng.weights["w_gu"][0], eng.weights["s_gu"][0]
        hbuf = torch.empty((T, cfg.inter), dtype=torch.bfloat16, device=dev)
        qkv = (torch.randn((T, cfg.qkv_dim), generator=g, device=dev)).to(torch.bfloat16)
        abuf = torch.empty((T, cfg.q_dim), dtype=torch.bfloat16, device=dev)

        def timeit(fn, n=3):
            fn()
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(n):
                fn()
            s1.record(stream)
            s1.synchronize()
            return s0.elapsed_time(s1) / n

        from minicpm5_mk import _lib
        ms_gu = timeit(lambda: ops.gemm_w8a16(x, w_gu, s_gu, _lib.MK_GEMM_SWIGLU, row_scale=rstd, out=hbuf))
        ms_at = timeit(lambda: ops.attention_prefill(qkv, bs, S, cfg.n_q, cfg.n_kv, hd, softmax_scale=hd ** -0.5,
                                                     out=abuf))
        for name, ms in (("gate_up", ms_gu), ("attn", ms_at)):
            fl = flops_per_launch[name]
            alone[name] = {"ms_per_launch": round(ms, 4), "achieved": round(fl / ms / 1e9, 1),
                           "frac": round(fl / ms / 1e9 / peaks["bf16_tflops"], 4)}
        del x, hbuf, qkv, abuf
    kernel_names = {"attn": "attn_tc_kernel", "gate_up": "gemm_w8a16_kernel (SWIGLU)"}
    traffic_keys = {"attn": "attn_prefill", "gate_up": "gemm_w8a16_swiglu"}
    dom = max(kernel_names, key=lambda k: in_step[k]["share_of_step"])
    k = in_step[dom]
    roofline = {"kernel": kernel_names[dom], "bound": "tensor", "achieved": k["achieved"], "peak": peak_sus,
                "unit": "TFLOP/s", "frac": k["frac"],
                "peak_kind": f"{peak_kind} (sustained: the kernel is timed inside a forward step)",
                "traffic": _traffic_per_launch(traffic_keys[dom]), "flops_per_launch": flops_per_launch[dom],
                "ms_per_launch": k["ms_per_launch"], "share_of_step": k["share_of_step"],
                "timing": "CUDA events between the launches of one mk_forward_timed step after the timed region",
                "stages": in_step,
                "alone": {"peak": peaks["bf16_tflops"], "peak_kind": f"{peak_kind} (burst)", "kernels": alone}}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, desc = cpu_sample(cfg, S, a.cpu_seconds, threads)
        cpu = {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc}

    fl_step = _flops_per_seq(cfg, S) * a.global_bs
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{a.config} prefill-score {a.global_bs}x{S} (1 greedy token per sequence), "
                              f"int8 weight-only linears, bf16 activations",
                   "model": a.config, "global_batch": a.global_bs, "seq_len": S, "per_gpu_batch": bs,
                   "parallelism": f"dp{world} (independent full replicas, no collective)",
                   "l2": "working set (0.9 GB weights + activations) larger than L2 every step"},
        "model_tflops": round(fl_step / (step_ms / 1e3) / 1e12, 1),
        "model_roofline_frac": round(fl_step / (step_ms / 1e3) / 1e12 / (peak_sus * world), 4),
        "model_roofline_peak": "sustained bf16 GEMM peak per GPU",
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": eng.launches_per_forward(bs, S) * a.steps,
        "clocks": clocks, "latency_1x8192": lat,
        "latency_1x8192_sp": lat_sp, "device_error": err,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
