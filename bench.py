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
    ap.add_argument("--kernel", default=None,
                    choices=["gemm_swiglu", "gemm_qkv", "gemm_qkv_rope", "gemm_o", "gemm_kv", "gemm_down", "attn",
                             "forward_sp",
                             "forward", "lm_head"],
                    help="time one isolated kernel of the forward, or whole forwards of --kernel-bs sequences "
                         "(profiling driver), instead of the bench")
    ap.add_argument("--kernel-bs", type=int, default=4, help="sequences of --seq tokens for --kernel")
    ap.add_argument("--sp-world", type=int, default=8,
                    help="--kernel forward_sp: rank 0 of this many sequence-parallel ranks on one GPU, the K/V "
                         "all-gather replaced by copies of the rank's own rows (profiling driver)")
    ap.add_argument("--kernel-iters", type=int, default=3)
    ap.add_argument("--isolated", action="store_true",
                    help="time the isolated-kernel configuration (GEMMs at M=8192, attention at S=8192) and print "
                         "one JSON line per kernel instead of the bench")
    ap.add_argument("--vllm-e2e", action="store_true",
                    help="end to end through vLLM: LLM(...) with the reference's engine arguments on a random-init "
                         "checkpoint of --config, LLM.generate(max_tokens=1, temperature=0) at 1 x seq and "
                         "--global-bs x seq; prints one JSON line")
    ap.add_argument("--vllm-child", nargs=2, metavar=("ROLE", "DIR"), default=None, help=argparse.SUPPRESS)
    ap.add_argument("--vllm-runs", type=int, default=20, help="timed generate calls at 1 x seq (--vllm-e2e)")
    ap.add_argument("--vllm-runs-batch", type=int, default=5, help="timed generate calls at the global batch")
    return ap.parse_args()


# ------------------------------------------------------------------------------ vLLM end to end
# The reference's headline numbers are LLM.generate end to end (README.md:52-56, benchmark/run_benchmark.py:
# 368-466) with the engine built as in examples/minimal_vllm_inference.py:90-103.  Each role runs in its own
# process: `make` writes a random-init checkpoint (bf16 safetensors + config.json), `serve` builds the engine
# with the reference's arguments and times generate, `direct` computes the same prompts' greedy ids through
# MkEngine on the same checkpoint (the drop-in must return exactly those).
VLLM_ENV = {"VLLM_ENABLE_V1_MULTIPROCESSING": "0", "MINICPM5_MK_FREE_STOCK": "1"}


def _vllm_prompts(cfg, bs, S, seed):
    from minicpm5_mk.mk_init import synthetic_ids
    ids = synthetic_ids(bs, S, seed=seed, vocab=cfg.vocab)
    ids[:, 0] = 0  # a BOS id first, as the reference's prompts (examples/minimal_vllm_inference.py:115-117)
    return ids


def _vllm_child_make(cfg_name, mdir):
    from safetensors.torch import save_file
    from minicpm5_mk.mk_config import get_config
    from minicpm5_mk.mk_init import param_shapes, make_param

    cfg = get_config(cfg_name)
    os.makedirs(mdir, exist_ok=True)
    dev = torch.device("cuda", 0)
    sd = {n: make_param(n, shp, seed=1234, device=dev).to(torch.bfloat16).cpu().contiguous()
          for n, shp in param_shapes(cfg).items()}
    save_file(sd, os.path.join(mdir, "model.safetensors"))
    hf = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": cfg.hidden,
          "intermediate_size": cfg.inter, "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.n_q,
          "num_key_value_heads": cfg.n_kv, "head_dim": cfg.head_dim, "vocab_size": cfg.vocab,
          "max_position_embeddings": 8256, "rms_norm_eps": cfg.eps, "rope_theta": cfg.rope_theta,
          "tie_word_embeddings": False, "torch_dtype": "bfloat16", "hidden_act": "silu", "bos_token_id": 0,
          "eos_token_id": 2}
    if cfg.scale_emb != 1.0 or cfg.residual_scale != 1.0 or cfg.logit_scale != 1.0:
        # MiniCPM's muP fields (read by minicpm5_mk.mk_config.from_hf_config)
        import math
        hf.update(scale_emb=cfg.scale_emb, scale_depth=cfg.residual_scale * math.sqrt(cfg.num_layers),
                  dim_model_base=cfg.logit_scale * cfg.hidden)
    with open(os.path.join(mdir, "config.json"), "w") as f:
        json.dump(hf, f)
    print(json.dumps({"made": mdir, "params": sum(v.numel() for v in sd.values())}))


def _vllm_child_direct(a, mdir):
    from minicpm5_mk import checkpoint, mk_weights, ops
    dev = torch.device("cuda", 0)
    cfg, sd = checkpoint.load_hf_checkpoint(mdir, device=dev, max_seq=8256)
    eng = ops.MkEngine(cfg, mk_weights.prepare_mk_weights({k: v.float() for k, v in sd.items()}, cfg), dev)
    del sd
    out = {}
    for bs, seed in ((1, 7), (a.global_bs, 8)):
        ids = _vllm_prompts(cfg, bs, a.seq, seed)
        _, _, top1 = eng.forward(ids.reshape(-1).contiguous().to(dev), bs, a.seq)
        out[f"{bs}x{a.seq}"] = top1.cpu().tolist()
    print(json.dumps({"direct": out}))


def _vllm_child_serve(a, mdir):
    for k, v in VLLM_ENV.items():
        os.environ.setdefault(k, v)
    os.environ["MINICPM5_MK_STATUS_DIR"] = os.path.join(mdir, "status")
    from vllm import LLM, SamplingParams
    from minicpm5_mk.mk_config import get_config

    cfg = get_config(a.config)
    t0 = time.perf_counter()
    # examples/minimal_vllm_inference.py:90-103, minus its TPU compile_sizes (on the GPU runner they ask
    # inductor for static-shape graphs of the stock model, which the fast path never runs)
    llm = LLM(model=mdir, skip_tokenizer_init=True, hf_overrides={"architectures": ["MiniCPM5MegakernelForCausalLM"]},
              tensor_parallel_size=1, dtype="bfloat16", enable_prefix_caching=False, max_model_len=8256,
              max_num_batched_tokens=262144, max_num_seqs=32, block_size=256, gpu_memory_utilization=0.5)
    load_s = time.perf_counter() - t0
    sp = SamplingParams(max_tokens=1, min_tokens=1, temperature=0.0, detokenize=False)
    res = {"load_s": round(load_s, 1)}
    for bs, seed, runs, warm in ((1, 7, a.vllm_runs, 5), (a.global_bs, 8, a.vllm_runs_batch, 2)):
        ids = _vllm_prompts(cfg, bs, a.seq, seed)
        prompts = [{"prompt_token_ids": ids[b].tolist()} for b in range(bs)]
        toks = None
        for _ in range(warm):
            outs = llm.generate(prompts, sp, use_tqdm=False)
            toks = [o.outputs[0].token_ids[0] for o in outs]
        ts = []
        for _ in range(runs):
            t = time.perf_counter()
            outs = llm.generate(prompts, sp, use_tqdm=False)
            ts.append((time.perf_counter() - t) * 1e3)
            assert [o.outputs[0].token_ids[0] for o in outs] == toks, "greedy tokens changed between runs"
        ts.sort()

        def pct(p):
            k = (len(ts) - 1) * p / 100.0
            lo = int(k)
            hi = min(lo + 1, len(ts) - 1)
            return ts[lo] + (ts[hi] - ts[lo]) * (k - lo)

        res[f"{bs}x{a.seq}"] = {"tokens": toks, "p50_ms": round(pct(50), 3), "p99_ms": round(pct(99), 3),
                                "runs": runs, "warmup": warm,
                                "tok_s": round(bs * a.seq / (statistics.mean(ts) / 1e3), 1)}
    st = os.path.join(mdir, "status", "minicpm5_mk_status_rank0.json")
    res["status"] = json.load(open(st)) if os.path.exists(st) else None
    print(json.dumps({"serve": res}))


def run_vllm_e2e(a):
    """LLM.generate end to end at 1 x seq and global_bs x seq (one JSON line), each role in a child."""
    import tempfile
    mdir = os.path.join(tempfile.mkdtemp(prefix="mk_vllm_"), a.config)

    def child(role):
        env = dict(os.environ)
        env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "minicpm5-vllm-tpu_b200"), ROOT,
                                             env.get("PYTHONPATH", "")])
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--config", a.config, "--seq", str(a.seq),
                            "--global-bs", str(a.global_bs), "--vllm-runs", str(a.vllm_runs),
                            "--vllm-runs-batch", str(a.vllm_runs_batch), "--vllm-child", role, mdir],
                           env=env, capture_output=True, text=True, timeout=1800)
        with open(os.path.join(os.path.dirname(mdir), f"{role}.log"), "w") as f:
            f.write(r.stdout + "\n" + r.stderr)
        if r.returncode != 0:
            err = r.stderr
            tb = err.rfind("Traceback (most recent call last)")
            raise RuntimeError(f"vllm child {role} failed (rc {r.returncode}): " + (err[tb:tb + 6000] if tb >= 0
                                                                                   else err[-4000:]))
        return json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])

    child("make")
    direct = child("direct")["direct"]
    serve = child("serve")["serve"]
    line = {"metric": "vLLM LLM.generate end to end (max_tokens=1, temperature=0)", "config": a.config,
            "engine_args": "examples/minimal_vllm_inference.py:90-103 without TPU compile_sizes; "
                           "VLLM_ENABLE_V1_MULTIPROCESSING=0, MINICPM5_MK_FREE_STOCK=1",
            "load_s": serve["load_s"], "status": serve["status"]}
    for key in (f"1x{a.seq}", f"{a.global_bs}x{a.seq}"):
        r = serve[key]
        line[key] = {k: r[k] for k in ("p50_ms", "p99_ms", "runs", "warmup", "tok_s")}
        line[key]["tokens_match_direct"] = r["tokens"] == direct[key]
    print(json.dumps(line), flush=True)


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
    if a.kernel == "lm_head":
        # --kernel-bs rows through lm_head + argmax (mk_lm_head_argmax): the vocabulary matrix (225.6 MB at
        # the 1B config) is streamed once per launch of up to 8 rows
        W = (torch.randn((cfg.vocab, cfg.hidden), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        hrow = torch.randn((a.kernel_bs, cfg.hidden), generator=g, device=dev)
        fn = lambda: ops.lm_head_argmax(hrow, W)  # noqa: E731
        flops = 2.0 * a.kernel_bs * cfg.vocab * cfg.hidden
    elif a.kernel == "forward":
        from minicpm5_mk import mk_weights
        from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
        cfg = cfg.replace(max_seq=max(a.seq, cfg.max_seq))
        sd = random_state_dict(cfg, seed=1234, device=dev)
        eng = ops.MkEngine(cfg, mk_weights.prepare_mk_weights(sd, cfg), dev)
        del sd
        ids = synthetic_ids(a.kernel_bs, a.seq, seed=1234).reshape(-1).contiguous().to(dev)
        fn = lambda: eng.forward(ids, a.kernel_bs, a.seq)  # noqa: E731
        flops = _flops_per_seq(cfg, a.seq) * a.kernel_bs
    elif a.kernel == "forward_sp":
        # rank 0 of a --sp-world layout on this GPU alone: every kernel of the rank's forward runs at its real
        # shape (the key-split attention included); the all-gather copies the rank's own K/V rows into every
        # rank's slot, so no other GPU is needed (the numbers are not a sequence-parallel result)
        from minicpm5_mk import mk_weights, sp
        from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
        cfg = cfg.replace(max_seq=max(a.seq, cfg.max_seq))
        sd = random_state_dict(cfg, seed=1234, device=dev)
        eng = ops.MkEngine(cfg, mk_weights.prepare_mk_weights(sd, cfg), dev)
        del sd
        ids = synthetic_ids(1, a.seq, seed=1234).reshape(-1).contiguous().to(dev)
        world = a.sp_world

        def bind(ws):
            def gather(send, recv, nbytes, s):
                src, dst = sp._slice(ws, send, nbytes), sp._slice(ws, recv, nbytes * world)
                for r in range(world):
                    dst[r * nbytes:(r + 1) * nbytes].copy_(src)
                return 0
            return gather

        fn = lambda: eng.forward_sp(ids, a.seq, 0, world, bind)  # noqa: E731
        flops = _flops_per_seq(cfg, a.seq) / world
    elif a.kernel == "gemm_qkv_rope":
        # the forward's QKV projection: rstd from per-tile sums of squares, RoPE on the Q/K columns
        from minicpm5_mk.mk_weights import rope_tables
        N, K = cfg.qkv_dim, H
        x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
        w8, s = quantize_per_out_channel(torch.randn((N, K), generator=g, device=dev) * 0.02)
        rowsq = torch.rand((T, H // 128), generator=g, device=dev) * 128.0 + 1.0
        cos, sin = (t.to(dev) for t in rope_tables(a.seq, cfg.head_dim, cfg.rope_theta))
        out = torch.empty((T, N), dtype=torch.bfloat16, device=dev)
        fn = lambda: ops.gemm_w8a16(x, w8, s, _lib.MK_GEMM_ROWSCALE, out=out, rowsq=rowsq,  # noqa: E731
                                    rowsq_np=H // 128, norm_dim=H, eps=cfg.eps, rope=(cos, sin),
                                    rope_cols=cfg.q_dim + cfg.kv_dim, head_dim=cfg.head_dim, rope_seq=a.seq)
        flops = 2.0 * T * N * K
    elif a.kernel.startswith("gemm"):
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
    line = {"kernel": a.kernel, "tokens": T, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}
    if a.kernel == "forward_sp":  # one sequence, this rank's share of it
        line.update(tokens=a.seq, ranks=a.sp_world, rank_rows=a.seq // a.sp_world)
    if a.kernel == "lm_head":
        line["weight_gbs"] = round(cfg.vocab * cfg.hidden * 2 * -(-a.kernel_bs // 8) / ms / 1e6, 1)
    if a.kernel == "forward":  # per-stage device time of one more forward (events between the launches)
        stages = {}
        eng.forward(ids, a.kernel_bs, a.seq, stage_times=stages)
        line["stages_ms"] = {k: round(v["ms"], 4) for k, v in stages.items()}
        line["stages_launches"] = {k: v["launches"] for k, v in stages.items()}
    print(json.dumps(line))


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


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), as the reference's benchmark records it
    (benchmark/run_benchmark.py:153-167)."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


class CpuLayerSample:
    """The CPU FP32 oracle (restatement of the reference's f32_golden path) on a bounded sample of the
    workload: one full decoder layer of one S-token sequence per call (the full model is num_layers such
    layers plus a last-token lm_head, which is under 0.1 % of the work).  `step()` returns the seconds
    one layer took; `tok_s(sec)` extrapolates a layer time to the whole model's tokens/s."""

    def __init__(self, cfg, S, threads):
        from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
        from oracle import golden

        torch.set_num_threads(threads)
        self.golden, self.cfg, self.S, self.threads = golden, cfg, S, threads
        self.c1 = cfg.replace(num_layers=1, vocab=min(cfg.vocab, 4096))
        self.W = golden.golden_weights(random_state_dict(self.c1, seed=1234), self.c1)
        self.ids = synthetic_ids(1, S, seed=1234, vocab=self.c1.vocab)[0]

    def step(self) -> float:
        t0 = time.perf_counter()
        self.golden.forward_logits(self.ids, self.W, self.c1, last_only=False)
        return time.perf_counter() - t0

    def tok_s(self, sec_per_layer: float) -> float:
        return self.S / (sec_per_layer * self.cfg.num_layers)

    def describe(self, n: int, sec_per_layer: float) -> str:
        return (f"1 x {self.S} tokens through {n} full decoder layer(s) of the FP32 oracle on {self.threads} "
                f"threads (median {sec_per_layer:.2f} s/layer); tok/s extrapolated to {self.cfg.num_layers} "
                f"layers (the last-token lm_head, <0.1% of the work, is left out)")


def cpu_sample(cfg, S, target_s, threads):
    """Time the CPU FP32 oracle on decoder layers of one S-token sequence until ~target_s of CPU time and
    extrapolate to the full model.  Returns (tok/s, sample description)."""
    smp = CpuLayerSample(cfg, S, threads)
    times = []
    t_start = time.perf_counter()
    while True:
        times.append(smp.step())
        if time.perf_counter() - t_start >= target_s or len(times) >= cfg.num_layers:
            break
    per_layer = statistics.median(times)
    return smp.tok_s(per_layer), smp.describe(len(times), per_layer)


def _workload_config(a, world, bs):
    return {"workload": f"{a.config} prefill-score {a.global_bs}x{a.seq} (1 greedy token per sequence), "
                        f"int8 weight-only linears, bf16 activations",
            "model": a.config, "global_batch": a.global_bs, "seq_len": a.seq, "per_gpu_batch": bs,
            "parallelism": f"dp{world} (independent full replicas, no collective)",
            "l2": "working set (0.9 GB weights + activations) larger than L2 every step"}


def run_reference(a, rank, world):
    """--impl reference: the reference's CPU FP32 path (oracle port of benchmark/f32_golden.py) on the
    host cores, rank 0 only.  Each step is a bounded sample of the workload -- one full decoder layer of one
    8192-token sequence -- and `ms_per_step` is the time those steps took; `value` extrapolates the mean
    layer time to whole-model tokens/s (the same unit as the GPU arm)."""
    if rank != 0:
        return
    from minicpm5_mk.mk_config import get_config
    from minicpm5_mk.replicas import shard_bounds

    cfg = get_config(a.config)
    threads = os.cpu_count() or 1
    smp = CpuLayerSample(cfg, a.seq, threads)
    for _ in range(a.warmup):
        smp.step()
    times = [smp.step() for _ in range(a.steps)]
    sec = statistics.mean(times)
    value = smp.tok_s(sec)
    sample = smp.describe(len(times), statistics.median(times))
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(sec * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": _workload_config(a, world, shard_bounds(a.global_bs, world, 0)[1]),
            "step": f"one decoder layer of one {a.seq}-token sequence (a bounded sample of the workload); value "
                    f"= {a.seq} tokens / ({cfg.num_layers} x mean step time)",
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(), "sample": sample},
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
    if a.vllm_child:
        role, mdir = a.vllm_child
        {"make": lambda: _vllm_child_make(a.config, mdir), "direct": lambda: _vllm_child_direct(a, mdir),
         "serve": lambda: _vllm_child_serve(a, mdir)}[role]()
        return
    if a.vllm_e2e:
        run_vllm_e2e(a)
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

    def all_ranks(vals):
        """Every rank's list of floats, rank by rank (the same collective on every rank)."""
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world == 1:
            return [t.tolist()]
        out = torch.empty((world, len(vals)), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(out, t)
        return out.tolist()

    # ---------------------------------------------------------------- latency at 1 x 8192
    # Measured first, before the throughput loop heats the GPU into its power cap (each of the two figures
    # is then taken in its own steady state, as the reference times its shapes in separate runs).
    lat = None
    if rank == 0 and a.latency_runs > 0:
        one = ids_dev[0][:S].contiguous()
        o1 = (hid[:1], lg[:1], top1[:1])
        for _ in range(5):
            eng.forward(one, 1, S, out=o1)
        torch.cuda.synchronize()
        ts = []
        lclk = _clock_sampler(local)
        for _ in range(a.latency_runs):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            eng.forward(one, 1, S, out=o1)
            s1.record(stream)
            s1.synchronize()
            ts.append(s0.elapsed_time(s1))
        lat_clocks = _clock_summary(lclk)
        ts.sort()

        def pct(p):
            k = (len(ts) - 1) * p / 100.0
            lo = int(k)
            hi = min(lo + 1, len(ts) - 1)
            return ts[lo] + (ts[hi] - ts[lo]) * (k - lo)

        lat = {"p50_ms": round(pct(50), 3), "p99_ms": round(pct(99), 3), "runs": len(ts), "warmup": 5,
               "timing": "device (CUDA events)", "clocks": lat_clocks}
    barrier()

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
    # every rank's own step time and median SM clock, to name the slowest replica
    per_rank = [{"rank": r, "ms_per_step": round(v[0], 3), "sequences": int(v[1]),
                 "sm_mhz": v[2] if v[2] >= 0 else None}
                for r, v in enumerate(all_ranks([dev_ms, float(bs), float((clocks or {}).get("sm_mhz") or -1)]))]
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
        cpu = {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
               "sample": desc}

    fl_step = _flops_per_seq(cfg, S) * a.global_bs
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _workload_config(a, world, bs),
        "model_tflops": round(fl_step / (step_ms / 1e3) / 1e12, 1),
        "model_roofline_frac": round(fl_step / (step_ms / 1e3) / 1e12 / (peak_sus * world), 4),
        "model_roofline_peak": "sustained bf16 GEMM peak per GPU",
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": eng.launches_per_forward(bs, S) * a.steps,
        "clocks": clocks, "per_rank": per_rank, "latency_1x8192": lat,
        "latency_1x8192_sp": lat_sp, "device_error": err,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
