// HBM-bound kernels around the GEMMs: embedding gather, RMSNorm row statistics, RoPE,
// last-row gather, final norm, lm_head + argmax.
#pragma once

#include "mk_common.cuh"

namespace mk {

// x32[t, :] = scale * E[ids[t], :] (f32 residual stream) and xb = bf16(x32) (the projections' A
// operand) -- `jnp.take(embed, ids)`, plugin/minicpm5_mk/mk_jax.py:532, with the MiniCPM scale_emb.
// One warp per token row, 16-byte vectors.  An id outside [0, V) writes a zero row and records
// DEV_ERR_BAD_TOKEN_ID.
__global__ void embed_kernel(const int32_t* __restrict__ ids, const __nv_bfloat16* __restrict__ E,
                             float* __restrict__ x32, __nv_bfloat16* __restrict__ xb, int T, int H, int V, float scale,
                             int* err, float* __restrict__ rowsq = nullptr, int rowsq_ld = 0,
                             SpLayout sp = SpLayout()) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int id = ids[sp_pos(sp, row)];  // sequence-parallel: ids are the whole sequence's
  uint4* db = reinterpret_cast<uint4*>(xb + static_cast<size_t>(row) * H);
  float4* d32 = reinterpret_cast<float4*>(x32 + static_cast<size_t>(row) * H);
  if (rowsq)  // fused RMSNorm statistics: the whole row's sum of squares in slot 0, other slots 0
    for (int p = lane; p < rowsq_ld; p += 32) rowsq[static_cast<size_t>(row) * rowsq_ld + p] = 0.f;
  if (id < 0 || id >= V) {
    if (lane == 0 && err) atomicCAS(err, 0, DEV_ERR_BAD_TOKEN_ID);
    for (int c = lane; c < H / 8; c += 32) {
      db[c] = make_uint4(0, 0, 0, 0);
      d32[2 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
      d32[2 * c + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(E + static_cast<size_t>(id) * H);
  float ss = 0.f;
  for (int c = lane; c < H / 8; c += 32) {
    uint4 v = __ldg(src + c);
    uint32_t* w = reinterpret_cast<uint32_t*>(&v);
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 p = unpack_bf16x2(w[e]);
      f[2 * e] = p.x * scale;
      f[2 * e + 1] = p.y * scale;
      w[e] = pack_bf16x2(f[2 * e], f[2 * e + 1]);
    }
    db[c] = v;
    d32[2 * c] = make_float4(f[0], f[1], f[2], f[3]);
    d32[2 * c + 1] = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
  }
  if (rowsq) {
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
    __syncwarp();
    if (lane == 0) rowsq[static_cast<size_t>(row) * rowsq_ld] = ss;
  }
}

// rstd[t] = rsqrt(mean(x[t]^2) + eps) over the f32 residual stream (`rms_norm_unit`,
// plugin/minicpm5_mk/mk_jax.py:32-36).  One warp per row.
__global__ void rms_rstd_kernel(const float* __restrict__ x, float* __restrict__ rstd, int T, int H, int ld,
                                float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * ld);
  float acc = 0.f;
  for (int c = lane; c < H / 4; c += 32) {
    const float4 v = __ldg(src + c);
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  if (lane == 0) rstd[row] = rsqrtf(acc / static_cast<float>(H) + eps);
}

// In-place rotate_half RoPE on `n_heads` consecutive heads starting at column col0 of each row:
//   x1' = x1 cos - x2 sin,  x2' = x2 cos + x1 sin      (benchmark/f32_golden.py:57-59, 88-89)
// position of row r = pos_base + r % seq; cos/sin tables are f32 [max_seq, hd/2].
// One thread per (row, head, pair of rotation indices).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int rows, int ld, int col0, int n_heads, int hd,
                            int seq, int pos_base) {
  const int half = hd / 2;
  const int pairs = half / 2;  // two rotation indices per thread
  const size_t total = static_cast<size_t>(rows) * n_heads * pairs;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(idx % pairs);
    const size_t rh = idx / pairs;
    const int h = static_cast<int>(rh % n_heads);
    const int r = static_cast<int>(rh / n_heads);
    const int pos = pos_base + r % seq;
    const int i = 2 * p;
    __nv_bfloat16* xp = x + static_cast<size_t>(r) * ld + col0 + h * hd;
    const float2 c = *reinterpret_cast<const float2*>(cos_t + static_cast<size_t>(pos) * half + i);
    const float2 s = *reinterpret_cast<const float2*>(sin_t + static_cast<size_t>(pos) * half + i);
    const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xp + i));
    const float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xp + half + i));
    *reinterpret_cast<uint32_t*>(xp + i) = pack_bf16x2(a.x * c.x - b.x * s.x, a.y * c.y - b.y * s.y);
    *reinterpret_cast<uint32_t*>(xp + half + i) = pack_bf16x2(b.x * c.x + a.x * s.x, b.y * c.y + a.y * s.y);
  }
}

// xl32[b, :] = x32[b*S + S-1, :], xlb = bf16 copy (the rows the last layer's token-local work needs).
__global__ void gather_last_kernel(const float* __restrict__ x32, float* __restrict__ xl32,
                                   __nv_bfloat16* __restrict__ xlb, int bs, int S, int H,
                                   const float* __restrict__ rowsq = nullptr, float* __restrict__ rowsql = nullptr,
                                   int rowsq_ld = 0) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const size_t srow = static_cast<size_t>(b) * S + S - 1;
  const float* src = x32 + srow * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float v = src[c];
    xl32[static_cast<size_t>(b) * H + c] = v;
    xlb[static_cast<size_t>(b) * H + c] = __float2bfloat16(v);
  }
  if (rowsq)
    for (int p = threadIdx.x; p < rowsq_ld; p += blockDim.x)
      rowsql[static_cast<size_t>(b) * rowsq_ld + p] = rowsq[srow * rowsq_ld + p];
}

// hf[b, :] = logit_scale * x[b] * rsqrt(mean(x[b]^2) + eps) * w   (f32; final norm of
// plugin/minicpm5_mk/mk_jax.py:569 with the logit scaling folded in); hidden[b, :] = bf16 of the
// unscaled normed row when requested (the reference op's (bs, H) bf16 output).
__global__ void final_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ hf,
                                  __nv_bfloat16* __restrict__ hidden, int H, float eps, float logit_scale) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* xr = x + static_cast<size_t>(b) * H;
  float acc = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float v = xr[k];
    acc += v * v;
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rs = rsqrtf(red[0] / static_cast<float>(H) + eps);
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float v = xr[k] * rs * w[k];
    hf[static_cast<size_t>(b) * H + k] = v * logit_scale;
    if (hidden) hidden[static_cast<size_t>(b) * H + k] = __float2bfloat16(v);
  }
}

// logits[b, v] = sum_k hf[b, k] * W[v, k] (f32 accumulate, bf16 W [V, H]) for up to NR rows per launch,
// with per-CTA argmax partials (value, lowest index on ties).  HBM-bound: W (225 MB for the 1B vocab) is
// streamed once per launch for all NR rows.
//
// Layout.  Warp = LM_R consecutive vocab rows at a time; lane l reads 16-byte chunks c = l, l + 32, ... of
// each row (a warp's load of one row is 512 contiguous bytes), so lane l owns the 8 k values of its chunks.
// The NR hidden rows sit in shared memory as f32 in a chunk-split layout, hs[n][half][c][4] holding
// hf[n][8c + 4 half + j], so each lane's 4 values of one half are one conflict-free 16-byte load.  Every
// weight value feeds NR FMAs and every loaded hidden value LM_R of them (two rows per packed f32x2 FMA).
// At the end of a vocab group the warp sums the LM_R x NR per-lane partials over its lanes (butterfly
// transpose-reduction) and each sum's owner lane stores the logit and keeps its running argmax.
constexpr int LM_THREADS = 256;
constexpr int LM_R = 4;  // vocab rows per warp group

// Rows per launch: 8 (the hidden rows of a launch take 8 * H * 4 bytes of shared memory, two CTAs per SM).
// At 16 rows the accumulators no longer fit the 128 registers a thread has at two CTAs per SM.
__host__ __device__ constexpr int lm_rows_max(int H) { return H * 8 * 4 <= 100 * 1024 ? 8 : 4; }

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// (d0, d1) += (a0, a1) * s in one packed f32x2 FMA.
__device__ __forceinline__ void fma2_acc(float& d0, float& d1, float a0, float a1, float s) {
  asm("{\n\t.reg .b64 x, y, z;\n\t"
      "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\tmov.b64 z, {%0, %1};\n\t"
      "fma.rn.f32x2 z, x, y, z;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(s));
}

// 16-byte streaming load of weights that are read once (not kept in L1).
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int NR>
__global__ void __launch_bounds__(LM_THREADS, 2)
    lm_head_kernel(const float* __restrict__ hf, const __nv_bfloat16* __restrict__ W, float* __restrict__ logits,
                   float* __restrict__ part_val, int* __restrict__ part_idx, int bs, int H, int V, int row0) {
  static_assert(NR == 1 || NR == 2 || NR == 4 || NR == 8, "rows per launch");
  constexpr int NV = LM_R * NR;  // partial sums per vocab group (index i = rr * NR + n)
  extern __shared__ float lm_smem[];  // [NR][2][H/8][4]
  __shared__ float bval[LM_THREADS / 32][NR];
  __shared__ int bidx[LM_THREADS / 32][NR];
  pdl_wait();
  pdl_trigger();
  const int nr = min(NR, bs - row0);
  const int kc = H / 8;  // 16-byte weight chunks per row
  for (int i = threadIdx.x; i < NR * H; i += blockDim.x) {
    const int n = i / H, k = i - n * H;
    const int c = k >> 3, e = k & 7;
    lm_smem[static_cast<size_t>(n) * H + (e >> 2) * (H >> 1) + c * 4 + (e & 3)] =
        n < nr ? hf[static_cast<size_t>(row0 + n) * H + k] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (LM_THREADS / 32);
  const int ngroups = (V + LM_R - 1) / LM_R;
  float best = -INFINITY;  // for row n = (owned index) % NR
  int bi = 0x7fffffff;
  for (int grp = blockIdx.x * (LM_THREADS / 32) + warp; grp < ngroups; grp += nwarps) {
    const int v0 = grp * LM_R;
    float acc[LM_R][NR];
#pragma unroll
    for (int rr = 0; rr < LM_R; ++rr)
#pragma unroll
      for (int n = 0; n < NR; ++n) acc[rr][n] = 0.f;
    // element offsets of the group's rows (V * H < 2^31 is checked on the host); rows past V repeat the
    // last one and their sums are dropped
    int wrow[LM_R];
#pragma unroll
    for (int rr = 0; rr < LM_R; ++rr) wrow[rr] = min(v0 + rr, V - 1) * H;
    // one chunk of every weight row is loaded a step ahead of the one being multiplied
    uint4 wn[LM_R];
    if (lane < kc) {
#pragma unroll
      for (int rr = 0; rr < LM_R; ++rr) wn[rr] = ldg_stream16(W + wrow[rr] + lane * 8);
    }
    for (int c = lane; c < kc; c += 32) {
      uint4 w[LM_R];
#pragma unroll
      for (int rr = 0; rr < LM_R; ++rr) w[rr] = wn[rr];
      if (c + 32 < kc) {
#pragma unroll
        for (int rr = 0; rr < LM_R; ++rr) wn[rr] = ldg_stream16(W + wrow[rr] + (c + 32) * 8);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float wf[LM_R][4];
#pragma unroll
        for (int rr = 0; rr < LM_R; ++rr) {
          const uint32_t lo = half ? w[rr].z : w[rr].x, hi = half ? w[rr].w : w[rr].y;
          const float2 a = unpack_bf16x2(lo), b = unpack_bf16x2(hi);
          wf[rr][0] = a.x;
          wf[rr][1] = a.y;
          wf[rr][2] = b.x;
          wf[rr][3] = b.y;
        }
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          const float4 hv = *reinterpret_cast<const float4*>(lm_smem + static_cast<size_t>(n) * H + half * (H >> 1) + c * 4);
          const float h4[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int rr = 0; rr < LM_R; rr += 2) fma2_acc(acc[rr][n], acc[rr + 1][n], wf[rr][j], wf[rr + 1][j], h4[j]);
          }
        }
      }
    }
    // sum the partials over the lanes; index i = rr * NR + n
    float* flat = &acc[0][0];
    if constexpr (NV >= 32) {
#pragma unroll
      for (int q = 0; q < NV / 32; ++q) {
        // in place: the partials are dead after the sum; lane owns index q * 32 + lane
        const float sum = warp_transpose_sum32(*reinterpret_cast<float(*)[32]>(flat + q * 32), lane);
        const int i = q * 32 + lane, rr = i / NR, n = i % NR, v = v0 + rr;
        if (v < V && n < nr) {
          logits[static_cast<size_t>(row0 + n) * V + v] = sum;
          if (better(sum, v, best, bi)) {
            best = sum;
            bi = v;
          }
        }
      }
    } else {
      float mine = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float t = flat[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == i) mine = t;
      }
      const int rr = lane / NR, n = lane % NR, v = v0 + rr;
      if (lane < NV && v < V && n < nr) {
        logits[static_cast<size_t>(row0 + n) * V + v] = mine;
        if (better(mine, v, best, bi)) {
          best = mine;
          bi = v;
        }
      }
    }
  }
  // lanes l, l ^ NR, l ^ 2NR, ... hold the same row n = l % NR
#pragma unroll
  for (int o = 16; o >= NR; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane < NR) {
    bval[warp][lane] = best;
    bidx[warp][lane] = bi;
  }
  __syncthreads();
  if (threadIdx.x < nr) {
    const int r = threadIdx.x;
    float bv = bval[0][r];
    int bb = bidx[0][r];
    for (int w = 1; w < LM_THREADS / 32; ++w)
      if (better(bval[w][r], bidx[w][r], bv, bb)) {
        bv = bval[w][r];
        bb = bidx[w][r];
      }
    part_val[static_cast<size_t>(row0 + r) * gridDim.x + blockIdx.x] = bv;
    part_idx[static_cast<size_t>(row0 + r) * gridDim.x + blockIdx.x] = bb;
  }
}

// top1[b] = argmax over the per-CTA partials of row b (warp-shuffle reduction, ties -> lowest id).
__global__ void argmax_reduce_kernel(const float* __restrict__ part_val, const int* __restrict__ part_idx,
                                     int nparts, int32_t* __restrict__ top1) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lane; i < nparts; i += 32) {
    const float v = part_val[static_cast<size_t>(b) * nparts + i];
    const int ix = part_idx[static_cast<size_t>(b) * nparts + i];
    if (better(v, ix, bv, bi)) {
      bv = v;
      bi = ix;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, bv, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) top1[b] = bi;
}

// ----------------------------------------------------------------------------------------------
// Top-k log-probabilities of each row of f32 logits [bs, V]: logprob = logit - logsumexp(row), and the
// k largest in descending order (equal logits: lower id first).  One 1024-thread CTA per row.
// Reference: the golden's log_softmax + top-k (benchmark/f32_golden.py:100-102), which the gate scorer
// compares (benchmark/gate.py:16-121); vLLM's logprobs path on the plugin's GPU runner.
// Selection runs k rounds of a block-wide arg-max restricted to the entries ordered after the previous
// pick in (value descending, id ascending) order, so no per-thread candidate lists are kept.
constexpr int TOPK_THREADS = 1024;
constexpr int TOPK_MAX = 64;

__device__ __forceinline__ bool topk_after(float v, int i, float pv, int pi) {
  return v < pv || (v == pv && i > pi);  // (v, i) comes after (pv, pi)
}
__device__ __forceinline__ bool topk_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(TOPK_THREADS)
    topk_logprobs_kernel(const float* __restrict__ logits, int V, int ld, int k, int32_t* __restrict__ ids,
                         float* __restrict__ lps) {
  __shared__ float red_v[TOPK_THREADS / 32];
  __shared__ int red_i[TOPK_THREADS / 32];
  __shared__ float bcast_v;
  __shared__ int bcast_i;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const float* row = logits + static_cast<size_t>(b) * ld;
  // 1) row max (the first pick) and 2) logsumexp
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += TOPK_THREADS) {
    const float v = row[i];
    if (topk_better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  auto block_best = [&](float v, int i) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (topk_better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    if (lane == 0) { red_v[w] = v; red_i[w] = i; }
    __syncthreads();
    if (w == 0) {
      v = red_v[lane];
      i = red_i[lane];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (topk_better(ov, oi, v, i)) { v = ov; i = oi; }
      }
      if (lane == 0) { bcast_v = v; bcast_i = i; }
    }
    __syncthreads();
  };
  block_best(bv, bi);
  const float m = bcast_v;
  float se = 0.f;
  for (int i = tid; i < V; i += TOPK_THREADS) se += __expf(row[i] - m);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
  __syncthreads();
  if (lane == 0) red_v[w] = se;
  __syncthreads();
  if (w == 0) {
    float t = red_v[lane];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red_v[0] = t;
  }
  __syncthreads();
  const float lse = m + logf(red_v[0]);
  __syncthreads();
  // 3) k picks
  float pv = bcast_v;
  int pi = bcast_i;
  if (tid == 0) {
    ids[static_cast<size_t>(b) * k] = pi;
    lps[static_cast<size_t>(b) * k] = pv - lse;
  }
  for (int r = 1; r < k; ++r) {
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int i = tid; i < V; i += TOPK_THREADS) {
      const float v = row[i];
      if (topk_after(v, i, pv, pi) && topk_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    block_best(bv, bi);
    pv = bcast_v;
    pi = bcast_i;
    if (tid == 0) {
      ids[static_cast<size_t>(b) * k + r] = pi;
      lps[static_cast<size_t>(b) * k + r] = pv - lse;
    }
    __syncthreads();
  }
}

}  // namespace mk
