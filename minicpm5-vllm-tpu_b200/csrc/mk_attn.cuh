// Causal GQA attention kernels.
//
// attn_prefill_kernel: full-sequence causal GQA flash attention (online softmax in f32).
//   Reference counterpart: `super_gqa_v2` (plugin/minicpm5_mk/mk_attn.py:557-710); math spec
//   `_attn_chunk` (benchmark/f32_golden.py:62-75).
//   One CTA = one KV head x one block of queries; its 8 warps are the G = n_q / n_kv query heads
//   of that KV group (stacked as 128 rows of 16 queries x 8 heads for G = 8), so every K/V tile is
//   staged in shared memory once per KV group and used by all of the group's heads.  Blocks are
//   scheduled heaviest-first (last query block first) to balance the causal triangle.
//   Q/K are expected already rotated (RoPE kernel) and Q pre-scaled by 1/sqrt(head_dim) (folded
//   into the Q weights); `scale_log2` multiplies raw scores into the exp2 domain.
//
// attn_last_kernel: attention of each sequence's last query against all of its keys (the last
//   layer only needs the last position), `last_layer_step` (plugin/minicpm5_mk/mk_jax.py:492-520).
#pragma once

#include "mk_common.cuh"

namespace mk {

struct AttnArgs {
  int S;          // sequence length
  int n_q, n_kv;  // heads
  int ld_qkv;     // elements per token row of the q/k/v buffer
  int q_col, k_col, v_col;  // column offsets of Q, K, V inside a row
  int ld_out;     // elements per token row of the output
  float scale_log2;
  int nqb;        // query blocks per sequence
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int ATT_ROWS = 128;  // (query, head) rows per CTA
constexpr int ATT_BK = 64;     // keys per tile
constexpr int ATT_THREADS = 256;

template <int HD>
struct AttnShape {
  static constexpr int RS = HD + 8;  // padded smem row (elements): conflict-free ldmatrix
  static constexpr size_t SMEM = static_cast<size_t>(ATT_ROWS + 4 * ATT_BK) * RS * 2;
};

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_prefill_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out, const AttnArgs a) {
  constexpr int RS = AttnShape<HD>::RS;
  constexpr int NKK = HD / 16;  // k-steps over head_dim for Q K^T
  constexpr int NDT = HD / 8;   // n-tiles over head_dim for P V
  extern __shared__ __align__(16) uint8_t att_smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(att_smem);
  __nv_bfloat16* sK = sQ + ATT_ROWS * RS;
  __nv_bfloat16* sV = sK + 2 * ATT_BK * RS;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.n_q / a.n_kv;
  const int QW = 8 / G;          // 16-query sub-blocks per CTA
  const int BQ = 16 * QW;
  const int qb = a.nqb - 1 - blockIdx.x;
  const int q0 = qb * BQ;
  const int g = blockIdx.y;
  const int b = blockIdx.z;
  const int hq = g * G + warp % G;
  const int qw0 = q0 + (warp / G) * 16;
  const __nv_bfloat16* base = qkv + static_cast<size_t>(b) * a.S * a.ld_qkv;

  // Q tile: row r = (warp r/16, row r%16)
  for (int c = tid; c < ATT_ROWS * (HD / 8); c += ATT_THREADS) {
    const int r = c / (HD / 8), cc = c % (HD / 8);
    const int wr = r >> 4, i = r & 15;
    const int head = g * G + wr % G;
    const int q = q0 + (wr / G) * 16 + i;
    cp_async16(sQ + r * RS + cc * 8, base + static_cast<size_t>(q) * a.ld_qkv + a.q_col + head * HD + cc * 8);
  }
  cp_async_commit();

  auto load_kv = [&](int j, int buf) {
    const int kb = j * ATT_BK;
    __nv_bfloat16* dk = sK + buf * ATT_BK * RS;
    __nv_bfloat16* dv = sV + buf * ATT_BK * RS;
    for (int c = tid; c < ATT_BK * (HD / 8); c += ATT_THREADS) {
      const int r = c / (HD / 8), cc = c % (HD / 8);
      const __nv_bfloat16* src = base + static_cast<size_t>(kb + r) * a.ld_qkv + g * HD + cc * 8;
      cp_async16(dk + r * RS + cc * 8, src + a.k_col);
      cp_async16(dv + r * RS + cc * 8, src + a.v_col);
    }
  };

  const int ntiles = (q0 + BQ - 1) / ATT_BK + 1;
  load_kv(0, 0);
  cp_async_commit();

  uint32_t qf[NKK][4];
  float o[NDT][4];
#pragma unroll
  for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int gq = lane >> 2, tq = lane & 3;
  const int qrow0 = qw0 + gq, qrow1 = qw0 + gq + 8;
  const float sc = a.scale_log2;

  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) {
      load_kv(j + 1, (j + 1) & 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
      const uint32_t qbase = smem_u32(sQ + (warp * 16) * RS);
#pragma unroll
      for (int kk = 0; kk < NKK; ++kk) {
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int cix = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qbase + (r * RS + cix) * 2, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const int kb = j * ATT_BK;
    if (kb <= qw0 + 15) {
      const __nv_bfloat16* tk = sK + (j & 1) * ATT_BK * RS;
      const __nv_bfloat16* tv = sV + (j & 1) * ATT_BK * RS;
      float s[ATT_BK / 8][4];
#pragma unroll
      for (int nt = 0; nt < ATT_BK / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < NKK; ++kk) {
#pragma unroll
        for (int nt = 0; nt < ATT_BK / 8; nt += 2) {
          const int mi = lane >> 3;
          const int key = nt * 8 + (mi >> 1) * 8 + (lane & 7);
          const int d = kk * 16 + (mi & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_u32(tk + key * RS + d), b0, b1, b2, b3);
          mma_16816(s[nt], qf[kk], b0, b1);
          mma_16816(s[nt + 1], qf[kk], b2, b3);
        }
      }
      // causal mask (only tiles that reach past the warp's first query need it)
      if (kb + ATT_BK - 1 > qw0) {
#pragma unroll
        for (int nt = 0; nt < ATT_BK / 8; ++nt) {
          const int k0 = kb + nt * 8 + 2 * tq;
          if (k0 > qrow0) s[nt][0] = -INFINITY;
          if (k0 + 1 > qrow0) s[nt][1] = -INFINITY;
          if (k0 > qrow1) s[nt][2] = -INFINITY;
          if (k0 + 1 > qrow1) s[nt][3] = -INFINITY;
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < ATT_BK / 8; ++nt) {
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
      const float mn0 = fmaxf(m0, mx0 * sc), mn1 = fmaxf(m1, mx1 * sc);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 *= al0;
      l1 *= al1;
#pragma unroll
      for (int dt = 0; dt < NDT; ++dt) {
        o[dt][0] *= al0;
        o[dt][1] *= al0;
        o[dt][2] *= al1;
        o[dt][3] *= al1;
      }
      uint32_t pf[ATT_BK / 16][4];
#pragma unroll
      for (int nt = 0; nt < ATT_BK / 8; ++nt) {
        const float p0 = exp2f(s[nt][0] * sc - mn0), p1 = exp2f(s[nt][1] * sc - mn0);
        const float p2 = exp2f(s[nt][2] * sc - mn1), p3 = exp2f(s[nt][3] * sc - mn1);
        l0 += p0 + p1;
        l1 += p2 + p3;
        pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(p0, p1);
        pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(p2, p3);
      }
#pragma unroll
      for (int kk = 0; kk < ATT_BK / 16; ++kk) {
        const uint32_t pa[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
        for (int dt = 0; dt < NDT; dt += 2) {
          const int mi = lane >> 3;
          const int key = kk * 16 + (mi & 1) * 8 + (lane & 7);
          const int d = (dt + (mi >> 1)) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(tv + key * RS + d), b0, b1, b2, b3);
          mma_16816(o[dt], pa, b0, b1);
          mma_16816(o[dt + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  l0 += __shfl_xor_sync(0xffffffff, l0, 1);
  l0 += __shfl_xor_sync(0xffffffff, l0, 2);
  l1 += __shfl_xor_sync(0xffffffff, l1, 1);
  l1 += __shfl_xor_sync(0xffffffff, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  __nv_bfloat16* o0 = out + (static_cast<size_t>(b) * a.S + qrow0) * a.ld_out + hq * HD;
  __nv_bfloat16* o1 = out + (static_cast<size_t>(b) * a.S + qrow1) * a.ld_out + hq * HD;
#pragma unroll
  for (int dt = 0; dt < NDT; ++dt) {
    const int d = dt * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(o0 + d) = pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
    *reinterpret_cast<uint32_t*>(o1 + d) = pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

// ----------------------------------------------------------------------------------------------
// Last-position attention: one CTA per (query head, sequence).  q: [bs, ld_q] (head h at h*HD),
// kv: [bs*S, ld_kv] with K at k_col and V at v_col.  Dynamic smem: S floats of scores.
struct AttnLastArgs {
  int S, n_q, n_kv, head_dim;
  int ld_q, ld_kv, k_col, v_col, ld_out;
  float scale_log2;
};

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (l < (blockDim.x >> 5)) ? red[l] : -INFINITY;
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (l < (blockDim.x >> 5)) ? red[l] : 0.f;
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

__global__ void __launch_bounds__(256)
    attn_last_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kv,
                     __nv_bfloat16* __restrict__ out, const AttnLastArgs a) {
  extern __shared__ float al_smem[];
  float* sc = al_smem;               // [S]
  __shared__ float qs[128];
  __shared__ float red[32];
  __shared__ float part[8][128];
  const int h = blockIdx.x, b = blockIdx.y;
  const int HD = a.head_dim;
  const int g = h / (a.n_q / a.n_kv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int d = tid; d < HD; d += blockDim.x)
    qs[d] = __bfloat162float(q[static_cast<size_t>(b) * a.ld_q + h * HD + d]);
  __syncthreads();
  const __nv_bfloat16* kb = kv + static_cast<size_t>(b) * a.S * a.ld_kv + a.k_col + g * HD;
  const __nv_bfloat16* vb = kv + static_cast<size_t>(b) * a.S * a.ld_kv + a.v_col + g * HD;
  float mx = -INFINITY;
  for (int j = tid; j < a.S; j += blockDim.x) {
    const uint4* kr = reinterpret_cast<const uint4*>(kb + static_cast<size_t>(j) * a.ld_kv);
    float acc = 0.f;
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 v = kr[c];
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w4[e]);
        acc += qs[c * 8 + 2 * e] * f.x + qs[c * 8 + 2 * e + 1] * f.y;
      }
    }
    acc *= a.scale_log2;
    sc[j] = acc;
    mx = fmaxf(mx, acc);
  }
  mx = block_reduce_max(mx, red);
  float sum = 0.f;
  for (int j = tid; j < a.S; j += blockDim.x) {
    const float p = exp2f(sc[j] - mx);
    sc[j] = p;
    sum += p;
  }
  sum = block_reduce_sum(sum, red);
  __syncthreads();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = warp; j < a.S; j += 8) {
    const float p = sc[j];
    const __nv_bfloat16* vr = vb + static_cast<size_t>(j) * a.ld_kv;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane + 32 * e;
      if (d < HD) acc[e] += p * __bfloat162float(vr[d]);
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane + 32 * e;
    if (d < HD) part[warp][d] = acc[e];
  }
  __syncthreads();
  const float inv = 1.f / sum;
  for (int d = tid; d < HD; d += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += part[w][d];
    out[static_cast<size_t>(b) * a.ld_out + h * HD + d] = __float2bfloat16(t * inv);
  }
}

}  // namespace mk
