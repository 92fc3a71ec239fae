// Last-position attention of the last layer (`last_layer_step`, plugin/minicpm5_mk/mk_jax.py:492-520):
// the last query of each sequence against all of its keys.  The full-sequence causal attention is
// attn_tc_kernel (mk_attn_tc.cuh).
//
// Split over keys (flash-decoding): one CTA per (KV group, sequence, block of AL_KEYS keys) scores the
// block for all G query heads of the group at once, so every K / V row is read once per group, and
// writes per head the block's running max, sum of exponentials and unnormalised output.  A second
// kernel combines the blocks of each (sequence, head) in block order.  A sequence of 8192 keys gives
// 64 blocks per group, 128 CTAs at batch 1 (one CTA per (head, sequence) walking all keys took 370 us).
#pragma once

#include "mk_common.cuh"

namespace mk {

constexpr int AL_KEYS = 128;    // keys per block (= threads of the block kernel)
constexpr int AL_GMAX = 8;      // query heads per KV head
constexpr int AL_HDMAX = 128;

// q: [bs, ld_q] (head h at h*HD), kv: [bs*S, ld_kv] with K at k_col and V at v_col.
struct AttnLastArgs {
  int S, n_q, n_kv, head_dim;
  int ld_q, ld_kv, k_col, v_col, ld_out;
  float scale_log2;
  int nblk;     // key blocks per sequence: ceil(S / AL_KEYS)
  float* part;  // [bs, n_q, nblk, head_dim + 2]: unnormalised output, block max, block sum
  SpLayout sp;  // sequence-parallel: kv is the rank-by-rank all-gather of one sequence (bs = 1)
};

// grid (nblk, n_kv, bs), AL_KEYS threads.
__global__ void __launch_bounds__(AL_KEYS)
    attn_last_block_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kv,
                           const AttnLastArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float qs[AL_GMAX][AL_HDMAX];
  __shared__ float ps[AL_GMAX][AL_KEYS];  // exponentials, then the exchange of the two key halves
  __shared__ float mred[AL_GMAX][AL_KEYS / 32];
  __shared__ float hm[AL_GMAX], hl[AL_GMAX];
  const int blk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int HD = a.head_dim, G = a.n_q / a.n_kv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < AL_GMAX * AL_HDMAX; i += blockDim.x) {
    const int hh = i / AL_HDMAX, d = i - hh * AL_HDMAX;
    qs[hh][d] = hh < G && d < HD ? __bfloat162float(q[static_cast<size_t>(b) * a.ld_q + (g * G + hh) * HD + d]) : 0.f;
  }
  __syncthreads();
  // scores: thread = key j of the block, all G heads
  const int j = blk * AL_KEYS + tid;
  const __nv_bfloat16* kvb = kv + static_cast<size_t>(b) * a.S * a.ld_kv;
  float sc[AL_GMAX];
#pragma unroll
  for (int hh = 0; hh < AL_GMAX; ++hh) sc[hh] = -INFINITY;
  if (j < a.S) {
    const uint4* kr = reinterpret_cast<const uint4*>(kvb + static_cast<size_t>(sp_row(a.sp, j)) * a.ld_kv + a.k_col +
                                                     g * HD);
#pragma unroll
    for (int hh = 0; hh < AL_GMAX; ++hh) sc[hh] = 0.f;
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 v = __ldg(kr + c);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w4[e]);
#pragma unroll
        for (int hh = 0; hh < AL_GMAX; ++hh) sc[hh] += qs[hh][c * 8 + 2 * e] * f.x + qs[hh][c * 8 + 2 * e + 1] * f.y;
      }
    }
#pragma unroll
    for (int hh = 0; hh < AL_GMAX; ++hh) sc[hh] = hh < G ? sc[hh] * a.scale_log2 : -INFINITY;
  }
  // per-head block max (finite for the heads of the group: every block holds at least one key)
#pragma unroll
  for (int hh = 0; hh < AL_GMAX; ++hh) {
    float m = sc[hh];
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) mred[hh][warp] = m;
  }
  __syncthreads();
  if (tid < AL_GMAX) {
    float m = mred[tid][0];
    for (int w = 1; w < AL_KEYS / 32; ++w) m = fmaxf(m, mred[tid][w]);
    hm[tid] = m;
  }
  __syncthreads();
#pragma unroll
  for (int hh = 0; hh < AL_GMAX; ++hh) {
    const float p = j < a.S && hh < G ? exp2f(sc[hh] - hm[hh]) : 0.f;
    ps[hh][tid] = p;
    float t = p;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) mred[hh][warp] = t;
  }
  __syncthreads();
  if (tid < AL_GMAX) {
    float l = 0.f;
    for (int w = 0; w < AL_KEYS / 32; ++w) l += mred[tid][w];
    hl[tid] = l;
  }
  // unnormalised outputs: thread = (pair of dimensions, half of the keys); the V rows are read once per
  // group, 4 bytes per thread, consecutive threads on consecutive dimensions
  const int npair = HD / 2;
  const int pair = tid % 64, half = tid / 64;
  float o0[AL_GMAX], o1[AL_GMAX];
#pragma unroll
  for (int hh = 0; hh < AL_GMAX; ++hh) o0[hh] = o1[hh] = 0.f;
  if (pair < npair) {
    const int k0 = half * (AL_KEYS / 2);
    for (int k = k0; k < k0 + AL_KEYS / 2; ++k) {
      const int jj = blk * AL_KEYS + k;
      if (jj >= a.S) break;
      const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(
          kvb + static_cast<size_t>(sp_row(a.sp, jj)) * a.ld_kv + a.v_col + g * HD + 2 * pair));
#pragma unroll
      for (int hh = 0; hh < AL_GMAX; ++hh) {
        const float p = ps[hh][k];
        o0[hh] += p * v.x;
        o1[hh] += p * v.y;
      }
    }
  }
  __syncthreads();  // every thread is done with ps: reuse it for the second half's partial outputs
  float* xo = &ps[0][0];  // [AL_GMAX][64][2] = 1024 floats = the size of ps
  if (half == 1 && pair < npair) {
#pragma unroll
    for (int hh = 0; hh < AL_GMAX; ++hh) {
      xo[(hh * 64 + pair) * 2] = o0[hh];
      xo[(hh * 64 + pair) * 2 + 1] = o1[hh];
    }
  }
  __syncthreads();
  if (half == 0 && pair < npair) {
#pragma unroll
    for (int hh = 0; hh < AL_GMAX; ++hh) {
      if (hh < G) {
        float* dst = a.part + ((static_cast<size_t>(b) * a.n_q + g * G + hh) * a.nblk + blk) * (HD + 2);
        dst[2 * pair] = o0[hh] + xo[(hh * 64 + pair) * 2];
        dst[2 * pair + 1] = o1[hh] + xo[(hh * 64 + pair) * 2 + 1];
        if (pair == 0) {
          dst[HD] = hm[hh];
          dst[HD + 1] = hl[hh];
        }
      }
    }
  }
}

// out[b, h*HD + d] = sum_blk o_blk[d] 2^(m_blk - M) / sum_blk l_blk 2^(m_blk - M), blocks in order.
// grid (n_q, bs), AL_HDMAX threads.
__global__ void __launch_bounds__(AL_HDMAX) attn_last_combine_kernel(__nv_bfloat16* __restrict__ out,
                                                                      const AttnLastArgs a) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int HD = a.head_dim;
  const float* p = a.part + (static_cast<size_t>(b) * a.n_q + h) * a.nblk * (HD + 2);
  float M = -INFINITY;
  for (int k = 0; k < a.nblk; ++k) M = fmaxf(M, p[k * (HD + 2) + HD]);
  float o = 0.f, l = 0.f;
  for (int k = 0; k < a.nblk; ++k) {
    const float* pk = p + k * (HD + 2);
    const float w = exp2f(pk[HD] - M);
    l += pk[HD + 1] * w;
    if (d < HD) o += pk[d] * w;
  }
  if (d < HD) out[static_cast<size_t>(b) * a.ld_out + h * HD + d] = __float2bfloat16(o / l);
}

}  // namespace mk
