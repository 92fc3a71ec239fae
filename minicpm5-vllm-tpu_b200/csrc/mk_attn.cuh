// attn_last_kernel: attention of each sequence's last query against all of its keys (the last
// layer only needs the last position), `last_layer_step` (plugin/minicpm5_mk/mk_jax.py:492-520).
// The full-sequence causal attention is attn_tc_kernel (mk_attn_tc.cuh).
#pragma once

#include "mk_common.cuh"

namespace mk {

// ----------------------------------------------------------------------------------------------
// Last-position attention: one CTA per (query head, sequence).  q: [bs, ld_q] (head h at h*HD),
// kv: [bs*S, ld_kv] with K at k_col and V at v_col.  Dynamic smem: S floats of scores.
struct AttnLastArgs {
  int S, n_q, n_kv, head_dim;
  int ld_q, ld_kv, k_col, v_col, ld_out;
  float scale_log2;
  SpLayout sp;  // sequence-parallel: kv is the rank-by-rank all-gather of one sequence (bs = 1)
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
    const uint4* kr = reinterpret_cast<const uint4*>(kb + static_cast<size_t>(sp_row(a.sp, j)) * a.ld_kv);
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
    const __nv_bfloat16* vr = vb + static_cast<size_t>(sp_row(a.sp, j)) * a.ld_kv;
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
