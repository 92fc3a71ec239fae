// W8A16 GEMM for sm_100a: tcgen05.mma (bf16 x bf16 -> f32 in TMEM) fed by TMA, with the int8
// weight-only operand dequantised to bf16 in shared memory.
//
//   out[m, n] = epilogue( sum_k A[m, k] * Wq[n, k] )        A bf16 [M, K] row-major
//                                                           Wq int8 [N, K] row-major (per-output-
//                                                           channel scale s[n], f32)
// Epilogue modes (the per-row / per-column scalings commute with the sum, so they are applied to
// the f32 accumulator read back from TMEM):
//   ROWSCALE : out = bf16(acc * rstd[m] * s[n])                   RMSNorm-fused projections (QKV),
//              optionally with RoPE applied to the Q/K columns before the bf16 rounding
//   RESID    : out = bf16(out + r * acc * s[n])   (in place)       bf16 residual
//   RESID32  : x32 = x32 + r * acc * s[n] (f32, in place), out = bf16(x32)
//              o_proj / down + scaled residual on the f32 residual stream; `out` is the bf16 copy
//              the next projection reads as its A operand
//   SWIGLU   : tile = 64 gate + 64 up channels (interleaved weight rows);
//              h[m, i] = bf16(silu(g * rstd[m] * s_g) * (u * rstd[m] * s_u))   (out width N/2)
//
// Reference counterparts: `fused_qkv` (plugin/minicpm5_mk/mk_mlp.py:161-206), `linear` +
// residual (plugin/minicpm5_mk/mk_jax.py:233-269, :394), `fused_mlp`
// (plugin/minicpm5_mk/mk_mlp.py:68-145).
//
// CTA layout (persistent, one CTA per SM, 14 warps):
// Tile = 256 rows of A x 128 output channels: two M=128 UMMAs share one converted weight tile,
// so every converted weight element feeds 256 rows.
//   warp 0 lane 0 : TMA producer of the A tiles (256 x 64 bf16, 128B swizzle), 4-slot ring
//   warp 0 lane 1 : TMA producer of the int8 weight tiles (128 x 64), 4-slot ring that runs ahead
//   warp 1        : TMEM allocator + single-thread tcgen05.mma issuer (2 x M=128, N=128, K=16)
//   warps 2..5    : epilogue (TMEM -> registers -> global), one 32-lane TMEM quarter each; while a
//                   tile's main loop runs they prefetch that tile's residual rows into L2
//   warps 6..13   : int8 -> bf16 converters filling a 3-slot ring of 128B-swizzled K-major B tiles
// The three rings are decoupled so the weight loads and their conversion run ahead of the MMAs and
// only the A-tile load latency has to be covered by the A ring.  TMEM holds two 128x256 f32
// accumulators (2 x 256 columns, each two 128x128 halves) so the epilogue of tile i overlaps the main
// loop of tile i+1.
#pragma once

#include "mk_common.cuh"

namespace mk {

enum GemmMode : int { GEMM_ROWSCALE = 0, GEMM_RESID = 1, GEMM_SWIGLU = 2, GEMM_COLSCALE = 3, GEMM_RESID32 = 4 };

constexpr int GM = 256;   // rows of A per tile: two UMMA M=128 halves sharing one converted weight tile
constexpr int UM = 128;   // UMMA M
constexpr int GN = 128;   // output channels per tile (UMMA N)
constexpr int GK = 64;    // K per stage (one 128-byte swizzle row of bf16)
constexpr int GA_SLOTS = 4;
constexpr int GQ_SLOTS = 4;
constexpr int GH_SLOTS = 3;
constexpr int G_THREADS = 448;
constexpr int G_EPI_WARP0 = 2;
constexpr int G_EPI_WARPS = 4;   // one per 32-lane TMEM quarter
constexpr int G_CONV_WARP0 = G_EPI_WARP0 + G_EPI_WARPS;
constexpr int G_CONV_WARPS = 8;
constexpr uint32_t G_A_BYTES = GM * GK * 2;     // 32 KB (two 16 KB halves)
constexpr uint32_t G_BQ_BYTES = GN * GK;        // 8 KB
constexpr uint32_t G_BH_BYTES = GN * GK * 2;    // 16 KB
constexpr uint32_t G_RING_BYTES = GA_SLOTS * G_A_BYTES + GQ_SLOTS * G_BQ_BYTES + GH_SLOTS * G_BH_BYTES;
constexpr uint32_t G_TMEM_COLS = 512;
constexpr size_t G_SMEM_BYTES = 1024 /*align pad*/ + G_RING_BYTES + 512 /*barriers*/;
static_assert(G_SMEM_BYTES <= 232448, "shared memory budget");

struct GemmArgs {
  int M, N, K;
  int mode;
  const float* row_scale;  // [M] (ROWSCALE, SWIGLU)
  const float* col_scale;  // [N]
  __nv_bfloat16* out;      // [M, ldo]
  int ldo;
  float resid_scale;
  float* resid32;          // [M, ld_resid32] (RESID32)
  int ld_resid32;
  // Fused RMSNorm statistics.  RESID32 writes, per row and 128-column tile, the sum of squares of
  // the updated residual into rowsq[row * rowsq_ld + tile].  ROWSCALE / SWIGLU with rowsq != null
  // take rstd = rsqrt(sum over rowsq_np partials / norm_dim + eps) instead of row_scale.
  float* rowsq;
  int rowsq_ld, rowsq_np;
  float inv_norm_dim, eps;
  // Fused RoPE (ROWSCALE): columns [0, rope_cols) hold heads of width head_dim whose rotation pairs
  // (i, i + head_dim/2) are stored interleaved as adjacent columns (2j, 2j + 1); position of row m
  // is rope_pos_base + m % rope_seq; tables f32 [max_seq, head_dim/2].
  const float* rope_cos;
  const float* rope_sin;
  int rope_cols, head_dim, rope_seq, rope_pos_base;
  int* err;
};

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

template <int MODE>
__global__ void __launch_bounds__(G_THREADS, 1)
    gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
  extern __shared__ uint8_t g_smem_raw[];
  const uint32_t raw = smem_u32(g_smem_raw);
  uint8_t* sbase = g_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = sbase;                                   // [GA_SLOTS] 32 KB
  uint8_t* sH = sA + GA_SLOTS * G_A_BYTES;               // [GH_SLOTS] 16 KB (bf16 B)
  uint8_t* sQ = sH + GH_SLOTS * G_BH_BYTES;              // [GQ_SLOTS] 8 KB (int8 B)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + GQ_SLOTS * G_BQ_BYTES);
  uint64_t* a_full = bars;                   // [GA_SLOTS] TMA landed
  uint64_t* a_empty = a_full + GA_SLOTS;     // [GA_SLOTS] MMAs reading the slot finished
  uint64_t* q_full = a_empty + GA_SLOTS;     // [GQ_SLOTS] TMA landed
  uint64_t* q_empty = q_full + GQ_SLOTS;     // [GQ_SLOTS] converters read the slot
  uint64_t* h_full = q_empty + GQ_SLOTS;     // [GH_SLOTS] converters wrote the slot
  uint64_t* h_empty = h_full + GH_SLOTS;     // [GH_SLOTS] MMAs reading the slot finished
  uint64_t* tfull = h_empty + GH_SLOTS;      // [2] accumulator ready
  uint64_t* tempty = tfull + 2;              // [2] accumulator drained by the epilogue
  uint64_t* drain = tempty + 2;              // all MMAs finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GA_SLOTS; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < GQ_SLOTS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], G_CONV_WARPS);
    }
    for (int s = 0; s < GH_SLOTS; ++s) {
      mbar_init(&h_full[s], G_CONV_WARPS);
      mbar_init(&h_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], G_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, G_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (args.M + GM - 1) / GM;
  const int num_n = (args.N + GN - 1) / GN;
  const int num_tiles = num_m * num_n;
  const int KT = args.K / GK;
  const int my_tiles = (num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);
  const int total = my_tiles * KT;  // k-steps this CTA runs (slot index = k-step mod ring size)

  if (warp == 0) {
    if (lane < 2) {
      // ------------------------------------------------------------------ TMA producers
      // lane 0: A tiles into the A ring; lane 1: int8 weight tiles into the int8 ring.
      const bool is_a = lane == 0;
      const int slots = is_a ? GA_SLOTS : GQ_SLOTS;
      uint64_t* full = is_a ? a_full : q_full;
      uint64_t* empty = is_a ? a_empty : q_empty;
      uint32_t issued = 0, issued_par = 0;
      for (int idx = 0; idx < total; ++idx) {
        const int s = idx % slots;
        const uint32_t ph = (idx / slots) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
        const int tile = blockIdx.x + (idx / KT) * gridDim.x;
        const int kt = idx % KT;
        if (is_a) {
          mbar_arrive_expect_tx(&full[s], G_A_BYTES);
          tma_load_2d(sA + s * G_A_BYTES, &tmA, &full[s], kt * GK, (tile / num_n) * GM);
        } else {
          mbar_arrive_expect_tx(&full[s], G_BQ_BYTES);
          tma_load_2d(sQ + s * G_BQ_BYTES, &tmB, &full[s], kt * GK, (tile % num_n) * GN);
        }
        issued |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (ph << s);
      }
      // Every issued copy must land before the CTA may exit.
      for (int i = 0; i < slots; ++i)
        if (issued & (1u << i)) mbar_wait_drain(&full[i], (issued_par >> i) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(UM, GN);
      int idx = 0;
      bool ok = true;
      for (int it = 0; ok && it < my_tiles; ++it) {
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * 2 * GN;  // halves at +0 and +GN columns
        for (int kt = 0; kt < KT; ++kt, ++idx) {
          const int sa = idx % GA_SLOTS, sh = idx % GH_SLOTS;
          if (!mbar_wait(&a_full[sa], (idx / GA_SLOTS) & 1, abort_flag) ||
              !mbar_wait(&h_full[sh], (idx / GH_SLOTS) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = sdesc_kmajor_sw128(smem_u32(sH + sh * G_BH_BYTES));
#pragma unroll
          for (int mi = 0; mi < GM / UM; ++mi) {
            const uint64_t da = sdesc_kmajor_sw128(smem_u32(sA + sa * G_A_BYTES + mi * (G_A_BYTES / 2)));
#pragma unroll
            for (int k = 0; k < GK / 16; ++k)
              mma_f16_ss(d + mi * GN, da + 2 * k, db + 2 * k, idesc, (kt | k) != 0 ? 1u : 0u);
          }
          mma_commit(&a_empty[sa]);
          mma_commit(&h_empty[sh]);
        }
        if (!ok) break;
        mma_commit(&tfull[a]);
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else if (warp < G_CONV_WARP0) {
    // -------------------------------------------------------------------- epilogue
    const int q = warp & 3;                       // TMEM lane quarter this warp may access
    constexpr int ch = 0;                         // columns handled: the whole tile
    for (int it = 0; it < my_tiles; ++it) {
      const int tile = blockIdx.x + it * gridDim.x;
      const int mb = tile / num_n, nb = tile % num_n;
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (MODE == GEMM_RESID32) {
        // Pull the residual row segments (128 f32 = 512 B per row) of the NEXT tile into L2 while this
        // one is drained, so their loads hit L2 even when the epilogue is the bottleneck (the first
        // tile also prefetches its own rows).
#pragma unroll 1
        for (int pt = (it == 0 ? 0 : 1); pt <= 1; ++pt) {
          if (it + pt >= my_tiles) break;
          const int ptile = blockIdx.x + (it + pt) * gridDim.x;
          const int pmb = ptile / num_n, pnb = ptile % num_n;
#pragma unroll
          for (int mi = 0; mi < GM / UM; ++mi) {
            const int row = pmb * GM + mi * UM + q * 32 + lane;
            if (row < args.M) {
              const char* xr = reinterpret_cast<const char*>(args.resid32 +
                                                             static_cast<size_t>(row) * args.ld_resid32 + pnb * GN);
#pragma unroll
              for (int l2 = 0; l2 < 4; ++l2) prefetch_l2(xr + l2 * 128);
            }
          }
        }
      }
      // per-row scalars that do not depend on the accumulator: fetched before waiting for it
      float rs2[GM / UM];
#pragma unroll
      for (int mi = 0; mi < GM / UM; ++mi) {
        const int row = mb * GM + mi * UM + q * 32 + lane;
        rs2[mi] = 1.0f;
        if ((MODE == GEMM_ROWSCALE || MODE == GEMM_SWIGLU) && row < args.M) {
          if (args.rowsq) {
            const float* ps = args.rowsq + static_cast<size_t>(row) * args.rowsq_ld;
            float ss = 0.f;
            for (int p = 0; p < args.rowsq_np; ++p) ss += ps[p];
            rs2[mi] = rsqrtf(ss * args.inv_norm_dim + args.eps);
          } else {
            rs2[mi] = __ldg(args.row_scale + row);
          }
        }
      }
      if (!mbar_wait(&tfull[a], aph, abort_flag)) break;
      tc_fence_after();
#pragma unroll 1
      for (int mi = 0; mi < GM / UM; ++mi) {
        const int row = mb * GM + mi * UM + q * 32 + lane;
        const bool row_ok = row < args.M;
        const uint32_t tbase = tmem_base + a * 2 * GN + mi * GN + (static_cast<uint32_t>(q * 32) << 16);
        const float rs = mi == 0 ? rs2[0] : rs2[1];
        float sumsq = 0.f;  // RESID32: sum of squares of this row's updated 128-column segment
        if (MODE == GEMM_SWIGLU) {
          const int n0 = nb * GN;           // weight rows: [n0, n0+64) gate, [n0+64, n0+128) up
          const int i0 = nb * (GN / 2);     // output channels
#pragma unroll 1
          for (int c0 = 0; c0 < GN / 2; c0 += 16) {
            uint32_t g[16], u[16];
            tmem_ld_32x32b_x16(tbase + c0, g);
            tmem_ld_32x32b_x16(tbase + GN / 2 + c0, u);
            tmem_ld_wait();
            if (row_ok) {
              const float4* sg = reinterpret_cast<const float4*>(args.col_scale + n0 + c0);
              const float4* su = reinterpret_cast<const float4*>(args.col_scale + n0 + GN / 2 + c0);
              uint32_t o[8];
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const float4 a4 = __ldg(sg + v), b4 = __ldg(su + v);
                const float ga[4] = {a4.x, a4.y, a4.z, a4.w}, ub[4] = {b4.x, b4.y, b4.z, b4.w};
                float hv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  hv[e] = silu_f(__uint_as_float(g[4 * v + e]) * rs * ga[e]) *
                          (__uint_as_float(u[4 * v + e]) * rs * ub[e]);
                o[2 * v] = pack_bf16x2(hv[0], hv[1]);
                o[2 * v + 1] = pack_bf16x2(hv[2], hv[3]);
              }
              st_global_v8(args.out + static_cast<size_t>(row) * args.ldo + i0 + c0, o[0], o[1], o[2], o[3], o[4],
                           o[5], o[6], o[7]);
            }
          }
        } else {
          const int n0 = nb * GN;
#pragma unroll 1
          for (int c0 = 0; c0 < GN; c0 += 32) {
            uint32_t acc[32];
            tmem_ld_32x32b_x32(tbase + c0, acc);
            tmem_ld_wait();
            if (row_ok && n0 + c0 < args.N) {
              const float4* sc4 = reinterpret_cast<const float4*>(args.col_scale + n0 + c0);
              float sc[32];
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 t4 = __ldg(sc4 + v);
                sc[4 * v] = t4.x;
                sc[4 * v + 1] = t4.y;
                sc[4 * v + 2] = t4.z;
                sc[4 * v + 3] = t4.w;
              }
              uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<size_t>(row) * args.ldo + n0 + c0);
              uint32_t o[16];
              if (MODE == GEMM_RESID32) {
                float* xr = args.resid32 + static_cast<size_t>(row) * args.ld_resid32 + n0 + c0;
                const float r = args.resid_scale;
                float xv[4][8];
#pragma unroll
                for (int v = 0; v < 4; ++v) ld_global_v8(xr + 8 * v, xv[v]);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  float x[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) {
                    x[e] = xv[v][e] + r * (__uint_as_float(acc[8 * v + e]) * sc[8 * v + e]);
                    sumsq += x[e] * x[e];
                  }
                  st_global_v8(xr + 8 * v, __float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]),
                               __float_as_uint(x[3]), __float_as_uint(x[4]), __float_as_uint(x[5]),
                               __float_as_uint(x[6]), __float_as_uint(x[7]));
#pragma unroll
                  for (int e = 0; e < 4; ++e) o[4 * v + e] = pack_bf16x2(x[2 * e], x[2 * e + 1]);
                }
              } else if (MODE == GEMM_RESID) {
                uint4 xin[4];
#pragma unroll
                for (int v = 0; v < 4; ++v) xin[v] = dst[v];
                const uint32_t* xw = reinterpret_cast<const uint32_t*>(xin);
                const float r = args.resid_scale;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float2 x = unpack_bf16x2(xw[j]);
                  o[j] = pack_bf16x2(x.x + r * (__uint_as_float(acc[2 * j]) * sc[2 * j]),
                                     x.y + r * (__uint_as_float(acc[2 * j + 1]) * sc[2 * j + 1]));
                }
              } else if (n0 + c0 < args.rope_cols) {
                // projection + RoPE on adjacent (x_j, x_{j+hd/2}) pairs, rounded to bf16 once
                const int pos = args.rope_pos_base + row % args.rope_seq;
                const float* ct = args.rope_cos + static_cast<size_t>(pos) * (args.head_dim >> 1);
                const float* st = args.rope_sin + static_cast<size_t>(pos) * (args.head_dim >> 1);
                // head-local column of this 32-column chunk; a chunk crosses at most one head boundary
                const int hl0 = (n0 + c0) % args.head_dim;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  int hl = hl0 + 2 * j;
                  hl = hl >= args.head_dim ? hl - args.head_dim : hl;
                  const int pj = hl >> 1;
                  const float c = __ldg(ct + pj), sn = __ldg(st + pj);
                  const float xa = __uint_as_float(acc[2 * j]) * rs * sc[2 * j];
                  const float xb = __uint_as_float(acc[2 * j + 1]) * rs * sc[2 * j + 1];
                  o[j] = pack_bf16x2(xa * c - xb * sn, xb * c + xa * sn);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  o[j] = pack_bf16x2(__uint_as_float(acc[2 * j]) * rs * sc[2 * j],
                                     __uint_as_float(acc[2 * j + 1]) * rs * sc[2 * j + 1]);
              }
              st_global_v8(dst, o[0], o[1], o[2], o[3], o[4], o[5], o[6], o[7]);
              st_global_v8(dst + 2, o[8], o[9], o[10], o[11], o[12], o[13], o[14], o[15]);
            }
          }
          if (MODE == GEMM_RESID32 && args.rowsq && row_ok)
            args.rowsq[static_cast<size_t>(row) * args.rowsq_ld + nb] = sumsq;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[a]);
    }
  } else {
    // -------------------------------------------------------------------- int8 -> bf16 converters
    const int ct = threadIdx.x - G_CONV_WARP0 * 32;  // 0..255
    for (int idx = 0; idx < total; ++idx) {
      const int sq = idx % GQ_SLOTS, sh = idx % GH_SLOTS;
      if (!mbar_wait(&q_full[sq], (idx / GQ_SLOTS) & 1, abort_flag)) break;
      const uint8_t* bq = sQ + sq * G_BQ_BYTES;
      uint4 v[(GN * GK / 16) / (G_CONV_WARPS * 32)];
#pragma unroll
      for (int i = 0; i < (GN * GK / 16) / (G_CONV_WARPS * 32); ++i) {
        const int c = ct + i * G_CONV_WARPS * 32;
        v[i] = *reinterpret_cast<const uint4*>(bq + (c >> 2) * GK + (c & 3) * 16);
      }
      if (!mbar_wait(&h_empty[sh], ((idx / GH_SLOTS) & 1) ^ 1u, abort_flag)) break;
      uint8_t* bh = sH + sh * G_BH_BYTES;
#pragma unroll
      for (int i = 0; i < (GN * GK / 16) / (G_CONV_WARPS * 32); ++i) {
        const int c = ct + i * G_CONV_WARPS * 32;  // 16-byte chunk of the int8 tile
        const int n = c >> 2, kc = c & 3;
        uint4 o0, o1;
        i8x4_to_bf16x4(v[i].x, o0.x, o0.y);
        i8x4_to_bf16x4(v[i].y, o0.z, o0.w);
        i8x4_to_bf16x4(v[i].z, o1.x, o1.y);
        i8x4_to_bf16x4(v[i].w, o1.z, o1.w);
        const int sw = n & 7;
        uint8_t* rowp = bh + n * 128;
        *reinterpret_cast<uint4*>(rowp + (((2 * kc) ^ sw) << 4)) = o0;
        *reinterpret_cast<uint4*>(rowp + (((2 * kc + 1) ^ sw) << 4)) = o1;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&q_empty[sq]);  // int8 slot consumed (its values were used above): may be refilled
        mbar_arrive(&h_full[sh]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, G_TMEM_COLS);
  if (threadIdx.x == 0 && *abort_flag && args.err) atomicCAS(args.err, 0, DEV_ERR_TIMEOUT_GEMM);
}

}  // namespace mk
