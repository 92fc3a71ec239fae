// W8A16 GEMM for sm_100a: tcgen05.mma (bf16 x bf16 -> f32 in TMEM) fed by TMA, with the int8
// weight-only operand dequantised to bf16 in shared memory.
//
//   out[m, n] = epilogue( sum_k A[m, k] * Wq[n, k] )        A bf16 [M, K] row-major
//                                                           Wq int8 [N, K] row-major (per-output-
//                                                           channel scale s[n], f32)
// Epilogue modes (the per-row / per-column scalings commute with the sum, so they are applied to
// the f32 accumulator read back from TMEM):
//   ROWSCALE : out = bf16(acc * rstd[m] * s[n])                   RMSNorm-fused projections (QKV)
//   RESID    : out = bf16(out + r * acc * s[n])   (in place)       bf16 residual
//   RESID32  : x32 = x32 + r * acc * s[n] (f32, in place), out = bf16(x32)
//              o_proj / down + scaled residual on the f32 residual stream; `out` is the bf16 copy
//              the next projection reads as its A operand
//   SWIGLU   : tile = 128 gate + 128 up channels (interleaved weight rows);
//              h[m, i] = bf16(silu(g * rstd[m] * s_g) * (u * rstd[m] * s_u))   (out width N/2)
//
// Reference counterparts: `fused_qkv` (plugin/minicpm5_mk/mk_mlp.py:161-206), `linear` +
// residual (plugin/minicpm5_mk/mk_jax.py:233-269, :394), `fused_mlp`
// (plugin/minicpm5_mk/mk_mlp.py:68-145).
//
// CTA layout (persistent, one CTA per SM, 14 warps):
//   warp 0      : TMA producer (A tile 128x64 bf16 SW128, W tile 256x64 int8)
//   warp 1      : TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=256, K=16)
//   warps 2..5  : epilogue (TMEM -> registers -> global), one 32-lane TMEM quarter each
//   warps 6..13 : int8 -> bf16 converters writing the 128B-swizzled K-major B tile
// TMEM holds two 128x256 f32 accumulators (512 columns) so the epilogue of tile i overlaps the
// main loop of tile i+1.
#pragma once

#include "mk_common.cuh"

namespace mk {

enum GemmMode : int { GEMM_ROWSCALE = 0, GEMM_RESID = 1, GEMM_SWIGLU = 2, GEMM_COLSCALE = 3, GEMM_RESID32 = 4 };

constexpr int GM = 128;   // rows of A per tile (UMMA M)
constexpr int GN = 256;   // output channels per tile (UMMA N)
constexpr int GK = 64;    // K per stage (one 128-byte swizzle row of bf16)
constexpr int GSTAGES = 3;
constexpr int G_THREADS = 448;
constexpr int G_CONV_WARP0 = 6;
constexpr int G_CONV_WARPS = 8;
constexpr uint32_t G_A_BYTES = GM * GK * 2;     // 16 KB
constexpr uint32_t G_BQ_BYTES = GN * GK;        // 16 KB
constexpr uint32_t G_BH_BYTES = GN * GK * 2;    // 32 KB
constexpr uint32_t G_STAGE_BYTES = G_A_BYTES + G_BQ_BYTES + G_BH_BYTES;
constexpr uint32_t G_TMEM_COLS = 512;
constexpr size_t G_SMEM_BYTES = 1024 /*align pad*/ + GSTAGES * G_STAGE_BYTES + 256 /*barriers*/;

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
  int* err;
};

__global__ void __launch_bounds__(G_THREADS, 1)
    gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
  extern __shared__ uint8_t g_smem_raw[];
  const uint32_t raw = smem_u32(g_smem_raw);
  uint8_t* sbase = g_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + GSTAGES * G_STAGE_BYTES);
  uint64_t* full = bars;                 // [GSTAGES] TMA landed (A + int8 W)
  uint64_t* conv = bars + GSTAGES;       // [GSTAGES] bf16 W tile written
  uint64_t* empty = bars + 2 * GSTAGES;  // [GSTAGES] MMAs reading the stage finished
  uint64_t* tfull = bars + 3 * GSTAGES;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;          // [2] accumulator drained by the epilogue
  uint64_t* drain = tempty + 2;          // [1] all MMAs finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], G_CONV_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
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

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_par = 0;  // per-stage: ever issued / parity of the last issue
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mb = tile / num_n, nb = tile % num_n;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) goto producer_done;
          uint8_t* st = sbase + s * G_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], G_A_BYTES + G_BQ_BYTES);
          tma_load_2d(st, &tmA, &full[s], kt * GK, mb * GM);
          tma_load_2d(st + G_A_BYTES, &tmB, &full[s], kt * GK, nb * GN);
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == GSTAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    producer_done:
      // Every issued copy must land before the CTA may exit.
      for (int i = 0; i < GSTAGES; ++i)
        if (issued & (1u << i)) mbar_wait_drain(&full[i], (issued_par >> i) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(GM, GN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * GN;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&conv[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(sbase + s * G_STAGE_BYTES);
          const uint32_t sb = sa + G_A_BYTES + G_BQ_BYTES;
          const uint64_t da = sdesc_kmajor_sw128(sa);
          const uint64_t db = sdesc_kmajor_sw128(sb);
#pragma unroll
          for (int k = 0; k < GK / 16; ++k)
            mma_f16_ss(d, da + 2 * k, db + 2 * k, idesc, (kt | k) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);
          if (++s == GSTAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[a]);
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else if (warp < G_CONV_WARP0) {
    // -------------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mb = tile / num_n, nb = tile % num_n;
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!mbar_wait(&tfull[a], aph, abort_flag)) break;
      tc_fence_after();
      const int row = mb * GM + q * 32 + lane;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + a * GN + (static_cast<uint32_t>(q * 32) << 16);
      float rs = 1.0f;
      if ((args.mode == GEMM_ROWSCALE || args.mode == GEMM_SWIGLU) && row_ok) rs = __ldg(args.row_scale + row);
      if (args.mode == GEMM_SWIGLU) {
        const int n0 = nb * GN;           // weight rows: [n0, n0+128) gate, [n0+128, n0+256) up
        const int i0 = nb * (GN / 2);     // output channels
#pragma unroll 1
        for (int c0 = 0; c0 < GN / 2; c0 += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c0, g);
          tmem_ld_32x32b_x32(tbase + GN / 2 + c0, u);
          tmem_ld_wait();
          if (row_ok) {
            const float* sg = args.col_scale + n0 + c0;
            const float* su = args.col_scale + n0 + GN / 2 + c0;
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float g0 = __uint_as_float(g[2 * j]) * rs * __ldg(sg + 2 * j);
              const float g1 = __uint_as_float(g[2 * j + 1]) * rs * __ldg(sg + 2 * j + 1);
              const float u0 = __uint_as_float(u[2 * j]) * rs * __ldg(su + 2 * j);
              const float u1 = __uint_as_float(u[2 * j + 1]) * rs * __ldg(su + 2 * j + 1);
              o[j] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            }
            uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<size_t>(row) * args.ldo + i0 + c0);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
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
            const float* sc = args.col_scale + n0 + c0;
            uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<size_t>(row) * args.ldo + n0 + c0);
            uint32_t o[16];
            if (args.mode == GEMM_RESID32) {
              float4* xr = reinterpret_cast<float4*>(args.resid32 + static_cast<size_t>(row) * args.ld_resid32 + n0 + c0);
              const float r = args.resid_scale;
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 x = xr[v];
                x.x += r * (__uint_as_float(acc[4 * v + 0]) * __ldg(sc + 4 * v + 0));
                x.y += r * (__uint_as_float(acc[4 * v + 1]) * __ldg(sc + 4 * v + 1));
                x.z += r * (__uint_as_float(acc[4 * v + 2]) * __ldg(sc + 4 * v + 2));
                x.w += r * (__uint_as_float(acc[4 * v + 3]) * __ldg(sc + 4 * v + 3));
                xr[v] = x;
                o[2 * v] = pack_bf16x2(x.x, x.y);
                o[2 * v + 1] = pack_bf16x2(x.z, x.w);
              }
            } else if (args.mode == GEMM_RESID) {
              uint4 xin[4];
#pragma unroll
              for (int v = 0; v < 4; ++v) xin[v] = dst[v];
              const uint32_t* xw = reinterpret_cast<const uint32_t*>(xin);
              const float r = args.resid_scale;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float2 x = unpack_bf16x2(xw[j]);
                const float y0 = x.x + r * (__uint_as_float(acc[2 * j]) * __ldg(sc + 2 * j));
                const float y1 = x.y + r * (__uint_as_float(acc[2 * j + 1]) * __ldg(sc + 2 * j + 1));
                o[j] = pack_bf16x2(y0, y1);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                o[j] = pack_bf16x2(__uint_as_float(acc[2 * j]) * rs * __ldg(sc + 2 * j),
                                   __uint_as_float(acc[2 * j + 1]) * rs * __ldg(sc + 2 * j + 1));
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[a]);
    }
  } else {
    // -------------------------------------------------------------------- int8 -> bf16 converters
    const int ct = threadIdx.x - G_CONV_WARP0 * 32;  // 0..255
    int s = 0;
    uint32_t ph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      bool ok = true;
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[s], ph, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* bq = sbase + s * G_STAGE_BYTES + G_A_BYTES;
        uint8_t* bh = sbase + s * G_STAGE_BYTES + G_A_BYTES + G_BQ_BYTES;
#pragma unroll
        for (int i = 0; i < (GN * GK / 16) / (G_CONV_WARPS * 32); ++i) {
          const int c = ct + i * G_CONV_WARPS * 32;  // 16-byte chunk of the int8 tile
          const int n = c >> 2, kc = c & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(bq + n * GK + kc * 16);
          uint4 o0, o1;
          i8x4_to_bf16x4(v.x, o0.x, o0.y);
          i8x4_to_bf16x4(v.y, o0.z, o0.w);
          i8x4_to_bf16x4(v.z, o1.x, o1.y);
          i8x4_to_bf16x4(v.w, o1.z, o1.w);
          const int sw = n & 7;
          uint8_t* rowp = bh + n * 128;
          *reinterpret_cast<uint4*>(rowp + (((2 * kc) ^ sw) << 4)) = o0;
          *reinterpret_cast<uint4*>(rowp + (((2 * kc + 1) ^ sw) << 4)) = o1;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
        if (++s == GSTAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, G_TMEM_COLS);
  if (threadIdx.x == 0 && *abort_flag && args.err) atomicCAS(args.err, 0, DEV_ERR_TIMEOUT_GEMM);
}


// ==============================================================================================
// CTA-pair version (cluster of 2, tcgen05.mma.cta_group::2): one 256 x 256 output tile per pair.
// CTA r of the pair stages A rows [256 mb + 128 r, +128) and weight rows [256 nb + 128 r, +128)
// (int8 by TMA, converted to bf16 by its own converter warps), so each SM moves and converts half
// of the weight tile the single-CTA kernel needs.  The leader CTA (rank 0) issues the pair MMA
// (M = 256, N = 256) once every converter warp of both CTAs has arrived on its conv barrier; the
// MMA's completion is multicast to both CTAs' stage-release and accumulator-ready barriers.
// Each CTA's epilogue drains its own 128 x 256 accumulator and arrives on the leader's
// accumulator-free barrier.  No TMA multicast is used.
// ==============================================================================================
constexpr int P_STAGES = 5;
constexpr uint32_t P_A_BYTES = 128 * GK * 2;    // 16 KB
constexpr uint32_t P_BH_BYTES = 128 * GK * 2;   // 16 KB (bf16 half tile)
constexpr uint32_t P_BQ_BYTES = 128 * GK;       // 8 KB  (int8 half tile)
constexpr uint32_t P_STAGE_BYTES = P_A_BYTES + P_BH_BYTES + P_BQ_BYTES;
constexpr size_t P_SMEM_BYTES = 1024 + P_STAGES * P_STAGE_BYTES + 512;
constexpr int P_TILE_M = 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(G_THREADS, 1)
    gemm_w8a16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs args) {
  extern __shared__ uint8_t p_smem_raw[];
  const uint32_t raw = smem_u32(p_smem_raw);
  uint8_t* sbase = p_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + P_STAGES * P_STAGE_BYTES);
  uint64_t* full = bars;                  // [P_STAGES] local TMA landed (A + int8 W half)
  uint64_t* conv = bars + P_STAGES;       // [P_STAGES] this CTA's bf16 half written (local arrivals)
  uint64_t* empty = bars + 2 * P_STAGES;  // [P_STAGES] pair MMAs reading the stage finished
  uint64_t* tfull = bars + 3 * P_STAGES;  // [2] accumulator ready (multicast)
  uint64_t* tempty = tfull + 2;           // [2] leader: both epilogues drained the accumulator
  uint64_t* conv_peer = tempty + 2;       // [P_STAGES] leader: the peer's bf16 half written (relayed)
  uint64_t* drain = conv_peer + P_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const int cid = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], G_CONV_WARPS);
      mbar_init(&conv_peer[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, G_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (args.M + P_TILE_M - 1) / P_TILE_M;
  const int num_n = (args.N + GN - 1) / GN;
  const int num_tiles = num_m * num_n;
  const int KT = args.K / GK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer (own halves)
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_par = 0;
      for (int tile = cid; tile < num_tiles; tile += ncl) {
        const int mb = tile / num_n, nb = tile % num_n;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait_cluster(&empty[s], ph ^ 1u, abort_flag)) goto producer_done;
          uint8_t* st = sbase + s * P_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], P_A_BYTES + P_BQ_BYTES);
          tma_load_2d(st, &tmA, &full[s], kt * GK, mb * P_TILE_M + static_cast<int>(cta) * 128);
          tma_load_2d(st + P_A_BYTES + P_BH_BYTES, &tmB, &full[s], kt * GK, nb * GN + static_cast<int>(cta) * 128);
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == P_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    producer_done:
      for (int i = 0; i < P_STAGES; ++i)
        if (issued & (1u << i)) mbar_wait_drain(&full[i], (issued_par >> i) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0 && cta == 0) {
      // ------------------------------------------------------------------ pair MMA issuer (leader)
      constexpr uint32_t idesc = idesc_bf16_f32(P_TILE_M, GN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int tile = cid; tile < num_tiles; tile += ncl, ++it) {
        const int a = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait_cluster(&tempty[a], aph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * GN;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&conv[s], ph, abort_flag) || !mbar_wait_cluster(&conv_peer[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(sbase + s * P_STAGE_BYTES);
          const uint64_t da = sdesc_kmajor_sw128(sa);
          const uint64_t db = sdesc_kmajor_sw128(sa + P_A_BYTES);
#pragma unroll
          for (int k = 0; k < GK / 16; ++k)
            mma_f16_ss_pair(d, da + 2 * k, db + 2 * k, idesc, (kt | k) != 0 ? 1u : 0u);
          mma_commit_pair_mc(&empty[s], 0x3);
          if (++s == P_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair_mc(&tfull[a], 0x3);
      }
      mma_commit_pair(drain);
      mbar_wait_drain(drain, 0);
    } else if (lane == 0 && cta == 1) {
      // ------------------------------------------------------------------ relay (peer CTA)
      // Forwards "this CTA's bf16 half of stage s is written" to the leader with one cluster-scope
      // release per stage, so the converter warps only do CTA-local arrivals.
      int s = 0;
      uint32_t ph = 0;
      const int my_tiles = (num_tiles - cid + ncl - 1) / ncl;
      for (int idx = 0; idx < my_tiles * KT; ++idx) {
        if (!mbar_wait(&conv[s], ph, abort_flag)) break;
        mbar_arrive_remote(mapa_shared(smem_u32(&conv_peer[s]), 0));
        if (++s == P_STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp < G_CONV_WARP0) {
    // -------------------------------------------------------------------- epilogue (own 128 rows)
    const int q = warp & 3;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int it = 0;
    for (int tile = cid; tile < num_tiles; tile += ncl, ++it) {
      const int mb = tile / num_n, nb = tile % num_n;
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!mbar_wait_cluster(&tfull[a], aph, abort_flag)) break;
      tc_fence_after();
      const int row = mb * P_TILE_M + static_cast<int>(cta) * 128 + q * 32 + lane;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + a * GN + (static_cast<uint32_t>(q * 32) << 16);
      float rs = 1.0f;
      if ((args.mode == GEMM_ROWSCALE || args.mode == GEMM_SWIGLU) && row_ok) rs = __ldg(args.row_scale + row);
      if (args.mode == GEMM_SWIGLU) {
        const int n0 = nb * GN;
        const int i0 = nb * (GN / 2);
#pragma unroll 1
        for (int c0 = 0; c0 < GN / 2; c0 += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c0, g);
          tmem_ld_32x32b_x32(tbase + GN / 2 + c0, u);
          tmem_ld_wait();
          if (row_ok) {
            const float4* sg = reinterpret_cast<const float4*>(args.col_scale + n0 + c0);
            const float4* su = reinterpret_cast<const float4*>(args.col_scale + n0 + GN / 2 + c0);
            uint32_t o[16];
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 a4 = __ldg(sg + v), b4 = __ldg(su + v);
              const float ga[4] = {a4.x, a4.y, a4.z, a4.w}, ub[4] = {b4.x, b4.y, b4.z, b4.w};
              float hv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                hv[e] = silu_f(__uint_as_float(g[4 * v + e]) * rs * ga[e]) * (__uint_as_float(u[4 * v + e]) * rs * ub[e]);
              o[2 * v] = pack_bf16x2(hv[0], hv[1]);
              o[2 * v + 1] = pack_bf16x2(hv[2], hv[3]);
            }
            uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<size_t>(row) * args.ldo + i0 + c0);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
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
            if (args.mode == GEMM_RESID32) {
              float4* xr = reinterpret_cast<float4*>(args.resid32 + static_cast<size_t>(row) * args.ld_resid32 + n0 + c0);
              const float r = args.resid_scale;
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 x = xr[v];
                x.x += r * (__uint_as_float(acc[4 * v + 0]) * sc[4 * v + 0]);
                x.y += r * (__uint_as_float(acc[4 * v + 1]) * sc[4 * v + 1]);
                x.z += r * (__uint_as_float(acc[4 * v + 2]) * sc[4 * v + 2]);
                x.w += r * (__uint_as_float(acc[4 * v + 3]) * sc[4 * v + 3]);
                xr[v] = x;
                o[2 * v] = pack_bf16x2(x.x, x.y);
                o[2 * v + 1] = pack_bf16x2(x.z, x.w);
              }
            } else if (args.mode == GEMM_RESID) {
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
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                o[j] = pack_bf16x2(__uint_as_float(acc[2 * j]) * rs * sc[2 * j],
                                   __uint_as_float(acc[2 * j + 1]) * rs * sc[2 * j + 1]);
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(a ? tempty_leader1 : tempty_leader0);
    }
  } else {
    // -------------------------------------------------------------------- int8 -> bf16 converters (own half)
    const int ct = threadIdx.x - G_CONV_WARP0 * 32;  // 0..255
    int s = 0;
    uint32_t ph = 0;
    for (int tile = cid; tile < num_tiles; tile += ncl) {
      bool ok = true;
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[s], ph, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* bq = sbase + s * P_STAGE_BYTES + P_A_BYTES + P_BH_BYTES;
        uint8_t* bh = sbase + s * P_STAGE_BYTES + P_A_BYTES;
#pragma unroll
        for (int i = 0; i < (128 * GK / 16) / (G_CONV_WARPS * 32); ++i) {
          const int c = ct + i * G_CONV_WARPS * 32;
          const int n = c >> 2, kc = c & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(bq + n * GK + kc * 16);
          uint4 o0, o1;
          i8x4_to_bf16x4(v.x, o0.x, o0.y);
          i8x4_to_bf16x4(v.y, o0.z, o0.w);
          i8x4_to_bf16x4(v.z, o1.x, o1.y);
          i8x4_to_bf16x4(v.w, o1.z, o1.w);
          const int sw = n & 7;
          uint8_t* rowp = bh + n * 128;
          *reinterpret_cast<uint4*>(rowp + (((2 * kc) ^ sw) << 4)) = o0;
          *reinterpret_cast<uint4*>(rowp + (((2 * kc + 1) ^ sw) << 4)) = o1;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
        if (++s == P_STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs read both CTAs' shared memory: nobody leaves early
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, G_TMEM_COLS);
  if (threadIdx.x == 0 && *abort_flag && args.err) atomicCAS(args.err, 0, DEV_ERR_TIMEOUT_GEMM_PAIR);
}

}  // namespace mk
