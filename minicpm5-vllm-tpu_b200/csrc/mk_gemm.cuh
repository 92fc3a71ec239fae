// W8A16 GEMM for sm_100a: tcgen05.mma with the int8 weight-only operand dequantised straight into
// tensor memory (the TMEM-A form of kind::f16), activations fed by TMA.
//
//   out[m, n] = epilogue( sum_k X[m, k] * Wq[n, k] )        X bf16 [M, K] row-major (tokens)
//                                                           Wq int8 [N, K] row-major (per-output-
//                                                           channel scale s[n], f32)
// The UMMA computes the transposed tile D[n, m] = Wq_tile . X_tile^T: the weight tile (128 output
// channels) is the A operand and lives in TMEM, the token tile is the B operand in shared memory.
// So the converted weights never touch shared memory: per k-step the tensor core reads only the
// token tile from shared memory, and the int8 -> bf16 conversion writes TMEM, which has its own
// bandwidth.  (The first version kept the converted weights in shared memory as the B operand;
// its shared-memory traffic per FLOP -- the tensor core reading both operands, TMA writes, the
// converters' loads and stores -- capped it near half of the bf16 peak.)
//
// Epilogue modes (the per-token / per-channel scalings commute with the sum, so they are applied
// to the f32 accumulator read back from TMEM):
//   ROWSCALE : out = bf16(acc * rstd[m] * s[n])                   RMSNorm-fused projections (QKV),
//              optionally with RoPE applied to the Q/K columns before the bf16 rounding
//   RESID    : out = bf16(out + r * acc * s[n])   (in place)       bf16 residual
//   RESID32  : x32 = x32 + r * acc * s[n] (f32, in place), out = bf16(x32)
//              o_proj / down + scaled residual on the f32 residual stream; `out` is the bf16 copy
//              the next projection reads as its A operand
//   SWIGLU   : weight rows alternate gate / up (row 2i = gate channel i, row 2i+1 = up channel i);
//              h[m, i] = bf16(silu(g * rstd[m] * s_g) * (u * rstd[m] * s_u))   (out width N/2)
//   COLSCALE : out = bf16(acc * s[n])
//
// Reference counterparts: `fused_qkv` (plugin/minicpm5_mk/mk_mlp.py:161-206), `linear` +
// residual (plugin/minicpm5_mk/mk_jax.py:233-269, :394), `fused_mlp`
// (plugin/minicpm5_mk/mk_mlp.py:68-145).
//
// CTA layout (persistent, one CTA per SM, 19 warps).  Tile = 128 output channels x nt tokens
// (nt = 192, or the token count rounded up to 16 when M is smaller); one pipeline stage covers 128 of K:
//   warp 0        : TMA producer of the token tiles (two nt x 64 bf16 panels per stage, 128B swizzle),
//                   3-slot ring; the warp runs the loop, one elected lane issues
//   warp 1        : TMEM allocator + tcgen05.mma issuer (M=128, N=nt, K=16, A in TMEM); the whole warp
//                   runs the loop (descriptors in uniform registers), one elected lane issues
//   warp 2        : TMA producer of the int8 weight tiles (128 x 128 B, 128B swizzle), 3-slot ring,
//                   run the same way as warp 0
//   warps 3..10   : epilogue (TMEM -> registers -> global), two warps per 32-lane TMEM quarter
//                   (= 32 output channels) taking alternate 32-token chunks; thread = channel,
//                   registers = consecutive tokens, so every global access of a warp covers 32
//                   consecutive channels of one token row
//   warps 11..18  : int8 -> bf16 converters, two per TMEM lane quarter (one half of the stage's K
//                   each): shared memory -> registers -> tcgen05.st into a 2-slot TMEM weight ring
// A warp can only reach the TMEM lane quarter of its SM sub-partition (warp slot mod 4), which fixes
// which quarter each epilogue and converter warp serves.
// TMEM (512 columns): two f32 accumulators of 192 columns (the epilogue of tile i overlaps the main
// loop of tile i+1) + 2 weight slots of 64 columns (128 x 128 bf16, two K values per column).
#pragma once

#include "mk_common.cuh"

namespace mk {

enum GemmMode : int { GEMM_ROWSCALE = 0, GEMM_RESID = 1, GEMM_SWIGLU = 2, GEMM_COLSCALE = 3, GEMM_RESID32 = 4 };

constexpr int GW = 128;   // output channels per tile (UMMA M, TMEM lanes)
constexpr int GT = 192;   // tokens per tile (UMMA N), upper bound of the runtime nt
constexpr int GK = 128;   // K per pipeline stage
constexpr int GKB = 64;   // K per token-tile TMA box (one 128-byte swizzle row of bf16)
constexpr int GX_SLOTS = 3;
constexpr int GQ_SLOTS = 3;
constexpr int GW_SLOTS = 2;
constexpr int G_THREADS = 608;
constexpr int G_QPROD_WARP = 2;  // int8 weight-tile producer (its own warp: a waiting lane of a shared
                                 // warp would hold up the other producer)
constexpr int G_EPI_WARP0 = 3;
constexpr int G_EPI_WARPS = 8;   // two per 32-lane TMEM quarter (alternate 32-token chunks)
constexpr int G_CONV_WARP0 = G_EPI_WARP0 + G_EPI_WARPS;
constexpr int G_CONV_WARPS = 8;  // two per 32-lane TMEM quarter (halves of the k-step)
constexpr uint32_t G_XSUB_BYTES = GT * GKB * 2;  // 24 KB: one 64-wide K panel of a token tile
constexpr uint32_t G_X_BYTES = 2 * G_XSUB_BYTES;  // 48 KB
constexpr uint32_t G_Q_BYTES = GW * GK;          // 16 KB
constexpr uint32_t G_TMEM_COLS = 512;
constexpr uint32_t G_W_COL0 = 2 * GT;         // weight ring after the two accumulators
constexpr uint32_t G_W_COLS = GK / 2;         // 64 columns per weight slot
static_assert(G_W_COL0 + GW_SLOTS * G_W_COLS <= G_TMEM_COLS, "TMEM budget");
static_assert(G_XSUB_BYTES % 1024 == 0 && G_Q_BYTES % 1024 == 0, "swizzle atoms stay aligned");
constexpr uint32_t G_RS_FLOATS = 2 * GT;                 // per-token rstd, double-buffered
constexpr uint32_t G_SS_FLOATS = 2 * 4 * GT;             // per-(lane quarter, token) sums of squares

// Weight-tile ring of the two weight formats: int8 (16 KB per 128 x 128 tile, 3 slots) or bf16 (two
// 128-row x 64-K panels of 16 KB per tile, 2 slots, so the ring still fits shared memory).
__host__ __device__ constexpr int gq_slots(bool wbf16) { return wbf16 ? 2 : GQ_SLOTS; }
__host__ __device__ constexpr uint32_t gq_bytes(bool wbf16) { return wbf16 ? 2 * G_Q_BYTES : G_Q_BYTES; }
__host__ __device__ constexpr size_t gemm_smem_bytes(bool wbf16) {
  return 1024 /*align pad*/ + GX_SLOTS * G_X_BYTES + gq_slots(wbf16) * gq_bytes(wbf16) +
         4 * (G_RS_FLOATS + G_SS_FLOATS) + 512;
}
constexpr size_t G_SMEM_BYTES = gemm_smem_bytes(false);
static_assert(gemm_smem_bytes(false) <= 232448 && gemm_smem_bytes(true) <= 232448, "shared memory budget");

// Tokens per tile for M tokens (a multiple of 16, the UMMA N granularity at M = 128).
__host__ __device__ constexpr int gemm_nt(int M) { return M >= GT ? GT : ((M + 15) / 16) * 16; }

struct GemmArgs {
  int M, N, K;
  int nt;                  // tokens per tile (gemm_nt(M)); the token tensor map's box height
  int mode;
  const float* row_scale;  // [M] (ROWSCALE, SWIGLU)
  const float* col_scale;  // [N]
  __nv_bfloat16* out;      // [M, ldo]
  int ldo;
  float resid_scale;
  float* resid32;          // [M, ld_resid32] (RESID32)
  int ld_resid32;
  // Fused RMSNorm statistics.  RESID32 writes, per token and 128-channel tile, the sum of squares
  // of the updated residual into rowsq[m * rowsq_ld + tile].  ROWSCALE / SWIGLU with rowsq != null
  // take rstd = rsqrt(sum over rowsq_np partials / norm_dim + eps) instead of row_scale.
  float* rowsq;
  int rowsq_ld, rowsq_np;
  float inv_norm_dim, eps;
  // Fused RoPE (ROWSCALE): columns [0, rope_cols) hold heads of width head_dim whose rotation pairs
  // (i, i + head_dim/2) are stored interleaved as adjacent columns (2j, 2j + 1); position of token m
  // is rope_pos_base + m % rope_seq; tables f32 [max_seq, head_dim/2].
  const float* rope_cos;
  const float* rope_sin;
  int rope_cols, head_dim, rope_seq, rope_pos_base;
  // Sequence-parallel rows (sp.blk > 0): token m is local row m of one zig-zag sequence, at
  // position sp_pos(sp, m); rope_seq is then the whole sequence's length and rope_pos_base 0.
  SpLayout sp;
  int* err;
};

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void st_global_b32(__nv_bfloat16* p, uint32_t v) { *reinterpret_cast<uint32_t*>(p) = v; }

// (d0, d1) = (a0, a1) * (b0, b1) and (d0, d1) += (a0, a1) * (b0, b1) as packed f32x2 operations.
__device__ __forceinline__ void mul2(float a0, float a1, float b0, float b1, float& d0, float& d1) {
  asm("{\n\t.reg .b64 x, y, z;\n\t"
      "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ void fma2(float a0, float a1, float b0, float b1, float& d0, float& d1) {
  asm("{\n\t.reg .b64 x, y, z;\n\t"
      "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%0, %1};\n\t"
      "fma.rn.f32x2 z, x, y, z;\n\tmov.b64 {%0, %1}, z;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void st_global_b16(__nv_bfloat16* p, float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  *p = b;
}

// WB: the weights are bf16 [N, K] instead of int8 (the same kernel without quantisation: the weight
// tiles arrive as two 64-K panels and the converter warps copy them into TMEM unchanged).
//
// PAIR: a cluster of two CTAs computes 256 output channels x nt tokens with 2-SM UMMAs (M = 256):
// each CTA converts its own 128 channels' weights into its TMEM and loads its half of the token tile
// (nt/2 rows; the token tensor map's box is nt/2 high), so each SM streams half the token bytes per
// FLOP.  The even CTA's MMA warp issues the MMAs; the token panels of both CTAs complete on the even
// CTA's x_full, both CTAs' converters and epilogues arrive on the even CTA's w_full and tempty, and its
// commits arrive on the barriers of both CTAs.  Each CTA's epilogue drains its own 128 channels.
template <int MODE, bool WB = false, bool PAIR = false>
__global__ void __launch_bounds__(G_THREADS, 1)
    gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                      const GemmArgs args) {
  constexpr int QS = gq_slots(WB);
  constexpr uint32_t QB = gq_bytes(WB);
  // Token ring: 3 slots of a whole tile's 128-K stage, or for a pair CTA (which loads half the tile's
  // rows) 6 slots in the same shared memory.  A token load takes about 2400 cycles to land whatever its
  // size, so the deeper ring is what lets the pair's MMAs run without waiting for it.
  constexpr int XS = PAIR ? 2 * GX_SLOTS : GX_SLOTS;
  constexpr uint32_t XSUB = PAIR ? G_XSUB_BYTES / 2 : G_XSUB_BYTES;  // one 64-K panel of the slot
  constexpr uint32_t XB = 2 * XSUB;
  static_assert(XS * XB == GX_SLOTS * G_X_BYTES && XSUB % 1024 == 0, "token ring layout");
  extern __shared__ uint8_t g_smem_raw[];
  const uint32_t raw = smem_u32(g_smem_raw);
  uint8_t* sbase = g_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sX = sbase;                                     // [XS] token stages
  uint8_t* sQ = sX + XS * XB;                              // [QS] weight tiles
  float* rs_s = reinterpret_cast<float*>(sQ + QS * QB);    // [2][GT]
  float* ss_s = rs_s + G_RS_FLOATS;                                    // [2][4][GT]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ss_s + G_SS_FLOATS);
  uint64_t* x_full = bars;                   // [XS] TMA landed
  uint64_t* x_empty = x_full + XS;           // [XS] MMAs reading the slot finished
  uint64_t* q_full = x_empty + XS;           // [QS] TMA landed
  uint64_t* q_empty = q_full + QS;           // [QS] converters read the slot
  uint64_t* w_full = q_empty + QS;           // [GW_SLOTS] converters wrote the TMEM weight slot
  uint64_t* w_empty = w_full + GW_SLOTS;     // [GW_SLOTS] MMAs reading the TMEM slot finished
  uint64_t* tfull = w_empty + GW_SLOTS;      // [2] accumulator ready
  uint64_t* tempty = tfull + 2;              // [2] accumulator drained by the epilogue
  uint64_t* esync = tempty + 2;              // [2] epilogue warps' shared per-token values ready
  uint64_t* drain = esync + 2;               // all MMAs finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;  // 0: the pair's MMA-issuing CTA
  // shared::cluster address of this CTA's barrier `b` in the even CTA / in the odd CTA
  auto lead_bar = [&](uint64_t* b) { return PAIR ? mapa_cluster(smem_u32(b), 0) : smem_u32(b); };
  auto peer_bar = [&](uint64_t* b) { return mapa_cluster(smem_u32(b), 1); };
  constexpr uint32_t kPairArrivals = PAIR ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < XS; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < QS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], G_CONV_WARPS);
    }
    for (int s = 0; s < GW_SLOTS; ++s) {
      mbar_init(&w_full[s], G_CONV_WARPS * kPairArrivals);
      mbar_init(&w_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], G_EPI_WARPS * kPairArrivals);
      mbar_init(&esync[a], G_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, G_TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, G_TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers and TMEM exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();

  const int nt = args.nt;
  const int num_c = args.N / GW;                 // 128-channel tiles
  const int num_u = PAIR ? num_c / 2 : num_c;    // channel units of a token tile (256 channels per pair)
  const int num_t = (args.M + nt - 1) / nt;      // token tiles
  const int num_tiles = num_t * num_u;
  const int KT = (args.K + GK - 1) / GK;  // K % 64 == 0; a last half stage covers K % 128 == 64
  const int unit = PAIR ? static_cast<int>(blockIdx.x) >> 1 : static_cast<int>(blockIdx.x);  // CTA or pair
  const int nunits = PAIR ? static_cast<int>(gridDim.x) >> 1 : static_cast<int>(gridDim.x);
  const int my_tiles = (num_tiles - unit + nunits - 1) / nunits;
  // token tile and 128-channel tile of this CTA in its it-th tile
  auto tile_tb = [&](int it) { return (unit + it * nunits) / num_u; };
  auto tile_cb = [&](int it) {
    const int u = (unit + it * nunits) % num_u;
    return PAIR ? 2 * u + static_cast<int>(crank) : u;
  };
  const int total = my_tiles * KT;  // k-steps this CTA runs (slot index = k-step mod ring size)

  if (warp == 0 || warp == G_QPROD_WARP) {
    // ------------------------------------------------------------------ TMA producers
    // warp 0: token tiles into the X ring; warp 2: int8 weight tiles into the int8 ring.  The whole
    // warp runs the loop (so slot indices and coordinates stay warp-uniform) and one elected lane
    // issues the copies.  Consecutive tiles of a CTA walk the channel tiles of one token tile, so the
    // 148 CTAs share a few token tiles in L2 at any time.
    const bool leader = elect_one();
    const bool is_x = warp == 0;
    // the token tiles come from the previous kernel; the weights are constant, so their producer (and the
    // converters and the MMA warp, which touch no global memory) start before the previous kernel ends
    if (is_x) pdl_wait();
    const int slots = is_x ? XS : QS;
    uint64_t* full = is_x ? x_full : q_full;
    uint64_t* empty = is_x ? x_empty : q_empty;
    // X panel bytes of the whole tile (a pair's two halves together complete the even CTA's x_full)
    const uint32_t x_panel = static_cast<uint32_t>(nt) * GKB * 2;
    const int x_row0 = PAIR ? static_cast<int>(crank) * (nt / 2) : 0;  // this CTA's half of the tile
    uint32_t issued = 0, issued_par = 0;
    for (int idx = 0; idx < total; ++idx) {
      const int s = idx % slots;
      const uint32_t ph = (idx / slots) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u, abort_flag))) break;
      const int it = idx / KT;
      const int kt = idx % KT;
      if (leader) {
        if (is_x) {
          const bool two = args.K - kt * GK > GKB;
          const int row = tile_tb(it) * nt + x_row0;
          if constexpr (PAIR) {
            if (crank == 0) mbar_arrive_expect_tx(&full[s], two ? 2 * x_panel : x_panel);
            const uint32_t fb = lead_bar(&full[s]);
            tma_load_2d_pair(sX + s * XB, &tmX, fb, kt * GK, row);
            if (two) tma_load_2d_pair(sX + s * XB + XSUB, &tmX, fb, kt * GK + GKB, row);
          } else {
            mbar_arrive_expect_tx(&full[s], two ? 2 * x_panel : x_panel);
            tma_load_2d(sX + s * XB, &tmX, &full[s], kt * GK, row);
            if (two) tma_load_2d(sX + s * XB + XSUB, &tmX, &full[s], kt * GK + GKB, row);
          }
        } else {
          // int8: one 128 x 128 box; bf16: two 128-row x 64-K boxes.  A half last stage reads zeros
          // past K.
          mbar_arrive_expect_tx(&full[s], QB);
          tma_load_2d(sQ + s * QB, &tmW, &full[s], kt * GK, tile_cb(it) * GW);
          if (WB) tma_load_2d(sQ + s * QB + G_Q_BYTES, &tmW, &full[s], kt * GK + GKB, tile_cb(it) * GW);
        }
      }
      __syncwarp();
      issued |= 1u << s;
      issued_par = (issued_par & ~(1u << s)) | (ph << s);
    }
    // Every issued copy must land before the CTA may exit.  (An odd CTA's token panels complete on the
    // even CTA's barrier, which waits for both halves; the pair leaves together after a cluster barrier.)
    if (!PAIR || crank == 0 || !is_x)
      for (int i = 0; i < slots; ++i)
        if (issued & (1u << i)) mbar_wait_drain(&full[i], (issued_par >> i) & 1u);
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop, so TMEM addresses and smem descriptors are warp-uniform values
    // (uniform registers feed tcgen05.mma directly); one elected lane issues the tcgen05 ops.
    const bool leader = elect_one();
    const uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * GW : GW, nt);
    int idx = 0;
    bool ok = !PAIR || crank == 0;  // the odd CTA of a pair issues nothing
    // arrive (on both CTAs' copies for a pair) when the MMAs issued so far have completed
    auto commit_all = [&](uint64_t* b) {
      if constexpr (PAIR) {
        mma_commit_pair(smem_u32(b));
        mma_commit_pair(peer_bar(b));
      } else {
        mma_commit(b);
      }
    };
    auto wait_cl = [&](uint64_t* b, uint32_t par) { return mbar_wait(b, par, abort_flag); };
    for (int it = 0; ok && it < my_tiles; ++it) {
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!__all_sync(0xffffffffu, wait_cl(&tempty[a], aph ^ 1u))) break;
      tc_fence_after();
      const uint32_t d = tmem_base + a * GT;
      for (int kt = 0; kt < KT; ++kt, ++idx) {
        const int sx = idx % XS, sw = idx % GW_SLOTS;
        ok = __all_sync(0xffffffffu, wait_cl(&x_full[sx], (idx / XS) & 1) &&
                                         wait_cl(&w_full[sw], (idx / GW_SLOTS) & 1));
        if (!ok) break;
        tc_fence_after();
        const uint64_t db0 = sdesc_kmajor_sw128(smem_u32(sX + sx * XB));
        const uint64_t db1 = sdesc_kmajor_sw128(smem_u32(sX + sx * XB + XSUB));
        const uint32_t wa = tmem_base + G_W_COL0 + sw * G_W_COLS;
        const int nk = args.K - kt * GK > GKB ? GK / 16 : GKB / 16;
        if (leader) {
#pragma unroll
          for (int k = 0; k < GK / 16; ++k)
            if (k < nk) {
              const uint64_t db = (k < 4 ? db0 : db1) + 2 * (k & 3);
              if constexpr (PAIR)
                mma_f16_ts_pair(d, wa + k * 8, db, idesc, (kt | k) != 0 ? 1u : 0u);
              else
                mma_f16_ts(d, wa + k * 8, db, idesc, (kt | k) != 0 ? 1u : 0u);
            }
          commit_all(&x_empty[sx]);
          commit_all(&w_empty[sw]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (leader) commit_all(&tfull[a]);
      __syncwarp();
    }
    if (!PAIR || crank == 0) {
      if (leader) {
        if constexpr (PAIR)
          mma_commit_pair(smem_u32(drain));
        else
          mma_commit(drain);
      }
      __syncwarp();
      mbar_wait_drain(drain, 0);
    }
  } else if (warp < G_CONV_WARP0) {
    // -------------------------------------------------------------------- epilogue
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    const int eh = (warp - G_EPI_WARP0) >> 2;  // which alternate 32-token chunks
    const int et = (warp - G_EPI_WARP0) * 32 + lane;
    const int ch = q * 32 + lane;            // output channel within the tile (= TMEM lane)
    const float r = args.resid_scale;
    pdl_wait();  // statistics, residual and outputs are shared with earlier kernels
    for (int it = 0; it < my_tiles; ++it) {
      const int tb = tile_tb(it), cb = tile_cb(it);
      const int a = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      const int tok0 = tb * nt;
      const int n = cb * GW + ch;
      if (MODE == GEMM_RESID32) {
        // Pull the residual rows (128 f32 = 512 B per token) of the next tile into L2 while this one
        // is drained (the first tile also prefetches its own rows).
        for (int pt = (it == 0 ? 0 : 1); pt <= 1; ++pt) {
          if (it + pt >= my_tiles) break;
          const int ptok0 = tile_tb(it + pt) * nt, pcb = tile_cb(it + pt);
          for (int l = et; l < nt * 4; l += G_EPI_WARPS * 32) {
            const int tok = ptok0 + (l >> 2);
            if (tok < args.M)
              prefetch_l2(args.resid32 + static_cast<size_t>(tok) * args.ld_resid32 + pcb * GW + (l & 3) * 32);
          }
        }
      }
      float* rsb = rs_s + a * GT;
      if (MODE == GEMM_ROWSCALE || MODE == GEMM_SWIGLU) {
        // per-token rstd of this tile, shared by the epilogue warps; computed before the
        // accumulator wait so it overlaps the main loop
        for (int j = et; j < nt; j += G_EPI_WARPS * 32) {
          const int tok = tok0 + j;
          float v = 1.0f;
          if (tok < args.M) {
            if (args.rowsq) {
              const float* ps = args.rowsq + static_cast<size_t>(tok) * args.rowsq_ld;
              float ss = 0.f;
              for (int p = 0; p < args.rowsq_np; ++p) ss += ps[p];
              v = rsqrtf(ss * args.inv_norm_dim + args.eps);
            } else {
              v = __ldg(args.row_scale + tok);
            }
          }
          rsb[j] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&esync[a]);
        if (!mbar_wait(&esync[a], aph, abort_flag)) break;
      }
      const float cs = __ldg(args.col_scale + n);
      // RESID32: the residual values of the warp's next chunk are loaded one chunk ahead (the first
      // before the accumulator wait), so their latency overlaps TMEM reads and the reduction.
      float xv[32];
      auto load_resid = [&](int c0) {
        const int jn = min(min(32, nt - c0), args.M - (tok0 + c0));
        const float* xr = args.resid32 + static_cast<size_t>(tok0 + c0) * args.ld_resid32 + n;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < jn) xv[j] = xr[static_cast<size_t>(j) * args.ld_resid32];
      };
      if (MODE == GEMM_RESID32 && eh * 32 < nt) load_resid(eh * 32);
      if (!mbar_wait(&tfull[a], aph, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + a * GT + (static_cast<uint32_t>(q * 32) << 16);
      float* ssb = ss_s + (a * 4 + q) * GT;
      // RoPE: rows n and n ^ 1 (adjacent lanes) form a rotation pair; rope_cols is a multiple of 32
      // for the supported head sizes, so the test is uniform across the warp.
      const bool rope = MODE == GEMM_ROWSCALE && cb * GW + q * 32 < args.rope_cols;
      const int pj = rope ? (n % args.head_dim) >> 1 : 0;
      const int hh = args.head_dim >> 1;
      // RoPE steps of this lane's rotation pair (the table's position-1 and position-2 entries), the sine
      // carrying the lane's sign: the even lane of a pair computes x_a c - x_b s, the odd one x_b c + x_a s
      const bool odd_lane = (lane & 1) != 0;
      const float sg = odd_lane ? 1.f : -1.f;
      float rct = 1.f, rst = 0.f, rct2 = 1.f, rst2 = 0.f;
      if (MODE == GEMM_ROWSCALE && rope && args.rope_seq >= 32) {
        rct = __ldg(args.rope_cos + hh + pj);
        rst = sg * __ldg(args.rope_sin + hh + pj);
        rct2 = __ldg(args.rope_cos + 2 * hh + pj);
        rst2 = sg * __ldg(args.rope_sin + 2 * hh + pj);
      }
#pragma unroll 1
      for (int c0 = eh * 32; c0 < nt; c0 += 64) {
        const int tokc = tok0 + c0;
        const int jn = min(min(32, nt - c0), args.M - tokc);  // valid tokens of the chunk (warp-uniform)
        // RoPE chunk whose 32 tokens have consecutive positions: its four table entries (one per 8
        // positions) are requested before the accumulator load, so their latency overlaps it
        int p0 = 0;
        bool rope_run = false;
        float tcs[4] = {1.f, 1.f, 1.f, 1.f}, tsn[4] = {0.f, 0.f, 0.f, 0.f};
        if (MODE == GEMM_ROWSCALE && rope && jn > 0) {
          // zig-zag blocks are multiples of 32 tokens, so a chunk's positions stay consecutive
          p0 = args.sp.blk > 0 ? sp_pos(args.sp, tokc) : args.rope_seq >= 32 ? tokc % args.rope_seq : 0;
          rope_run = args.rope_seq >= 32 && p0 + 32 <= args.rope_seq;
          if (rope_run) {
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              const size_t e = static_cast<size_t>(p0 + 8 * qd + args.rope_pos_base) * hh + pj;
              tcs[qd] = __ldg(args.rope_cos + e);
              tsn[qd] = __ldg(args.rope_sin + e);
            }
          }
        }
        uint32_t acc[32];
        tmem_ld_32x32b_x32(tbase + c0, acc);
        tmem_ld_wait();
        if (jn <= 0) continue;
        if (MODE == GEMM_RESID32) {
          float* xr = args.resid32 + static_cast<size_t>(tokc) * args.ld_resid32 + n;
          __nv_bfloat16* ob = args.out + static_cast<size_t>(tokc) * args.ldo + n;
          float sq[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = xv[j] + r * (__uint_as_float(acc[j]) * cs);
            if (j < jn) {
              xr[static_cast<size_t>(j) * args.ld_resid32] = x;
              st_global_b16(ob + static_cast<size_t>(j) * args.ldo, x);
            }
            sq[j] = j < jn ? x * x : 0.f;
          }
          if (c0 + 64 < nt) load_resid(c0 + 64);
          const float ss = warp_transpose_sum32(sq, lane);
          if (c0 + lane < nt) ssb[c0 + lane] = ss;
        } else if (MODE == GEMM_SWIGLU) {
          // even lane = gate row of channel i, odd lane = up row; the even lane outputs the even
          // token of each pair, the odd lane the odd token
          const int i = (cb * GW + ch) >> 1;
          const bool odd = (lane & 1) != 0;
          __nv_bfloat16* ob = args.out + static_cast<size_t>(tokc + (odd ? 1 : 0)) * args.ldo + i;
#pragma unroll
          for (int j4 = 0; j4 < 32; j4 += 4) {
            const float4 r4 = *reinterpret_cast<const float4*>(rsb + c0 + j4);  // broadcast
            const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              const int j0 = j4 + h;
              const float x0 = __uint_as_float(acc[j0]) * rr[h] * cs;
              const float x1 = __uint_as_float(acc[j0 + 1]) * rr[h + 1] * cs;
              const float recv = __shfl_xor_sync(0xffffffffu, odd ? x0 : x1, 1);
              const float g = odd ? recv : x0, u = odd ? x1 : recv;
              if (j0 + (odd ? 1 : 0) < jn) st_global_b16(ob + static_cast<size_t>(j0) * args.ldo, silu_f(g) * u);
            }
          }
        } else if (MODE == GEMM_RESID) {
          __nv_bfloat16* ob = args.out + static_cast<size_t>(tokc) * args.ldo + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < jn) {
              const float x = __bfloat162float(ob[static_cast<size_t>(j) * args.ldo]);
              st_global_b16(ob + static_cast<size_t>(j) * args.ldo, x + r * (__uint_as_float(acc[j]) * cs));
            }
        } else if (MODE == GEMM_ROWSCALE) {
          __nv_bfloat16* ob = args.out + static_cast<size_t>(tokc) * args.ldo + n;
          if (rope) {
            const bool odd = odd_lane;
            if (rope_run) {
              // The chunk's 32 tokens have consecutive positions: (cos, sin) of the pair's angle at
              // each position follow from a table entry by the angle-addition rotation.  The table is read
              // every 8 positions (at p, with the one-position step giving p + 1), and the token pairs
              // (p + 2k, p + 2k + 1) then advance together by the two-position step (the table's position-2
              // entry), so at most 3 rotations (a few f32 ulps) separate any value from a table entry.
              // Token pairs also share the packed f32x2 arithmetic, and adjacent lanes swap one result so
              // that each stores two channels of one token as one 32-bit word.
              const float ct = rct, st = rst, ct2 = rct2, st2 = rst2;
#pragma unroll
              for (int hb = 0; hb < 32; hb += 8) {
                float cA = tcs[hb >> 3], sA = sg * tsn[hb >> 3];
                float cB = cA * ct - sA * st, sB = sA * ct + cA * st;
#pragma unroll
                for (int jj = 0; jj < 8; jj += 2) {
                  const int j = hb + jj;
                  const float2 r2 = *reinterpret_cast<const float2*>(rsb + c0 + j);  // broadcast
                  float xA, xB;
                  mul2(__uint_as_float(acc[j]), __uint_as_float(acc[j + 1]), r2.x * cs, r2.y * cs, xA, xB);
                  const float yA = __shfl_xor_sync(0xffffffffu, xA, 1);
                  const float yB = __shfl_xor_sync(0xffffffffu, xB, 1);
                  float oA, oB;
                  mul2(xA, xB, cA, cB, oA, oB);
                  fma2(yA, yB, sA, sB, oA, oB);
                  // even lane: token j, channels (n, n + 1); odd lane: token j + 1, channels (n - 1, n)
                  const float other = __shfl_xor_sync(0xffffffffu, odd ? oA : oB, 1);
                  if (odd) {
                    if (j + 1 < jn) st_global_b32(ob - 1 + static_cast<size_t>(j + 1) * args.ldo, pack_bf16x2(other, oB));
                  } else {
                    if (j < jn) st_global_b32(ob + static_cast<size_t>(j) * args.ldo, pack_bf16x2(oA, other));
                  }
                  // both tokens two positions on
                  float nA, nB, mA, mB;
                  mul2(cA, cB, ct2, ct2, nA, nB);
                  fma2(sA, sB, -st2, -st2, nA, nB);
                  mul2(sA, sB, ct2, ct2, mA, mB);
                  fma2(cA, cB, st2, st2, mA, mB);
                  cA = nA;
                  cB = nB;
                  sA = mA;
                  sB = mB;
                }
              }
            } else {
              // positions wrap inside the chunk (short sequences, or one position per row): per-token
              // table entries, loaded 4 tokens at a time before use
#pragma unroll
              for (int hb = 0; hb < 32; hb += 4) {
                float cv[4], sv[4];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                  const int j = hb + jj < jn ? hb + jj : 0;
                  const int pos = args.sp.blk > 0 ? sp_pos(args.sp, tokc + j) : (tokc + j) % args.rope_seq;
                  const size_t e = static_cast<size_t>(pos + args.rope_pos_base) * hh + pj;
                  cv[jj] = __ldg(args.rope_cos + e);
                  sv[jj] = __ldg(args.rope_sin + e);
                }
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                  const int j = hb + jj;
                  const float x = __uint_as_float(acc[j]) * rsb[c0 + j] * cs;
                  const float y = __shfl_xor_sync(0xffffffffu, x, 1);
                  if (j < jn)
                    st_global_b16(ob + static_cast<size_t>(j) * args.ldo,
                                  odd ? x * cv[jj] + y * sv[jj] : x * cv[jj] - y * sv[jj]);
                }
              }
            }
          } else {
            // adjacent lanes swap one value per token pair and each stores two channels of one token
            const bool odd = (lane & 1) != 0;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float2 r2 = *reinterpret_cast<const float2*>(rsb + c0 + j);  // broadcast
              float xA, xB;
              mul2(__uint_as_float(acc[j]), __uint_as_float(acc[j + 1]), r2.x * cs, r2.y * cs, xA, xB);
              const float other = __shfl_xor_sync(0xffffffffu, odd ? xA : xB, 1);
              if (odd) {
                if (j + 1 < jn) st_global_b32(ob - 1 + static_cast<size_t>(j + 1) * args.ldo, pack_bf16x2(other, xB));
              } else {
                if (j < jn) st_global_b32(ob + static_cast<size_t>(j) * args.ldo, pack_bf16x2(xA, other));
              }
            }
          }
        } else {  // COLSCALE
          __nv_bfloat16* ob = args.out + static_cast<size_t>(tokc) * args.ldo + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < jn) st_global_b16(ob + static_cast<size_t>(j) * args.ldo, __uint_as_float(acc[j]) * cs);
        }
      }
      // accumulator drained: the MMAs of tile it + 2 may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(lead_bar(&tempty[a]));
        else
          mbar_arrive(&tempty[a]);
      }
      if (MODE == GEMM_RESID32 && args.rowsq) {
        // combine the four lane quarters' partial sums per token (fixed order) into the tile's statistic
        __syncwarp();
        if (lane == 0) mbar_arrive(&esync[a]);
        if (!mbar_wait(&esync[a], aph, abort_flag)) break;
        const float* s0 = ss_s + a * 4 * GT;
        for (int j = et; j < nt; j += G_EPI_WARPS * 32) {
          const int tok = tok0 + j;
          if (tok < args.M)
            args.rowsq[static_cast<size_t>(tok) * args.rowsq_ld + cb] =
                ((s0[j] + s0[GT + j]) + s0[2 * GT + j]) + s0[3 * GT + j];
        }
      }
    }
  } else {
    // -------------------------------------------------------------------- int8 -> bf16 converters (bf16: copy)
    // Thread = one weight row (output channel) of the tile, half of the stage's 128 K values.
    // Weight tiles arrive 128B-swizzled: 16-byte chunk c of row rr sits at rr*128 + ((c ^ (rr&7))<<4),
    // so the eight rows of each quarter-warp phase hit distinct banks.
    constexpr int CPT = (GK / 16) / (G_CONV_WARPS / 4);    // 16-byte chunks of the row per thread
    const int cq = warp & 3;                               // TMEM lane quarter
    const int kh = (warp - G_CONV_WARP0) >> 2;             // which part of the k-step
    const int rr = cq * 32 + lane;                         // weight row within the tile
    const uint32_t xsw = rr & 7;
    const uint32_t toff = static_cast<uint32_t>(cq * 32) << 16;
    for (int idx = 0; idx < total; ++idx) {
      const int sq = idx % QS, sw = idx % GW_SLOTS;
      if (!mbar_wait(&q_full[sq], (idx / QS) & 1, abort_flag)) break;
      uint32_t o[8 * CPT];
      if constexpr (WB) {
        // bf16 weights: this thread's half of the row is panel kh (64 K = eight 16-byte chunks), already
        // in the TMEM operand's format (two consecutive K per 32-bit word, lower K in the low half)
        static_assert(CPT == 4, "bf16 weights: one 64-K panel per converter thread");
        const uint8_t* rowp = sQ + sq * QB + kh * G_Q_BYTES + rr * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((c ^ xsw) << 4));
          o[4 * c] = v.x;
          o[4 * c + 1] = v.y;
          o[4 * c + 2] = v.z;
          o[4 * c + 3] = v.w;
        }
      } else {
        const uint8_t* rowp = sQ + sq * QB + rr * GK;
        uint4 v[CPT];
#pragma unroll
        for (int c = 0; c < CPT; ++c) v[c] = *reinterpret_cast<const uint4*>(rowp + (((kh * CPT + c) ^ xsw) << 4));
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          i8x4_to_bf16x4(v[c].x, o[8 * c + 0], o[8 * c + 1]);
          i8x4_to_bf16x4(v[c].y, o[8 * c + 2], o[8 * c + 3]);
          i8x4_to_bf16x4(v[c].z, o[8 * c + 4], o[8 * c + 5]);
          i8x4_to_bf16x4(v[c].w, o[8 * c + 6], o[8 * c + 7]);
        }
      }
      // Every lane has consumed its loaded bytes (the conversion used them), so the TMA may now
      // overwrite the slot.  Releasing it right after issuing the loads let a refill race them.
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[sq]);
      if (!mbar_wait(&w_empty[sw], ((idx / GW_SLOTS) & 1) ^ 1u, abort_flag)) break;
      tc_fence_after();
      const uint32_t ta = tmem_base + toff + G_W_COL0 + sw * G_W_COLS + kh * 8 * CPT;  // 8 columns per chunk
      if constexpr (CPT == 4)
        tmem_st_32x32b_x32(ta, *reinterpret_cast<const uint32_t(*)[32]>(o));
      else
        tmem_st_32x32b_x16(ta, *reinterpret_cast<const uint32_t(*)[16]>(o));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(lead_bar(&w_full[sw]));
        else
          mbar_arrive(&w_full[sw]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (PAIR) {
    // neither CTA frees its TMEM or leaves while the pair's MMAs may still read its operands
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, G_TMEM_COLS);
  } else {
    if (warp == 1) tmem_dealloc(tmem_base, G_TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && args.err) atomicCAS(args.err, 0, DEV_ERR_TIMEOUT_GEMM);
}

}  // namespace mk
