// C ABI of the minicpm5_mk B200 library: handle / weight binding / whole-model forward
// orchestration, plus the isolated per-stage entry points.  See include/minicpm5_mk.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <queue>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/minicpm5_mk.h"
#include "mk_attn.cuh"
#include "mk_attn_tc.cuh"
#include "mk_common.cuh"
#include "mk_gemm.cuh"
#include "mk_small.cuh"

namespace {

using mk::AttnLastArgs;
using mk::GemmArgs;

// Library device error word (one per device that loads the library); first error wins.
__device__ int g_mk_err;

constexpr int kMaxDevices = 64;
// Weight-operand TMA box rows (one int8 weight tile per k-step).
constexpr int kWeightBoxRows = mk::GW;
constexpr int kLmParts = 296;                // lm_head CTAs (2 per SM) = argmax partials per row
constexpr int kLmSmemMax = 100 * 1024;       // lm_head hidden rows in shared memory (2 CTAs per SM)

// lm_head launches for bs rows: up to lm_rows_max(H) rows per launch.
int lm_launches(int bs, int H) {
  const int nr = mk::lm_rows_max(H);
  return (bs + nr - 1) / nr;
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int pair_clusters[2] = {0, 0};  // co-resident 2-CTA clusters of the pair GEMM (int8, bf16 weights)
  int* err = nullptr;
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
PFN_encodeTiled g_encode = nullptr;

mk_status cuda_status(cudaError_t e) { return e == cudaSuccess ? MK_OK : MK_ERR_CUDA; }

#define MK_CUDA(x)                                   \
  do {                                               \
    cudaError_t e_ = (x);                            \
    if (e_ != cudaSuccess) return MK_ERR_CUDA;       \
  } while (0)
#define MK_TRY(x)                \
  do {                           \
    mk_status s_ = (x);          \
    if (s_ != MK_OK) return s_;  \
  } while (0)

// Per-device one-time set-up: SM count, error-word address, kernel attributes, driver entry point.
mk_status device_state(DeviceState** out) {
  int dev = 0;
  MK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return MK_ERR_BAD_ARG;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    MK_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    void* p = nullptr;
    MK_CUDA(cudaGetSymbolAddress(&p, g_mk_err));
    d.err = static_cast<int*>(p);
    for (auto fn : {mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE>, mk::gemm_w8a16_kernel<MK_GEMM_RESID>,
                    mk::gemm_w8a16_kernel<MK_GEMM_SWIGLU>, mk::gemm_w8a16_kernel<MK_GEMM_COLSCALE>,
                    mk::gemm_w8a16_kernel<MK_GEMM_RESID32>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(mk::gemm_smem_bytes(false))));
    for (auto fn : {mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE, true>, mk::gemm_w8a16_kernel<MK_GEMM_RESID, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_SWIGLU, true>, mk::gemm_w8a16_kernel<MK_GEMM_COLSCALE, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_RESID32, true>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(mk::gemm_smem_bytes(true))));
    for (auto fn : {mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE, false, true>, mk::gemm_w8a16_kernel<MK_GEMM_RESID, false, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_SWIGLU, false, true>, mk::gemm_w8a16_kernel<MK_GEMM_COLSCALE, false, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_RESID32, false, true>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(mk::gemm_smem_bytes(false))));
    for (auto fn : {mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE, true, true>, mk::gemm_w8a16_kernel<MK_GEMM_RESID, true, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_SWIGLU, true, true>, mk::gemm_w8a16_kernel<MK_GEMM_COLSCALE, true, true>,
                    mk::gemm_w8a16_kernel<MK_GEMM_RESID32, true, true>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(mk::gemm_smem_bytes(true))));
    // how many CTA pairs fit on the GPU at once (clusters must sit in one GPC, so an odd SM of a GPC
    // stays out): the persistent pair GEMM launches that many
    for (int wb = 0; wb < 2; ++wb) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (d.sm_count / 2));
      cfg.blockDim = dim3(mk::G_THREADS);
      cfg.dynamicSmemBytes = mk::gemm_smem_bytes(wb == 1);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      const cudaError_t e =
          wb ? cudaOccupancyMaxActiveClusters(&n, mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE, true, true>, &cfg)
             : cudaOccupancyMaxActiveClusters(&n, mk::gemm_w8a16_kernel<MK_GEMM_ROWSCALE, false, true>, &cfg);
      d.pair_clusters[wb] = e == cudaSuccess && n > 0 ? n : 0;
      if (e != cudaSuccess) (void)cudaGetLastError();
    }
    for (auto fn : {mk::attn_tc_kernel<96, false>, mk::attn_tc_kernel<128, false>, mk::attn_tc_kernel<96, true>,
                    mk::attn_tc_kernel<128, true>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(mk::TA_SMEM)));
    for (auto fn : {mk::lm_head_kernel<1>, mk::lm_head_kernel<2>, mk::lm_head_kernel<4>, mk::lm_head_kernel<8>})
      MK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kLmSmemMax));
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      MK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
      if (q != cudaDriverEntryPointSuccess || !fn) return MK_ERR_CUDA;
      g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
    }
    d.ready = true;
  }
  *out = &d;
  return MK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch `k` on `st`; with `pdl` the launch carries programmatic stream serialization, so the kernel may
// begin while the previous kernel of the stream drains (every kernel of the forward calls pdl_wait()
// before touching memory an earlier kernel uses).
template <typename... KArgs, typename... Args>
mk_status launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...) == cudaSuccess ? MK_OK : MK_ERR_CUDA;
}
// The same with clusters of two CTAs along x (grid.x even).
template <typename... KArgs, typename... Args>
mk_status launch_k_pair(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                        Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...) == cudaSuccess ? MK_OK : MK_ERR_CUDA;
}

// Tokens per GEMM tile for M tokens and N output channels on `sms` SMs.  The persistent GEMM runs
// ceil(tiles / sms) waves of tiles; a tile of nt tokens costs about nt + 32 token-steps (the weight tile's
// conversion and the epilogue's fixed work).  At large M every size fills its waves and the largest tile
// wins (ties go to the larger tile); when all tiles fit in one or two waves (the projections of one
// sequence-parallel rank, an isolated N = 1792 GEMM at M = 8192) smaller tiles finish sooner: at 8 ranks
// (1024 rows) o_proj and down take 96-token tiles.  Candidates are multiples of 32 from 192 down to 64: the
// epilogue works in 32-token chunks, and with 32-aligned tiles no chunk straddles a sequence or zig-zag
// block boundary, and every position's RoPE angle comes from the same table entry and the same number
// of angle-addition steps whatever the batch size -- which keeps the forward batch-invariant bit for bit.
int choose_nt(int M, int N, int sms) {
  if (M < mk::GT) return mk::gemm_nt(M);
  const int nc = N / mk::GW;
  int best = mk::GT;
  long best_cost = -1;
  for (int nt = mk::GT; nt >= 64; nt -= 32) {
    const long tiles = static_cast<long>((M + nt - 1) / nt) * nc;
    const long cost = ((tiles + sms - 1) / sms) * (nt + 32);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = nt;
    }
  }
  return best;
}

// A GEMM of M tokens and N output channels runs on CTA pairs (2-SM UMMAs over 256 channels) when N is a
// multiple of 256 and M is more than a few rows.  The choice depends on N only once M > 64, so every
// forward shape of one projection (any batch, sequence-parallel rank rows) takes the same path.
bool pair_gemm(int M, int N) { return N % (2 * mk::GW) == 0 && M > 64; }
// Tokens per tile: choose_nt, but a multiple of 32 for pairs (2-SM UMMA N) also below GT tokens.
int plan_nt(int M, int N, int sms) {
  if (pair_gemm(M, N) && M < mk::GT) return ((M + 31) / 32) * 32;
  return choose_nt(M, N, sms);
}
// Rows of the token tensor map's box: a pair CTA loads half of the tile.
int a_box(int M, int N, int nt) { return pair_gemm(M, N) ? nt / 2 : nt; }

// Token operand: bf16 [rows, ld], box 64 (K) x nt rows (tokens per tile, or half of them for a CTA pair),
// 128-byte swizzle.
mk_status map_a(CUtensorMap* m, const void* a, int rows, int K, int ld, int nt = 0) {
  if (nt <= 0) nt = mk::gemm_nt(rows);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(mk::GKB), static_cast<cuuint32_t>(nt)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MK_OK : MK_ERR_CUDA;
}

// Weight operand [N, K] (K contiguous), 128-byte swizzle (the converters read one row per thread; the
// swizzle spreads a quarter-warp's rows over all banks).  int8: box 128 (K) x box_rows; bf16
// (wbf16): box 64 (K) x box_rows, two boxes per 128-K stage.
mk_status map_b(CUtensorMap* m, const void* w, int N, int K, int box_rows = mk::GW, bool wbf16 = false) {
  const int es_bytes = wbf16 ? 2 : 1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * es_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(wbf16 ? mk::GKB : mk::GK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, wbf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                        const_cast<void*>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MK_OK : MK_ERR_CUDA;
}

// Optional fused epilogue work of one GEMM launch (RMSNorm statistics, RoPE).
struct GemmFusion {
  float* rowsq = nullptr;  // per-(token, 128-channel tile) sums of squares of the f32 residual
  int rowsq_ld = 0, rowsq_np = 0;
  float inv_norm_dim = 0.f, eps = 0.f;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_cols = 0, head_dim = 0, rope_seq = 1, rope_pos_base = 0;
  mk::SpLayout sp;  // sequence-parallel rows (RoPE positions)
  bool pdl = false;  // launch with programmatic stream serialization (inside the forward)
  int nt = 0;        // tokens per tile, the token tensor map's box height (0: gemm_nt(M))
  bool wbf16 = false;  // bf16 weights (the weight tensor map is bf16) instead of int8
};

mk_status launch_gemm(const DeviceState* d, const CUtensorMap& ma, const CUtensorMap& mb, int M, int N, int K,
                      int mode, const float* row_scale, const float* col_scale, void* out, int ldo, float resid,
                      cudaStream_t st, float* resid32 = nullptr, int ld_resid32 = 0,
                      const GemmFusion& fu = GemmFusion()) {
  GemmArgs ga;
  ga.M = M;
  ga.N = N;
  ga.K = K;
  ga.nt = fu.nt > 0 ? fu.nt : plan_nt(M, N, d->sm_count);
  ga.mode = mode;
  ga.row_scale = row_scale;
  ga.col_scale = col_scale;
  ga.out = static_cast<__nv_bfloat16*>(out);
  ga.ldo = ldo;
  ga.resid_scale = resid;
  ga.resid32 = resid32;
  ga.ld_resid32 = ld_resid32;
  ga.rowsq = fu.rowsq;
  ga.rowsq_ld = fu.rowsq_ld;
  ga.rowsq_np = fu.rowsq_np;
  ga.inv_norm_dim = fu.inv_norm_dim;
  ga.eps = fu.eps;
  ga.rope_cos = fu.rope_cos;
  ga.rope_sin = fu.rope_sin;
  ga.rope_cols = fu.rope_cols;
  ga.head_dim = fu.head_dim > 0 ? fu.head_dim : 1;
  ga.rope_seq = fu.rope_seq > 0 ? fu.rope_seq : 1;
  ga.rope_pos_base = fu.rope_pos_base;
  ga.sp = fu.sp;
  ga.err = d->err;
  const bool pair = pair_gemm(M, N) && d->pair_clusters[fu.wbf16 ? 1 : 0] > 0;
  if (pair_gemm(M, N) && !pair) return MK_ERR_CUDA;  // the token map was built for pairs
  if (pair && ga.nt % 32) return MK_ERR_BAD_SHAPE;
  const int tiles = ((M + ga.nt - 1) / ga.nt) * (N / mk::GW);
  const int grid = pair ? 2 * std::max(1, std::min(tiles / 2, d->pair_clusters[fu.wbf16 ? 1 : 0]))
                        : std::max(1, std::min(tiles, d->sm_count));
  const dim3 g(grid), b(mk::G_THREADS);
  const bool pdl = fu.pdl;
  const size_t smem = mk::gemm_smem_bytes(fu.wbf16);
#define MK_GEMM_CASE(MODE)                                                                                      \
  case MODE:                                                                                                    \
    if (pair)                                                                                                   \
      return fu.wbf16 ? launch_k_pair(mk::gemm_w8a16_kernel<MODE, true, true>, g, b, smem, st, pdl, ma, mb, ga) \
                      : launch_k_pair(mk::gemm_w8a16_kernel<MODE, false, true>, g, b, smem, st, pdl, ma, mb, ga); \
    return fu.wbf16 ? launch_k(mk::gemm_w8a16_kernel<MODE, true>, g, b, smem, st, pdl, ma, mb, ga)              \
                    : launch_k(mk::gemm_w8a16_kernel<MODE, false>, g, b, smem, st, pdl, ma, mb, ga);
  switch (mode) {
    MK_GEMM_CASE(MK_GEMM_ROWSCALE)
    MK_GEMM_CASE(MK_GEMM_RESID)
    MK_GEMM_CASE(MK_GEMM_SWIGLU)
    MK_GEMM_CASE(MK_GEMM_COLSCALE)
    MK_GEMM_CASE(MK_GEMM_RESID32)
    default:
      return MK_ERR_BAD_ARG;
  }
#undef MK_GEMM_CASE
}

mk_status check_gemm_shape(int M, int N, int K, int mode) {
  if (M <= 0 || N <= 0 || K <= 0) return MK_ERR_BAD_SHAPE;
  if (N % 128 || K % mk::GKB) return MK_ERR_BAD_SHAPE;
  if (mode == MK_GEMM_SWIGLU && N % 2) return MK_ERR_BAD_SHAPE;  // alternating gate / up rows
  if (mode < 0 || mode > 4) return MK_ERR_BAD_ARG;
  return MK_OK;
}

// bf16 [T, ld] viewed as [T, heads, hd] (3D), box 64 x box_heads x box_rows, 128-byte swizzle.
mk_status map_heads(CUtensorMap* m, const void* base, int T, int heads, int hd, int ld, int box_heads,
                    int box_rows) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(hd) * 2, static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_heads), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MK_OK : MK_ERR_CUDA;
}

int ilog2(int v) {
  int r = 0;
  while ((1 << r) < v) ++r;
  return r;
}

// tcgen05 causal GQA attention (mk_attn_tc.cuh).  Queries (rows per sequence `rows`) and keys /
// values (S per sequence) may live in different buffers; under sequence parallelism the queries are
// a rank's zig-zag rows and K/V the rank-by-rank all-gather (`sp`).
// kchunk > 0 (one sequence) cuts query blocks with more key tiles into ranges of at most kchunk tiles,
// one CTA each; their partial results go to `part` and attn_split_combine_kernel merges them.
mk_status launch_attn_split(const DeviceState* d, const void* q_base, int rows, int ld_q, int q_col, const void* kv_base,
                            int S, int ld_kv, int k_col, int v_col, int bs, int n_q, int n_kv, int hd, float scale_log2,
                            void* out, int ld_out, cudaStream_t st, const mk::SpLayout& sp = mk::SpLayout(),
                            bool pdl = false, int kchunk = 0, float* part = nullptr) {
  const int G = n_q / n_kv;
  const int qpt = 128 / G;
  if (rows % (2 * qpt) || S % mk::TA_BK) return MK_ERR_BAD_SHAPE;
  if (sp.blk > 0 && (bs != 1 || sp.blk % (2 * qpt) || sp.blk % mk::TA_BK)) return MK_ERR_BAD_SHAPE;
  const auto* qb = static_cast<const __nv_bfloat16*>(q_base);
  const auto* kvb = static_cast<const __nv_bfloat16*>(kv_base);
  CUtensorMap mq, mkm, mv;
  MK_TRY(map_heads(&mq, qb + q_col, bs * rows, n_q, hd, ld_q, G, qpt));
  MK_TRY(map_heads(&mkm, kvb + k_col, bs * S, n_kv, hd, ld_kv, 1, mk::TA_BK));
  MK_TRY(map_heads(&mv, kvb + v_col, bs * S, n_kv, hd, ld_kv, 1, mk::TA_BK));
  mk::AttnTcArgs a;
  a.S = S;
  a.rows = rows;
  a.sp = sp;
  a.lg2G = ilog2(G);
  a.nqb = rows / (2 * qpt);
  a.ld_out = ld_out;
  a.scale_log2 = scale_log2;
  a.kchunk = kchunk;
  a.n_q = n_q;
  a.part = part;
  a.err = d->err;
  if (kchunk > 0 && (bs != 1 || !part)) return MK_ERR_BAD_ARG;
  auto* o = static_cast<__nv_bfloat16*>(out);
  const dim3 blk(mk::TA_THREADS);
  if (kchunk == 0) {
    const dim3 grid(a.nqb, n_kv, bs);
    if (hd == 96) return launch_k(mk::attn_tc_kernel<96, false>, grid, blk, mk::TA_SMEM, st, pdl, mq, mkm, mv, o, a);
    return launch_k(mk::attn_tc_kernel<128, false>, grid, blk, mk::TA_SMEM, st, pdl, mq, mkm, mv, o, a);
  }
  // with a key split the grid is (key range, query block, KV head), as many ranges as any block needs
  const dim3 grid(mk::ta_nsplit(S / mk::TA_BK, kchunk), a.nqb, n_kv), cgrid(a.nqb, n_kv, hd / 8);
  if (hd == 96) {
    MK_TRY(launch_k(mk::attn_tc_kernel<96, true>, grid, blk, mk::TA_SMEM, st, pdl, mq, mkm, mv, o, a));
    return launch_k(mk::attn_split_combine_kernel<96>, cgrid, dim3(256), 0, st, pdl, o, a);
  }
  MK_TRY(launch_k(mk::attn_tc_kernel<128, true>, grid, blk, mk::TA_SMEM, st, pdl, mq, mkm, mv, o, a));
  return launch_k(mk::attn_split_combine_kernel<128>, cgrid, dim3(256), 0, st, pdl, o, a);
}

// Key tiles per attention CTA under sequence parallelism (0 = no split).  A rank holds few query blocks
// and their causal key ranges are very unequal: at 4 and 8 ranks the longest CTA walks all 128 key tiles
// of an 8192-token sequence while the rank's whole attention is 56 or 28 tiles per SM.  The choice
// replays the grid's dispatch order (key ranges of a block together, heaviest blocks first, KV heads
// outermost) on `sms` SMs: each CTA takes its start-up and drain (about 4.5 us, measured) plus 0.9 us per
// key tile, an empty one 0.3 us, and goes to the SM that frees first; a split also pays the merge kernel
// (about 5 us).  The smallest simulated time wins, and a split must gain 3 % to be used.  Planned on
// rank 0's layout, so every rank sizes the same workspace.
int sp_key_chunk(const mk_config& c, const mk::SpLayout& sp, int S, int sms) {
  if (sp.world <= 1 || sms <= 0) return 0;
  const int G = c.n_q / c.n_kv, qpt = 128 / G;
  const int nqb = sp.rows_per_rank / (2 * qpt);
  std::vector<int> ntot(nqb);
  for (int y = 0; y < nqb; ++y) {  // dispatch order: heaviest (last local) block first
    const int qb = nqb - 1 - y;
    ntot[y] = (mk::sp_pos(sp, qb * 2 * qpt) + 2 * qpt - 1) / mk::TA_BK + 1;
  }
  auto makespan = [&](int kchunk) {
    std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
    for (int i = 0; i < sms; ++i) free_at.push(0.0);
    auto run = [&](double cost) {
      const double t = free_at.top();
      free_at.pop();
      free_at.push(t + cost);
    };
    const int zmax = kchunk > 0 ? mk::ta_nsplit(S / mk::TA_BK, kchunk) : 1;
    for (int g = 0; g < c.n_kv; ++g)
      for (int y = 0; y < nqb; ++y) {
        const int ns = mk::ta_nsplit(ntot[y], kchunk), per = mk::ta_split_per(ntot[y], ns);
        for (int z = 0; z < zmax; ++z) run(z >= ns ? 0.3 : 4.5 + 0.9 * (std::min(ntot[y], z * per + per) - z * per));
      }
    double m = 0.0;
    while (!free_at.empty()) {
      m = std::max(m, free_at.top());
      free_at.pop();
    }
    return m + (kchunk > 0 ? 5.0 : 0.0);
  };
  double best = makespan(0) * 0.97;
  int best_k = 0;
  for (int k : {8, 12, 16, 20, 24, 28, 32, 36, 40, 44, 48, 56, 64, 72, 80, 96, 112}) {
    if (k >= S / mk::TA_BK) break;
    const double m = makespan(k);
    if (m < best) {
      best = m;
      best_k = k;
    }
  }
  return best_k;
}

mk_status launch_attn(const DeviceState* d, const void* qkv, int bs, int S, int n_q, int n_kv, int hd, int ld_qkv,
                      int q_col, int k_col, int v_col, float scale_log2, void* out, int ld_out, cudaStream_t st,
                      bool pdl = false) {
  return launch_attn_split(d, qkv, S, ld_qkv, q_col, qkv, S, ld_qkv, k_col, v_col, bs, n_q, n_kv, hd, scale_log2, out,
                           ld_out, st, mk::SpLayout(), pdl);
}

mk_status check_attn_shape(int bs, int S, int n_q, int n_kv, int hd, int ld_qkv, int q_col, int k_col, int v_col,
                           int ld_out) {
  if (bs <= 0 || S <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv) return MK_ERR_BAD_SHAPE;
  const int G = n_q / n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return MK_ERR_BAD_SHAPE;
  if (hd != 96 && hd != 128) return MK_ERR_BAD_SHAPE;
  if (S % 128) return MK_ERR_BAD_SHAPE;
  if (ld_qkv % 8 || q_col % 8 || k_col % 8 || v_col % 8 || ld_out % 8) return MK_ERR_BAD_ALIGN;
  if (S % (256 / G)) return MK_ERR_BAD_SHAPE;  // two 128-row (query x head) tiles per CTA
  return MK_OK;
}

constexpr float kLog2e = 1.4426950408889634f;

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

struct mk_handle {
  mk_config cfg;
  int device = 0;
  DeviceState* dev = nullptr;
  bool bound = false;
  mk_weight_ptrs w;
  int n_qkv = 0, q_dim = 0, kv_dim = 0;
  bool wbf16 = false;  // bf16 projection weights (weight_bits 16) instead of int8
  bool sp_key_split = true;  // mk_forward_sp cuts long causal key ranges over several attention CTAs
  mutable std::vector<std::array<int, 3>> sp_chunk_cache;  // (seq, world, key tiles per CTA) already planned
  std::vector<CUtensorMap> m_qkv, m_o, m_gu, m_down;  // per layer
  CUtensorMap m_kv_last, m_q_last;
};

extern "C" {

const char* mk_status_string(mk_status s) {
  switch (s) {
    case MK_OK: return "ok";
    case MK_ERR_BAD_SHAPE: return "unsupported shape";
    case MK_ERR_BAD_ALIGN: return "misaligned pointer or stride";
    case MK_ERR_CUDA: return "CUDA error";
    case MK_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case MK_ERR_BAD_ARG: return "bad argument";
    case MK_ERR_NOT_BOUND: return "weights not bound";
    case MK_ERR_BAD_TOKEN: return "token id out of range";
    case MK_ERR_WORKSPACE: return "workspace too small";
    case MK_ERR_TOO_LARGE: return "request exceeds a fixed library capacity";
  }
  return "unknown status";
}

int32_t mk_version(void) { return 100; }

mk_status mk_create(const mk_config* cfg, int32_t device, mk_handle** out) {
  if (!cfg || !out) return MK_ERR_BAD_ARG;
  const mk_config& c = *cfg;
  if (c.num_layers < 1 || c.hidden <= 0 || c.inter <= 0 || c.n_q <= 0 || c.n_kv <= 0 || c.vocab <= 0 ||
      c.max_seq <= 0)
    return MK_ERR_BAD_SHAPE;
  if (c.head_dim != 96 && c.head_dim != 128) return MK_ERR_BAD_SHAPE;
  if (c.n_q % c.n_kv) return MK_ERR_BAD_SHAPE;
  const int G = c.n_q / c.n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return MK_ERR_BAD_SHAPE;
  const int n_qkv = (c.n_q + 2 * c.n_kv) * c.head_dim;
  if (c.hidden % 128 || c.inter % 128 || (c.n_q * c.head_dim) % 128 || n_qkv % 128 ||
      (2 * c.n_kv * c.head_dim) % 128)
    return MK_ERR_BAD_SHAPE;
  if (c.max_seq > 16384) return MK_ERR_BAD_SHAPE;
  if (c.weight_bits != 0 && c.weight_bits != 8 && c.weight_bits != 16) return MK_ERR_BAD_ARG;
  MK_CUDA(cudaSetDevice(device));
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  mk_handle* h = new mk_handle();
  h->cfg = c;
  h->device = device;
  h->dev = d;
  h->n_qkv = n_qkv;
  h->wbf16 = c.weight_bits == 16;
  h->q_dim = c.n_q * c.head_dim;
  h->kv_dim = c.n_kv * c.head_dim;
  *out = h;
  return MK_OK;
}

mk_status mk_bind_weights(mk_handle* h, const mk_weight_ptrs* w) {
  if (!h || !w) return MK_ERR_BAD_ARG;
  const void* ptrs[] = {w->embed, w->lm_head, w->final_norm, w->rope_cos, w->rope_sin, w->w_qkv, w->s_qkv,
                        w->w_o,   w->s_o,     w->w_gu,       w->s_gu,     w->w_down,   w->s_down};
  for (const void* p : ptrs) {
    if (!p) return MK_ERR_BAD_ARG;
    if (!aligned16(p)) return MK_ERR_BAD_ALIGN;
  }
  MK_CUDA(cudaSetDevice(h->device));
  const mk_config& c = h->cfg;
  const int L = c.num_layers, H = c.hidden, I = c.inter;
  h->m_qkv.resize(L);
  h->m_o.resize(L);
  h->m_gu.resize(L);
  h->m_down.resize(L);
  const bool wb = h->wbf16;
  const size_t es = wb ? 2 : 1;  // bytes per weight
  auto at = [es](const void* base, size_t elems) { return static_cast<const uint8_t*>(base) + elems * es; };
  for (int l = 0; l < L; ++l) {
    MK_TRY(map_b(&h->m_qkv[l], at(w->w_qkv, static_cast<size_t>(l) * h->n_qkv * H), h->n_qkv, H, kWeightBoxRows, wb));
    MK_TRY(map_b(&h->m_o[l], at(w->w_o, static_cast<size_t>(l) * H * h->q_dim), H, h->q_dim, kWeightBoxRows, wb));
    MK_TRY(map_b(&h->m_gu[l], at(w->w_gu, static_cast<size_t>(l) * 2 * I * H), 2 * I, H, kWeightBoxRows, wb));
    MK_TRY(map_b(&h->m_down[l], at(w->w_down, static_cast<size_t>(l) * H * I), H, I, kWeightBoxRows, wb));
  }
  const uint8_t* wl = at(w->w_qkv, static_cast<size_t>(L - 1) * h->n_qkv * H);
  MK_TRY(map_b(&h->m_q_last, wl, h->q_dim, H, kWeightBoxRows, wb));
  MK_TRY(map_b(&h->m_kv_last, wl + static_cast<size_t>(h->q_dim) * H * es, 2 * h->kv_dim, H, kWeightBoxRows, wb));
  h->w = *w;
  h->bound = true;
  return MK_OK;
}

namespace {
struct Workspace {
  size_t x32, xb, qkv, attn, hbuf, rowsq, xl32, xlb, ql, al, alpart, hl, rowsql, hf, logits, pval, pidx, top1, total;
};

Workspace plan_workspace(const mk_handle* h, int bs, int seq) {
  const mk_config& c = h->cfg;
  const size_t T = static_cast<size_t>(bs) * seq;
  Workspace w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  w.x32 = take(T * c.hidden * 4);
  w.xb = take(T * c.hidden * 2);
  w.qkv = take(T * h->n_qkv * 2);
  w.attn = take(T * h->q_dim * 2);
  w.hbuf = take(T * c.inter * 2);
  w.rowsq = take(T * (c.hidden / 128) * 4);
  w.xl32 = take(static_cast<size_t>(bs) * c.hidden * 4);
  w.xlb = take(static_cast<size_t>(bs) * c.hidden * 2);
  w.ql = take(static_cast<size_t>(bs) * h->q_dim * 2);
  w.al = take(static_cast<size_t>(bs) * h->q_dim * 2);
  w.alpart = take(static_cast<size_t>(bs) * c.n_q * ((seq + mk::AL_KEYS - 1) / mk::AL_KEYS) * (c.head_dim + 2) * 4);
  w.hl = take(static_cast<size_t>(bs) * c.inter * 2);
  w.rowsql = take(static_cast<size_t>(bs) * (c.hidden / 128) * 4);
  w.hf = take(static_cast<size_t>(bs) * c.hidden * 4);
  w.logits = take(static_cast<size_t>(bs) * c.vocab * 4);
  w.pval = take(static_cast<size_t>(bs) * kLmParts * 4);
  w.pidx = take(static_cast<size_t>(bs) * kLmParts * 4);
  w.top1 = take(static_cast<size_t>(bs) * 4);
  w.total = off;
  return w;
}

mk_status lm_head_launch(const DeviceState*, const float* hf, int bs, int H, const void* lm, int V, float* logits,
                         float* pval, int* pidx, int32_t* top1, cudaStream_t st, bool pdl = false) {
  const int nr_max = mk::lm_rows_max(H);
  if (static_cast<size_t>(nr_max) * H * 4 > static_cast<size_t>(kLmSmemMax)) return MK_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(V) * H >= (int64_t{1} << 31)) return MK_ERR_BAD_SHAPE;  // 32-bit row offsets
  const auto* W = static_cast<const __nv_bfloat16*>(lm);
  for (int r0 = 0; r0 < bs; r0 += nr_max) {
    const int left = std::min(nr_max, bs - r0);
    const int nr = left <= 1 ? 1 : left <= 2 ? 2 : left <= 4 ? 4 : 8;  // rows this launch holds
    const size_t smem = static_cast<size_t>(nr) * H * 4;
    auto k = nr == 1 ? mk::lm_head_kernel<1> : nr == 2 ? mk::lm_head_kernel<2> : nr == 4 ? mk::lm_head_kernel<4>
                                                                                  : mk::lm_head_kernel<8>;
    MK_TRY(launch_k(k, dim3(kLmParts), dim3(mk::LM_THREADS), smem, st, pdl, hf, W, logits, pval, pidx, bs, H, V, r0));
  }
  return launch_k(mk::argmax_reduce_kernel, dim3(bs), dim3(32), 0, st, pdl, static_cast<const float*>(pval),
                  static_cast<const int*>(pidx), static_cast<int>(kLmParts), top1);
}
}  // namespace

mk_status mk_workspace_size(const mk_handle* h, int32_t bs, int32_t seq, size_t* bytes) {
  if (!h || !bytes) return MK_ERR_BAD_ARG;
  if (bs <= 0 || seq <= 0) return MK_ERR_BAD_SHAPE;
  *bytes = plan_workspace(h, bs, seq).total;
  return MK_OK;
}

}  // extern "C"

namespace {
// Per-stage timing of one forward: an event before the first launch and one after each stage's
// launches, all on the forward's stream.  A null clock records nothing.
class StageClock {
 public:
  ~StageClock() {
    for (cudaEvent_t e : ev_) cudaEventDestroy(e);
  }
  mk_status start(cudaStream_t st) {
    st_ = st;
    return record();
  }
  mk_status mark(int stage, int launches) {
    stage_.push_back(stage);
    launches_.push_back(launches);
    return record();
  }
  mk_status finish(mk_stage_times* out) {
    std::memset(out, 0, sizeof(*out));
    if (ev_.empty()) return MK_OK;
    MK_CUDA(cudaEventSynchronize(ev_.back()));
    for (size_t i = 0; i < stage_.size(); ++i) {
      float ms = 0.f;
      MK_CUDA(cudaEventElapsedTime(&ms, ev_[i], ev_[i + 1]));
      out->ms[stage_[i]] += ms;
      out->launches[stage_[i]] += launches_[i];
    }
    return MK_OK;
  }

 private:
  mk_status record() {
    cudaEvent_t e;
    MK_CUDA(cudaEventCreate(&e));
    ev_.push_back(e);
    MK_CUDA(cudaEventRecord(e, st_));
    return MK_OK;
  }
  cudaStream_t st_ = nullptr;
  std::vector<cudaEvent_t> ev_;
  std::vector<int> stage_, launches_;
};

mk_status forward_impl(mk_handle* h, const int32_t* d_ids, int32_t bs, int32_t seq, void* d_workspace,
                       size_t workspace_bytes, void* d_hidden, float* d_logits, int32_t* d_top1, void* stream,
                       StageClock* clk) {
  if (!h || !d_ids || !d_workspace) return MK_ERR_BAD_ARG;
  if (!h->bound) return MK_ERR_NOT_BOUND;
  const mk_config& c = h->cfg;
  if (bs <= 0 || seq <= 0 || seq % 128 || seq > c.max_seq) return MK_ERR_BAD_SHAPE;
  if ((reinterpret_cast<uintptr_t>(d_workspace) & 255u) || !aligned16(d_ids)) return MK_ERR_BAD_ALIGN;
  if ((d_hidden && !aligned16(d_hidden)) || (d_logits && !aligned16(d_logits))) return MK_ERR_BAD_ALIGN;
  const Workspace ws = plan_workspace(h, bs, seq);
  if (workspace_bytes < ws.total) return MK_ERR_WORKSPACE;
  MK_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DeviceState* d = h->dev;
  uint8_t* base = static_cast<uint8_t*>(d_workspace);
  auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(base + off); };
  auto f32 = [&](size_t off) { return reinterpret_cast<float*>(base + off); };

  const int L = c.num_layers, H = c.hidden, I = c.inter, hd = c.head_dim;
  const int T = bs * seq;
  const int nqkv = h->n_qkv, qd = h->q_dim, kvd = h->kv_dim;
  // f32 residual stream (x32 / xl32) with bf16 copies (xb / xlb) feeding the projections
  float *x32 = f32(ws.x32), *xl32 = f32(ws.xl32);
  __nv_bfloat16 *xb = bf(ws.xb), *qkv = bf(ws.qkv), *attn = bf(ws.attn), *hb = bf(ws.hbuf);
  __nv_bfloat16 *xlb = bf(ws.xlb), *ql = bf(ws.ql), *al = bf(ws.al), *hl = bf(ws.hl);
  float *rowsq = f32(ws.rowsq), *rowsql = f32(ws.rowsql), *hf = f32(ws.hf);
  float* logits = d_logits ? d_logits : f32(ws.logits);
  int32_t* top1 = d_top1 ? d_top1 : reinterpret_cast<int32_t*>(base + ws.top1);
  const float r = c.residual_scale;

  // token tiles sized per projection (choose_nt); one token tensor map per (buffer, tile size)
  const int sms = d->sm_count;
  const int nt_qkv = plan_nt(T, nqkv, sms), nt_o = plan_nt(T, H, sms), nt_gu = plan_nt(T, 2 * I, sms);
  const int nt_down = nt_o, nt_kv = plan_nt(T, 2 * kvd, sms);
  CUtensorMap mx_qkv, mx_gu, mx_kv, mattn, mh, mxl, mxl_gu, mal, mhl;
  MK_TRY(map_a(&mx_qkv, xb, T, H, H, a_box(T, nqkv, nt_qkv)));
  MK_TRY(map_a(&mx_gu, xb, T, H, H, a_box(T, 2 * I, nt_gu)));
  MK_TRY(map_a(&mx_kv, xb, T, H, H, a_box(T, 2 * kvd, nt_kv)));
  MK_TRY(map_a(&mattn, attn, T, qd, qd, a_box(T, H, nt_o)));
  MK_TRY(map_a(&mh, hb, T, I, I, a_box(T, H, nt_down)));
  // the last rows' projections (bs rows); each map's box follows its GEMM's plan
  MK_TRY(map_a(&mxl, xlb, bs, H, H, a_box(bs, qd, plan_nt(bs, qd, sms))));
  MK_TRY(map_a(&mxl_gu, xlb, bs, H, H, a_box(bs, 2 * I, plan_nt(bs, 2 * I, sms))));
  MK_TRY(map_a(&mal, al, bs, qd, qd, a_box(bs, H, plan_nt(bs, H, sms))));
  MK_TRY(map_a(&mhl, hl, bs, I, I, a_box(bs, H, plan_nt(bs, H, sms))));
  auto tiles = [](GemmFusion f, int nt) {
    f.nt = nt;
    return f;
  };

  const int rows_per_blk = 8;  // warps per 256-thread block, one row each
  const int np = H / 128;       // 128-column tiles of the residual: RMSNorm partial sums per row
  auto mark = [&](int stage, int launches) { return clk ? clk->mark(stage, launches) : MK_OK; };
  if (clk) MK_TRY(clk->start(st));
  mk::embed_kernel<<<(T + rows_per_blk - 1) / rows_per_blk, 256, 0, st>>>(
      d_ids, static_cast<const __nv_bfloat16*>(h->w.embed), x32, xb, T, H, c.vocab, c.scale_emb, d->err, rowsq, np);
  MK_CUDA(cudaGetLastError());
  MK_TRY(mark(MK_STAGE_EMBED, 1));

  // RMSNorm folded into the projections: rstd comes from the residual's per-tile sums of squares
  // (written by the embedding and by every residual-update epilogue).
  auto norm_from = [&](float* sq) {
    GemmFusion f;
    f.rowsq = sq;
    f.rowsq_ld = np;
    f.rowsq_np = np;
    f.inv_norm_dim = 1.0f / static_cast<float>(H);
    f.eps = c.eps;
    f.pdl = true;
    f.wbf16 = h->wbf16;
    return f;
  };
  auto with_rope = [&](GemmFusion f, int cols, int sq, int pos_base) {
    f.rope_cos = h->w.rope_cos;
    f.rope_sin = h->w.rope_sin;
    f.rope_cols = cols;
    f.head_dim = hd;
    f.rope_seq = sq;
    f.rope_pos_base = pos_base;
    return f;
  };
  GemmFusion resid_stats;  // residual epilogues write the statistics
  resid_stats.rowsq = rowsq;
  resid_stats.pdl = true;
  resid_stats.wbf16 = h->wbf16;
  resid_stats.rowsq_ld = np;
  GemmFusion resid_stats_last = resid_stats;
  resid_stats_last.rowsq = rowsql;

  for (int l = 0; l < L - 1; ++l) {
    // QKV projection with RMSNorm and RoPE (Q/K) fused into the epilogue
    MK_TRY(launch_gemm(d, mx_qkv, h->m_qkv[l], T, nqkv, H, MK_GEMM_ROWSCALE, nullptr,
                       h->w.s_qkv + static_cast<size_t>(l) * nqkv, qkv, nqkv, 0.f, st, nullptr, 0,
                       tiles(with_rope(norm_from(rowsq), qd + kvd, seq, 0), nt_qkv)));
    MK_TRY(mark(MK_STAGE_QKV, 1));
    MK_TRY(launch_attn(d, qkv, bs, seq, c.n_q, c.n_kv, hd, nqkv, 0, qd, qd + kvd, kLog2e, attn, qd, st, true));
    MK_TRY(mark(MK_STAGE_ATTN, 1));
    MK_TRY(launch_gemm(d, mattn, h->m_o[l], T, H, qd, mk::GEMM_RESID32, nullptr,
                       h->w.s_o + static_cast<size_t>(l) * H, xb, H, r, st, x32, H, tiles(resid_stats, nt_o)));
    MK_TRY(mark(MK_STAGE_O, 1));
    MK_TRY(launch_gemm(d, mx_gu, h->m_gu[l], T, 2 * I, H, MK_GEMM_SWIGLU, nullptr,
                       h->w.s_gu + static_cast<size_t>(l) * 2 * I, hb, I, 0.f, st, nullptr, 0,
                       tiles(norm_from(rowsq), nt_gu)));
    MK_TRY(mark(MK_STAGE_GATE_UP, 1));
    MK_TRY(launch_gemm(d, mh, h->m_down[l], T, H, I, mk::GEMM_RESID32, nullptr,
                       h->w.s_down + static_cast<size_t>(l) * H, xb, H, r, st, x32, H, tiles(resid_stats, nt_down)));
    MK_TRY(mark(MK_STAGE_DOWN, 1));
  }

  // Last layer: K/V for every position, everything else for the last position only
  // (`last_layer_step`, plugin/minicpm5_mk/mk_jax.py:492-520).
  {
    const int l = L - 1;
    const float* sq = h->w.s_qkv + static_cast<size_t>(l) * nqkv;
    __nv_bfloat16* kv = qkv;  // [T, 2 kv_dim]
    MK_TRY(launch_gemm(d, mx_kv, h->m_kv_last, T, 2 * kvd, H, MK_GEMM_ROWSCALE, nullptr, sq + qd, kv, 2 * kvd, 0.f, st,
                       nullptr, 0, tiles(with_rope(norm_from(rowsq), kvd, seq, 0), nt_kv)));
    MK_TRY(launch_k(mk::gather_last_kernel, dim3(bs), dim3(256), 0, st, true, x32, xl32, xlb, bs, seq, H, rowsq, rowsql,
                    np));
    MK_TRY(launch_gemm(d, mxl, h->m_q_last, bs, qd, H, MK_GEMM_ROWSCALE, nullptr, sq, ql, qd, 0.f, st, nullptr, 0,
                       with_rope(norm_from(rowsql), qd, 1, seq - 1)));
    AttnLastArgs la;
    la.S = seq;
    la.n_q = c.n_q;
    la.n_kv = c.n_kv;
    la.head_dim = hd;
    la.ld_q = qd;
    la.ld_kv = 2 * kvd;
    la.k_col = 0;
    la.v_col = kvd;
    la.ld_out = qd;
    la.scale_log2 = kLog2e;
    la.nblk = (seq + mk::AL_KEYS - 1) / mk::AL_KEYS;
    la.part = f32(ws.alpart);
    MK_TRY(launch_k(mk::attn_last_block_kernel, dim3(la.nblk, c.n_kv, bs), dim3(mk::AL_KEYS), 0, st, true,
                    static_cast<const __nv_bfloat16*>(ql), static_cast<const __nv_bfloat16*>(kv), la));
    MK_TRY(launch_k(mk::attn_last_combine_kernel, dim3(c.n_q, bs), dim3(mk::AL_HDMAX), 0, st, true, al, la));
    MK_TRY(launch_gemm(d, mal, h->m_o[l], bs, H, qd, mk::GEMM_RESID32, nullptr,
                       h->w.s_o + static_cast<size_t>(l) * H, xlb, H, r, st, xl32, H, resid_stats_last));
    MK_TRY(launch_gemm(d, mxl_gu, h->m_gu[l], bs, 2 * I, H, MK_GEMM_SWIGLU, nullptr,
                       h->w.s_gu + static_cast<size_t>(l) * 2 * I, hl, I, 0.f, st, nullptr, 0, norm_from(rowsql)));
    MK_TRY(launch_gemm(d, mhl, h->m_down[l], bs, H, I, mk::GEMM_RESID32, nullptr,
                       h->w.s_down + static_cast<size_t>(l) * H, xlb, H, r, st, xl32, H, resid_stats_last));
    MK_TRY(mark(MK_STAGE_LAST_LAYER, 8));
  }

  MK_TRY(launch_k(mk::final_norm_kernel, dim3(bs), dim3(256), 0, st, true, xl32, h->w.final_norm, hf,
                  static_cast<__nv_bfloat16*>(d_hidden), H, c.eps, c.logit_scale));
  MK_TRY(lm_head_launch(d, hf, bs, H, h->w.lm_head, c.vocab, logits, f32(ws.pval),
                        reinterpret_cast<int*>(base + ws.pidx), top1, st, true));
  return mark(MK_STAGE_HEAD, 1 + lm_launches(bs, H) + 1);
}
}  // namespace

extern "C" {

mk_status mk_forward(mk_handle* h, const int32_t* d_ids, int32_t bs, int32_t seq, void* d_workspace,
                     size_t workspace_bytes, void* d_hidden, float* d_logits, int32_t* d_top1, void* stream) {
  return forward_impl(h, d_ids, bs, seq, d_workspace, workspace_bytes, d_hidden, d_logits, d_top1, stream, nullptr);
}

mk_status mk_forward_timed(mk_handle* h, const int32_t* d_ids, int32_t bs, int32_t seq, void* d_workspace,
                           size_t workspace_bytes, void* d_hidden, float* d_logits, int32_t* d_top1, void* stream,
                           mk_stage_times* times) {
  if (!times) return MK_ERR_BAD_ARG;
  StageClock clk;
  MK_TRY(forward_impl(h, d_ids, bs, seq, d_workspace, workspace_bytes, d_hidden, d_logits, d_top1, stream, &clk));
  return clk.finish(times);
}

}  // extern "C"

namespace {
// Zig-zag block length for (seq, world); 0 if none fits.  A block holds whole attention query blocks
// (2 * 128 / G rows), whole 64-key tiles and whole 32-token RoPE chunks.
int sp_block(const mk_config& c, int seq, int world) {
  if (world < 1 || seq <= 0 || c.n_kv <= 0) return 0;
  const int min_blk = std::max(64, 256 / (c.n_q / c.n_kv));
  for (int b = 512; b >= min_blk; b >>= 1)
    if (seq % (2 * world * b) == 0) return b;
  return 0;
}

struct SpWorkspace {
  Workspace local;  // the single-sequence workspace of a rank's seq / world rows
  size_t kv_send, kv_all, alpart, apart, total;  // alpart: last-position attention partials over all seq keys
  int kchunk = 0;   // key tiles per attention CTA (0: no key split); apart: the split ranges' partials
};

SpWorkspace plan_workspace_sp(const mk_handle* h, int seq, int world) {
  SpWorkspace w;
  const int T = seq / world;
  w.local = plan_workspace(h, 1, T);
  const size_t kv_row = static_cast<size_t>(2 * h->kv_dim) * 2;
  w.kv_send = w.local.total;
  w.kv_all = align256(w.kv_send + T * kv_row);
  w.alpart = align256(w.kv_all + static_cast<size_t>(seq) * kv_row);
  w.apart = align256(w.alpart + static_cast<size_t>(h->cfg.n_q) * ((seq + mk::AL_KEYS - 1) / mk::AL_KEYS) *
                                    (h->cfg.head_dim + 2) * 4);
  const int blk = sp_block(h->cfg, seq, world);
  if (h->sp_key_split && blk > 0) {
    w.kchunk = -1;
    for (const auto& e : h->sp_chunk_cache)
      if (e[0] == seq && e[1] == world) w.kchunk = e[2];
    if (w.kchunk < 0) {
      mk::SpLayout sp;  // rank 0's layout
      sp.blk = blk;
      sp.world = world;
      sp.rows_per_rank = T;
      w.kchunk = sp_key_chunk(h->cfg, sp, seq, h->dev->sm_count);
      h->sp_chunk_cache.push_back({seq, world, w.kchunk});
    }
  }
  const size_t nsplit = w.kchunk > 0 ? mk::ta_nsplit(seq / mk::TA_BK, w.kchunk) : 0;
  w.total = align256(w.apart + nsplit * T * h->cfg.n_q * (h->cfg.head_dim + 4) * 4);
  return w;
}

mk_status forward_sp_impl(mk_handle* h, const int32_t* d_ids, int32_t seq, int32_t rank, int32_t world,
                          mk_allgather_fn allgather, void* ctx, void* d_workspace, size_t workspace_bytes,
                          void* d_hidden, float* d_logits, int32_t* d_top1, void* stream, StageClock* clk) {
  if (!h || !d_ids || !d_workspace || !allgather) return MK_ERR_BAD_ARG;
  if (world < 1 || rank < 0 || rank >= world) return MK_ERR_BAD_ARG;
  if (!h->bound) return MK_ERR_NOT_BOUND;
  const mk_config& c = h->cfg;
  if (seq <= 0 || seq % 128 || seq > c.max_seq) return MK_ERR_BAD_SHAPE;
  const int blk = sp_block(c, seq, world);
  if (blk == 0) return MK_ERR_BAD_SHAPE;
  if ((reinterpret_cast<uintptr_t>(d_workspace) & 255u) || !aligned16(d_ids)) return MK_ERR_BAD_ALIGN;
  if ((d_hidden && !aligned16(d_hidden)) || (d_logits && !aligned16(d_logits))) return MK_ERR_BAD_ALIGN;
  const SpWorkspace sw = plan_workspace_sp(h, seq, world);
  if (workspace_bytes < sw.total) return MK_ERR_WORKSPACE;
  MK_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DeviceState* d = h->dev;
  const Workspace& ws = sw.local;
  uint8_t* base = static_cast<uint8_t*>(d_workspace);
  auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(base + off); };
  auto f32 = [&](size_t off) { return reinterpret_cast<float*>(base + off); };

  const int L = c.num_layers, H = c.hidden, I = c.inter, hd = c.head_dim;
  const int T = seq / world;  // this rank's rows
  const int nqkv = h->n_qkv, qd = h->q_dim, kvd = h->kv_dim;
  mk::SpLayout sp;
  sp.blk = blk;
  sp.rank = rank;
  sp.world = world;
  sp.rows_per_rank = T;
  float *x32 = f32(ws.x32), *xl32 = f32(ws.xl32);
  __nv_bfloat16 *xb = bf(ws.xb), *qkv = bf(ws.qkv), *attn = bf(ws.attn), *hb = bf(ws.hbuf);
  __nv_bfloat16 *xlb = bf(ws.xlb), *ql = bf(ws.ql), *al = bf(ws.al), *hl = bf(ws.hl);
  __nv_bfloat16 *kv_send = bf(sw.kv_send), *kv_all = bf(sw.kv_all);
  float *rowsq = f32(ws.rowsq), *rowsql = f32(ws.rowsql), *hf = f32(ws.hf);
  float* logits = d_logits ? d_logits : f32(ws.logits);
  int32_t* top1 = d_top1 ? d_top1 : reinterpret_cast<int32_t*>(base + ws.top1);
  const float r = c.residual_scale;
  const size_t kv_row_bytes = static_cast<size_t>(2 * kvd) * 2;

  const int sms = d->sm_count;
  const int nt_qkv = plan_nt(T, nqkv, sms), nt_o = plan_nt(T, H, sms), nt_gu = plan_nt(T, 2 * I, sms);
  const int nt_down = nt_o, nt_kv = plan_nt(T, 2 * kvd, sms);
  CUtensorMap mx_qkv, mx_gu, mx_kv, mattn, mh, mxl, mxl_gu, mal, mhl;
  MK_TRY(map_a(&mx_qkv, xb, T, H, H, a_box(T, nqkv, nt_qkv)));
  MK_TRY(map_a(&mx_gu, xb, T, H, H, a_box(T, 2 * I, nt_gu)));
  MK_TRY(map_a(&mx_kv, xb, T, H, H, a_box(T, 2 * kvd, nt_kv)));
  MK_TRY(map_a(&mattn, attn, T, qd, qd, a_box(T, H, nt_o)));
  MK_TRY(map_a(&mh, hb, T, I, I, a_box(T, H, nt_down)));
  MK_TRY(map_a(&mxl, xlb, 1, H, H));
  MK_TRY(map_a(&mxl_gu, xlb, 1, H, H));
  MK_TRY(map_a(&mal, al, 1, qd, qd));
  MK_TRY(map_a(&mhl, hl, 1, I, I));
  auto tiles = [](GemmFusion f, int nt) {
    f.nt = nt;
    return f;
  };

  auto mark = [&](int stage, int launches) { return clk ? clk->mark(stage, launches) : MK_OK; };
  if (clk) MK_TRY(clk->start(st));
  const int rows_per_blk = 8;
  const int np = H / 128;
  mk::embed_kernel<<<(T + rows_per_blk - 1) / rows_per_blk, 256, 0, st>>>(
      d_ids, static_cast<const __nv_bfloat16*>(h->w.embed), x32, xb, T, H, c.vocab, c.scale_emb, d->err, rowsq, np,
      sp);
  MK_CUDA(cudaGetLastError());
  MK_TRY(mark(MK_STAGE_EMBED, 1));

  auto norm_from = [&](float* sq) {
    GemmFusion f;
    f.rowsq = sq;
    f.rowsq_ld = np;
    f.rowsq_np = np;
    f.inv_norm_dim = 1.0f / static_cast<float>(H);
    f.eps = c.eps;
    f.pdl = true;
    f.wbf16 = h->wbf16;
    return f;
  };
  // RoPE at the zig-zag positions of this rank's rows
  auto with_rope_sp = [&](GemmFusion f, int cols) {
    f.rope_cos = h->w.rope_cos;
    f.rope_sin = h->w.rope_sin;
    f.rope_cols = cols;
    f.head_dim = hd;
    f.rope_seq = seq;
    f.rope_pos_base = 0;
    f.sp = sp;
    return f;
  };
  GemmFusion resid_stats;
  resid_stats.rowsq = rowsq;
  resid_stats.pdl = true;
  resid_stats.wbf16 = h->wbf16;
  resid_stats.rowsq_ld = np;
  GemmFusion resid_stats_last = resid_stats;
  resid_stats_last.rowsq = rowsql;
  // K/V columns of the local QKV rows -> packed send rows -> every rank's rows, rank by rank
  auto gather_kv = [&](const __nv_bfloat16* src, int ld_src) -> mk_status {
    MK_CUDA(cudaMemcpy2DAsync(kv_send, kv_row_bytes, src, static_cast<size_t>(ld_src) * 2, kv_row_bytes, T,
                              cudaMemcpyDeviceToDevice, st));
    if (allgather(ctx, kv_send, kv_all, static_cast<size_t>(T) * kv_row_bytes, stream) != 0) return MK_ERR_CUDA;
    return MK_OK;
  };

  for (int l = 0; l < L - 1; ++l) {
    MK_TRY(launch_gemm(d, mx_qkv, h->m_qkv[l], T, nqkv, H, MK_GEMM_ROWSCALE, nullptr,
                       h->w.s_qkv + static_cast<size_t>(l) * nqkv, qkv, nqkv, 0.f, st, nullptr, 0,
                       tiles(with_rope_sp(norm_from(rowsq), qd + kvd), nt_qkv)));
    MK_TRY(mark(MK_STAGE_QKV, 1));
    MK_TRY(gather_kv(qkv + qd, nqkv));
    MK_TRY(mark(MK_STAGE_KV_GATHER, 0));
    MK_TRY(launch_attn_split(d, qkv, T, nqkv, 0, kv_all, seq, 2 * kvd, 0, kvd, 1, c.n_q, c.n_kv, hd, kLog2e, attn, qd,
                             st, sp, true, sw.kchunk, f32(sw.apart)));
    MK_TRY(mark(MK_STAGE_ATTN, sw.kchunk > 0 ? 2 : 1));
    MK_TRY(launch_gemm(d, mattn, h->m_o[l], T, H, qd, mk::GEMM_RESID32, nullptr,
                       h->w.s_o + static_cast<size_t>(l) * H, xb, H, r, st, x32, H, tiles(resid_stats, nt_o)));
    MK_TRY(mark(MK_STAGE_O, 1));
    MK_TRY(launch_gemm(d, mx_gu, h->m_gu[l], T, 2 * I, H, MK_GEMM_SWIGLU, nullptr,
                       h->w.s_gu + static_cast<size_t>(l) * 2 * I, hb, I, 0.f, st, nullptr, 0,
                       tiles(norm_from(rowsq), nt_gu)));
    MK_TRY(mark(MK_STAGE_GATE_UP, 1));
    MK_TRY(launch_gemm(d, mh, h->m_down[l], T, H, I, mk::GEMM_RESID32, nullptr,
                       h->w.s_down + static_cast<size_t>(l) * H, xb, H, r, st, x32, H, tiles(resid_stats, nt_down)));
    MK_TRY(mark(MK_STAGE_DOWN, 1));
  }

  // Last layer: every rank projects K/V of its rows; rank 0 owns the last position (the second block
  // of the last zig-zag group) and runs the rest for it.
  {
    const int l = L - 1;
    const float* sq = h->w.s_qkv + static_cast<size_t>(l) * nqkv;
    __nv_bfloat16* kv = qkv;  // [T, 2 kv_dim]
    MK_TRY(launch_gemm(d, mx_kv, h->m_kv_last, T, 2 * kvd, H, MK_GEMM_ROWSCALE, nullptr, sq + qd, kv, 2 * kvd, 0.f, st,
                       nullptr, 0, tiles(with_rope_sp(norm_from(rowsq), kvd), nt_kv)));
    MK_TRY(mark(MK_STAGE_LAST_LAYER, 1));
    MK_TRY(gather_kv(kv, 2 * kvd));
    MK_TRY(mark(MK_STAGE_KV_GATHER, 0));
    if (rank != 0) return MK_OK;
    MK_TRY(launch_k(mk::gather_last_kernel, dim3(1), dim3(256), 0, st, true, x32, xl32, xlb, 1, T, H, rowsq, rowsql, np));
    GemmFusion fq = norm_from(rowsql);
    fq.rope_cos = h->w.rope_cos;
    fq.rope_sin = h->w.rope_sin;
    fq.rope_cols = qd;
    fq.head_dim = hd;
    fq.rope_seq = 1;
    fq.rope_pos_base = seq - 1;
    MK_TRY(launch_gemm(d, mxl, h->m_q_last, 1, qd, H, MK_GEMM_ROWSCALE, nullptr, sq, ql, qd, 0.f, st, nullptr, 0, fq));
    AttnLastArgs la;
    la.S = seq;
    la.n_q = c.n_q;
    la.n_kv = c.n_kv;
    la.head_dim = hd;
    la.ld_q = qd;
    la.ld_kv = 2 * kvd;
    la.k_col = 0;
    la.v_col = kvd;
    la.ld_out = qd;
    la.scale_log2 = kLog2e;
    la.sp = sp;
    la.nblk = (seq + mk::AL_KEYS - 1) / mk::AL_KEYS;
    la.part = f32(sw.alpart);
    MK_TRY(launch_k(mk::attn_last_block_kernel, dim3(la.nblk, c.n_kv, 1), dim3(mk::AL_KEYS), 0, st, true,
                    static_cast<const __nv_bfloat16*>(ql), static_cast<const __nv_bfloat16*>(kv_all), la));
    MK_TRY(launch_k(mk::attn_last_combine_kernel, dim3(c.n_q, 1), dim3(mk::AL_HDMAX), 0, st, true, al, la));
    MK_TRY(launch_gemm(d, mal, h->m_o[l], 1, H, qd, mk::GEMM_RESID32, nullptr,
                       h->w.s_o + static_cast<size_t>(l) * H, xlb, H, r, st, xl32, H, resid_stats_last));
    MK_TRY(launch_gemm(d, mxl_gu, h->m_gu[l], 1, 2 * I, H, MK_GEMM_SWIGLU, nullptr,
                       h->w.s_gu + static_cast<size_t>(l) * 2 * I, hl, I, 0.f, st, nullptr, 0, norm_from(rowsql)));
    MK_TRY(launch_gemm(d, mhl, h->m_down[l], 1, H, I, mk::GEMM_RESID32, nullptr,
                       h->w.s_down + static_cast<size_t>(l) * H, xlb, H, r, st, xl32, H, resid_stats_last));
    MK_TRY(mark(MK_STAGE_LAST_LAYER, 7));
  }
  MK_TRY(launch_k(mk::final_norm_kernel, dim3(1), dim3(256), 0, st, true, xl32, h->w.final_norm, hf,
                  static_cast<__nv_bfloat16*>(d_hidden), H, c.eps, c.logit_scale));
  MK_TRY(lm_head_launch(d, hf, 1, H, h->w.lm_head, c.vocab, logits, f32(ws.pval), reinterpret_cast<int*>(base + ws.pidx),
                        top1, st, true));
  return mark(MK_STAGE_HEAD, 3);
}
}  // namespace

extern "C" {

int32_t mk_sp_block(const mk_handle* h, int32_t seq, int32_t world) { return h ? sp_block(h->cfg, seq, world) : 0; }

mk_status mk_set_sp_key_split(mk_handle* h, int32_t enabled) {
  if (!h) return MK_ERR_BAD_ARG;
  h->sp_key_split = enabled != 0;
  return MK_OK;
}

mk_status mk_workspace_size_sp(const mk_handle* h, int32_t seq, int32_t world, size_t* bytes) {
  if (!h || !bytes) return MK_ERR_BAD_ARG;
  if (world < 1) return MK_ERR_BAD_ARG;
  if (sp_block(h->cfg, seq, world) == 0) return MK_ERR_BAD_SHAPE;
  *bytes = plan_workspace_sp(h, seq, world).total;
  return MK_OK;
}

mk_status mk_forward_sp(mk_handle* h, const int32_t* d_ids, int32_t seq, int32_t rank, int32_t world,
                        mk_allgather_fn allgather, void* allgather_ctx, void* d_workspace, size_t workspace_bytes,
                        void* d_hidden, float* d_logits, int32_t* d_top1, void* stream, mk_stage_times* times) {
  if (!times)
    return forward_sp_impl(h, d_ids, seq, rank, world, allgather, allgather_ctx, d_workspace, workspace_bytes, d_hidden,
                           d_logits, d_top1, stream, nullptr);
  StageClock clk;
  MK_TRY(forward_sp_impl(h, d_ids, seq, rank, world, allgather, allgather_ctx, d_workspace, workspace_bytes, d_hidden,
                         d_logits, d_top1, stream, &clk));
  return clk.finish(times);
}

int32_t mk_launches_per_forward(const mk_handle* h, int32_t bs, int32_t seq) {
  if (!h || bs <= 0 || seq <= 0) return 0;
  const int per_layer = 5;  // qkv gemm (+RMSNorm, RoPE), attention, o gemm, gate/up gemm, down gemm
  const int last_layer = 8; // kv gemm, gather, q gemm, attention (blocks + combine), o, gate/up, down gemms
  return 1 + (h->cfg.num_layers - 1) * per_layer + last_layer + 1 + lm_launches(bs, h->cfg.hidden) + 1;
}

mk_status mk_get_error(mk_handle* h, int32_t* device_err) {
  if (h) MK_CUDA(cudaSetDevice(h->device));
  MK_CUDA(cudaDeviceSynchronize());
  int v = 0;
  MK_CUDA(cudaMemcpyFromSymbol(&v, g_mk_err, sizeof(int)));
  const int zero = 0;
  MK_CUDA(cudaMemcpyToSymbol(g_mk_err, &zero, sizeof(int)));
  if (device_err) *device_err = v;
  if (v == 0) return MK_OK;
  if (v == mk::DEV_ERR_BAD_TOKEN_ID) return MK_ERR_BAD_TOKEN;
  return MK_ERR_DEVICE_TIMEOUT;
}

void mk_destroy(mk_handle* h) { delete h; }

// ------------------------------------------------------------------------------ isolated kernels
mk_status mk_gemm_w8a16_fused(const void* a, int32_t M, int32_t K, int32_t lda, const void* w,
                              const float* col_scale, int32_t N, int32_t mode, const float* row_scale,
                              float resid_scale, void* out, int32_t ldo, float* resid32, int32_t ld_resid32,
                              const mk_gemm_fusion* fusion, void* stream) {
  if (!a || !w || !col_scale || !out) return MK_ERR_BAD_ARG;
  MK_TRY(check_gemm_shape(M, N, K, mode));
  GemmFusion fu;
  const bool norm_in = fusion && fusion->rowsq && fusion->rowsq_np > 0 &&
                       (mode == MK_GEMM_ROWSCALE || mode == MK_GEMM_SWIGLU);
  if (fusion) {
    if (fusion->weight_bits != 0 && fusion->weight_bits != 8 && fusion->weight_bits != 16) return MK_ERR_BAD_ARG;
    fu.wbf16 = fusion->weight_bits == 16;
    if (fusion->rowsq) {
      if (reinterpret_cast<uintptr_t>(fusion->rowsq) & 3u) return MK_ERR_BAD_ALIGN;
      if (norm_in) {
        if (fusion->rowsq_np > fusion->rowsq_ld || fusion->norm_dim <= 0) return MK_ERR_BAD_SHAPE;
      } else if (mode == MK_GEMM_RESID32) {
        if (fusion->rowsq_ld < N / 128) return MK_ERR_BAD_SHAPE;
      } else {
        return MK_ERR_BAD_ARG;  // statistics are read by ROWSCALE / SWIGLU and written by RESID32 only
      }
      fu.rowsq = fusion->rowsq;
      fu.rowsq_ld = fusion->rowsq_ld;
      fu.rowsq_np = norm_in ? fusion->rowsq_np : 0;
      fu.inv_norm_dim = norm_in ? 1.0f / static_cast<float>(fusion->norm_dim) : 0.f;
      fu.eps = fusion->eps;
    }
    if (fusion->rope_cols > 0) {
      if (mode != MK_GEMM_ROWSCALE || !fusion->rope_cos || !fusion->rope_sin) return MK_ERR_BAD_ARG;
      if (fusion->rope_cols % 32 || fusion->rope_cols > N || fusion->head_dim <= 0 || fusion->head_dim % 2 ||
          fusion->rope_seq <= 0 || fusion->rope_pos_base < 0)
        return MK_ERR_BAD_SHAPE;
      fu.rope_cos = fusion->rope_cos;
      fu.rope_sin = fusion->rope_sin;
      fu.rope_cols = fusion->rope_cols;
      fu.head_dim = fusion->head_dim;
      fu.rope_seq = fusion->rope_seq;
      fu.rope_pos_base = fusion->rope_pos_base;
    }
  }
  if ((mode == MK_GEMM_ROWSCALE || mode == MK_GEMM_SWIGLU) && !row_scale && !norm_in) return MK_ERR_BAD_ARG;
  if (mode == MK_GEMM_RESID32 && (!resid32 || !aligned16(resid32) || ld_resid32 % 4 || ld_resid32 < N))
    return resid32 ? MK_ERR_BAD_ALIGN : MK_ERR_BAD_ARG;
  if (!aligned16(a) || !aligned16(w) || !aligned16(out) || lda % 8 || ldo % 8 || lda < K) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  fu.nt = plan_nt(M, N, d->sm_count);
  CUtensorMap ma, mb;
  MK_TRY(map_a(&ma, a, M, K, lda, a_box(M, N, fu.nt)));
  MK_TRY(map_b(&mb, w, N, K, kWeightBoxRows, fu.wbf16));
  return launch_gemm(d, ma, mb, M, N, K, mode, row_scale, col_scale, out, ldo, resid_scale,
                     static_cast<cudaStream_t>(stream), resid32, ld_resid32, fu);
}

mk_status mk_gemm_w8a16(const void* a, int32_t M, int32_t K, int32_t lda, const int8_t* w, const float* col_scale,
                        int32_t N, int32_t mode, const float* row_scale, float resid_scale, void* out, int32_t ldo,
                        float* resid32, int32_t ld_resid32, void* stream) {
  return mk_gemm_w8a16_fused(a, M, K, lda, w, col_scale, N, mode, row_scale, resid_scale, out, ldo, resid32,
                             ld_resid32, nullptr, stream);
}

mk_status mk_attention_prefill(const void* qkv, int32_t bs, int32_t seq, int32_t n_q, int32_t n_kv,
                               int32_t head_dim, int32_t ld_qkv, int32_t q_col, int32_t k_col, int32_t v_col,
                               float softmax_scale, void* out, int32_t ld_out, void* stream) {
  if (!qkv || !out) return MK_ERR_BAD_ARG;
  MK_TRY(check_attn_shape(bs, seq, n_q, n_kv, head_dim, ld_qkv, q_col, k_col, v_col, ld_out));
  if (!aligned16(qkv) || !aligned16(out)) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  return launch_attn(d, qkv, bs, seq, n_q, n_kv, head_dim, ld_qkv, q_col, k_col, v_col, softmax_scale * kLog2e, out,
                     ld_out, static_cast<cudaStream_t>(stream));
}

mk_status mk_rope(void* x, int32_t rows, int32_t ld, int32_t col0, int32_t n_heads, int32_t head_dim,
                  const float* rope_cos, const float* rope_sin, int32_t seq, int32_t pos_base, void* stream) {
  if (!x || !rope_cos || !rope_sin) return MK_ERR_BAD_ARG;
  if (rows <= 0 || n_heads <= 0 || seq <= 0 || head_dim % 4 || pos_base < 0) return MK_ERR_BAD_SHAPE;
  if (ld % 2 || col0 % 2 || (reinterpret_cast<uintptr_t>(x) & 3u)) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  const size_t work = static_cast<size_t>(rows) * n_heads * (head_dim / 4);
  const int blocks = static_cast<int>(std::min<size_t>((work + 255) / 256, static_cast<size_t>(d->sm_count) * 16));
  mk::rope_kernel<<<std::max(blocks, 1), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), rope_cos, rope_sin, rows, ld, col0, n_heads, head_dim, seq, pos_base);
  return cuda_status(cudaGetLastError());
}

mk_status mk_rms_rstd(const float* x, int32_t T, int32_t H, int32_t ld, float eps, float* rstd, void* stream) {
  if (!x || !rstd) return MK_ERR_BAD_ARG;
  if (T <= 0 || H <= 0 || H % 8) return MK_ERR_BAD_SHAPE;
  if (!aligned16(x) || ld % 4) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  mk::rms_rstd_kernel<<<(T + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, rstd, T, H, ld, eps);
  return cuda_status(cudaGetLastError());
}

mk_status mk_embed(const int32_t* ids, int32_t T, const void* embed, int32_t V, int32_t H, float scale, float* x32,
                   void* xb, void* stream) {
  if (!ids || !embed || !x32 || !xb) return MK_ERR_BAD_ARG;
  if (T <= 0 || V <= 0 || H <= 0 || H % 8) return MK_ERR_BAD_SHAPE;
  if (!aligned16(embed) || !aligned16(x32) || !aligned16(xb)) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  mk::embed_kernel<<<(T + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, static_cast<const __nv_bfloat16*>(embed), x32, static_cast<__nv_bfloat16*>(xb), T, H, V, scale, d->err);
  return cuda_status(cudaGetLastError());
}

int32_t mk_lm_head_parts(void) { return kLmParts; }

mk_status mk_lm_head_argmax(const float* hvec, int32_t bs, int32_t H, const void* lm_head, int32_t V, float* logits,
                            float* part_val, int32_t* part_idx, int32_t* top1, void* stream) {
  if (!hvec || !lm_head || !logits || !part_val || !part_idx || !top1) return MK_ERR_BAD_ARG;
  if (bs <= 0 || H <= 0 || H % 8 || V <= 0) return MK_ERR_BAD_SHAPE;
  if (!aligned16(lm_head)) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  return lm_head_launch(d, hvec, bs, H, lm_head, V, logits, part_val, part_idx, top1,
                        static_cast<cudaStream_t>(stream));
}

mk_status mk_topk_logprobs(const float* logits, int32_t bs, int32_t V, int32_t ld, int32_t k, int32_t* ids,
                           float* logprobs, void* stream) {
  if (!logits || !ids || !logprobs) return MK_ERR_BAD_ARG;
  if (bs <= 0 || V <= 0 || ld < V || k <= 0 || k > mk::TOPK_MAX || k > V) return MK_ERR_BAD_SHAPE;
  if (reinterpret_cast<uintptr_t>(logits) & 3u) return MK_ERR_BAD_ALIGN;
  mk::topk_logprobs_kernel<<<bs, mk::TOPK_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(logits, V, ld, k, ids,
                                                                                          logprobs);
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------------------------------------ allocation-free lm_head
}  // extern "C"

namespace {
// Scratch of mk_lm_head_argmax_noalloc: per-block argmax values then indices for up to
// MK_LM_HEAD_NOALLOC_MAX_ROWS rows.  One copy per device that loads the library, kept until exit.
constexpr int kNoAllocRows = MK_LM_HEAD_NOALLOC_MAX_ROWS;
constexpr size_t kNoAllocValBytes = static_cast<size_t>(kNoAllocRows) * kLmParts * sizeof(float);
constexpr size_t kNoAllocBytes = kNoAllocValBytes + static_cast<size_t>(kNoAllocRows) * kLmParts * sizeof(int32_t);
static __device__ __align__(256) unsigned char g_lm_noalloc_scratch[kNoAllocBytes];

// Device address of g_lm_noalloc_scratch per device (host code may only use the symbol through
// cudaGetSymbolAddress: its name on the host is a stand-in, not a device pointer).
unsigned char* g_noalloc_ptr[kMaxDevices] = {};

mk_status noalloc_scratch(unsigned char** out) {
  int dev = 0;
  MK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return MK_ERR_BAD_ARG;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_lm_noalloc_scratch);
    if (e != cudaSuccess || !p) return MK_ERR_CUDA;
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MK_OK;
}
}  // namespace

extern "C" mk_status mk_lm_head_argmax_noalloc(const float* hvec, int32_t bs, int32_t H, const void* lm_head,
                                               int32_t V, float* logits, int32_t* top1, void* stream) {
  if (!hvec || !lm_head || !logits || !top1) return MK_ERR_BAD_ARG;
  if (bs > kNoAllocRows) return MK_ERR_TOO_LARGE;
  if (bs <= 0 || H <= 0 || H % 8 || V <= 0) return MK_ERR_BAD_SHAPE;
  if (!aligned16(lm_head)) return MK_ERR_BAD_ALIGN;
  DeviceState* d = nullptr;
  MK_TRY(device_state(&d));
  unsigned char* scratch = nullptr;
  MK_TRY(noalloc_scratch(&scratch));
  float* pval = reinterpret_cast<float*>(scratch);
  int* pidx = reinterpret_cast<int*>(scratch + kNoAllocValBytes);
  return lm_head_launch(d, hvec, bs, H, lm_head, V, logits, pval, pidx, top1, static_cast<cudaStream_t>(stream));
}
