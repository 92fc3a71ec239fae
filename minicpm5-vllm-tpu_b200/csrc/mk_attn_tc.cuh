// Causal GQA flash attention on tcgen05 (sm_100a): S = Q K^T and O += P V run on the tensor
// cores with S, P and O held in TMEM; the online softmax runs in f32 with one thread per row.
//
// Reference counterpart: `super_gqa_v2` (plugin/minicpm5_mk/mk_attn.py:557-710): causal GQA
// prefill where every K/V tile is staged once per KV group and shared by all of the group's query
// heads.  Math spec: `_attn_chunk` (benchmark/f32_golden.py:62-75).
//
// One CTA = one KV head g of one sequence x one block of queries.  The G = n_q / n_kv query heads
// of the group are stacked with the queries into 128-row tiles (row r = query r / G, head r % G);
// the CTA owns two such tiles (Q0, Q1) that share each 64-key K/V tile:
//
//   warp 0      TMA producer: Q0/Q1 once (3D map over [token, head, dim], 128B swizzle), then a
//               4-stage ring of K and V tiles (K: K-major operand; V: MN-major operand)
//   warps 1, 2  MMA issuers, one per query tile (warp 1 also allocates TMEM); each runs its loop
//               warp-wide and one elected lane issues.  For 64-key tile j it issues
//                 S_t(j+1) = Q_t K_{j+1}^T into the other S buffer of tile t  (M=128, N=64, K=hd)
//                 O_t += P_t(j) V_j  once the softmax has written P_t(j)        (M=128, N=hd, K=64)
//               so the tensor core computes the next scores while the softmax works on this tile;
//               it relies on the in-order execution of one thread's tcgen05.mma ops instead of
//               waiting for O_t += P_t(j-1) V before reusing its S buffer.
//   warps 4..7  softmax of tile 0, warps 8..11 softmax of tile 1: thread i owns row i of S_t
//               (TMEM lane i), loads its 64 scores once, takes the max, writes P = exp2(S*c - m) as
//               bf16 pairs over the same TMEM columns (P_t aliases S_t).  The running max is only
//               moved (and O_t rescaled in TMEM) when it grows by more than 2^8, so rescaling is
//               rare; P stays <= 256.  At the end the same threads normalise O_t by the row sum and
//               store bf16 rows.
//
// TMEM (512 columns): S_t[b] at [128t + 64b, +64) for tile t and buffer b; O_t at [256 + 128t, +hd);
// for head_dim 96, Q_t's dimensions [0, 64) as bf16 pairs at [256 + 128t + 96, +32).
// Shared memory: Q 2 tiles x 2 chunks (128 rows x 128 B each), K and V 4 stages x 2 chunks
// (64 rows x 128 B each).  head_dim 96 uses a second 64-column chunk whose upper 32 columns are
// TMA zero-fill and never read by the MMAs.
#pragma once

#include "mk_common.cuh"

namespace mk {

constexpr int TA_BK = 64;
constexpr int TA_STAGES = 4;
constexpr int TA_THREADS = 384;
constexpr uint32_t TA_QCHUNK = 128 * 128;   // 128 rows x 128 bytes
constexpr uint32_t TA_KCHUNK = TA_BK * 128;  // 64 rows x 128 bytes
constexpr uint32_t TA_STAGE = 4 * TA_KCHUNK;  // K (2 chunks) + V (2 chunks)
constexpr size_t TA_SMEM = 1024 + 4 * TA_QCHUNK + TA_STAGES * TA_STAGE + 256;
constexpr float TA_RESCALE_THRESHOLD = 8.0f;  // log2 units

// head_dim 96 leaves 32 TMEM columns after each O_t: they hold Q_t's first 64 dimensions, so the first
// four K-steps of S = Q K^T take A from TMEM and read only K from shared memory.  An SS UMMA with
// N = 64 is bound by shared-memory bandwidth (6 KB of operands per 32 tensor cycles); from TMEM it
// runs at the full tensor rate.
template <int HD>
__host__ __device__ constexpr int ta_q_tmem_ksteps() { return HD == 96 ? 4 : 0; }

// Pairs of softmax exponentials e with (e & TA_FMA_EXP_MASK) == TA_FMA_EXP_MASK go to the FMA pipe.
constexpr int TA_FMA_EXP_MASK = 15;

// 2^x on the FMA pipe for a share of the softmax exponentials: 16 MUFU results per clock per SM
// cannot keep up with the tensor core at head_dim 96.  x = j + f with j = round(x) (adding
// 1.5 * 2^23 rounds x into the low mantissa bits of t) and f in [-0.5, 0.5]; 2^f is a cubic fitted by
// least squares to 2^f on [-0.5, 0.5] (max relative error 7.8e-5, far below the bf16 rounding of P);
// 2^j is added to the exponent field.  x is clamped at -125 (result about 2e-38, so the exponent
// field stays positive; -inf maps there too).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.0550887659f, f, 0.242604658f), f, 0.693276286f), f, 0.999928892f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

struct AttnTcArgs {
  int S;       // sequence length (K/V rows per sequence)
  int rows;    // query / output rows per sequence (S, or a rank's rows under sequence parallelism)
  int lg2G;    // log2(query heads per KV head)
  int nqb;     // query blocks (of 2 * 128/G queries) per sequence: rows / (2 * 128/G)
  int ld_out;  // elements per output row
  float scale_log2;
  // Sequence parallelism (sp.blk > 0, bs = 1): the query rows are this rank's zig-zag rows (row m at
  // position sp_pos(sp, m)) and K/V is the rank-by-rank all-gather (position p at row sp_row(sp, p)).
  SpLayout sp;
  // Key split (the KSPLIT instantiation, kchunk > 0, one sequence): a query block with more than kchunk
  // key tiles is cut into ta_nsplit near-equal key ranges, one CTA each (blockIdx.x = range); such CTAs
  // write the unnormalised O, the running max and the row sum to `part` ([range][row][n_q][hd + 4] f32)
  // and attn_split_combine_kernel merges the ranges.  Query blocks of one range write `out` directly.
  int kchunk;
  int n_q;
  float* part;
  int* err;
};

// Key ranges of a query block with ntot key tiles: nsplit ranges of `per` tiles (the last one may be
// shorter); none is empty.
__host__ __device__ __forceinline__ int ta_nsplit(int ntot, int kchunk) {
  return kchunk > 0 ? (ntot + kchunk - 1) / kchunk : 1;
}
__host__ __device__ __forceinline__ int ta_split_per(int ntot, int nsplit) { return (ntot + nsplit - 1) / nsplit; }

// KSPLIT: the key-split variant (AttnTcArgs::kchunk); the other instantiation keeps the plain code path.
template <int HD, bool KSPLIT>
__global__ void __launch_bounds__(TA_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out, const AttnTcArgs a) {
  static_assert(HD == 96 || HD == 128, "head_dim");
  extern __shared__ uint8_t ta_smem_raw[];
  const uint32_t raw = smem_u32(ta_smem_raw);
  uint8_t* sbase = ta_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sbase;                    // [tile][chunk], 16 KB each
  uint8_t* sKV = sbase + 4 * TA_QCHUNK;   // [stage]{K chunk 0, K chunk 1, V chunk 0, V chunk 1}, 8 KB each
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + TA_STAGES * TA_STAGE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                  // [TA_STAGES]
  uint64_t* v_full = k_full + TA_STAGES;        // [TA_STAGES]
  uint64_t* kv_empty = v_full + TA_STAGES;      // [TA_STAGES]
  uint64_t* s_full = kv_empty + TA_STAGES;      // [2 tiles][2 buffers]
  uint64_t* p_ready = s_full + 4;               // [2 tiles][2 buffers]
  uint64_t* pv_done = p_ready + 4;              // [2 tiles]
  uint64_t* drain = pv_done + 2;
  uint64_t* q_tm = drain + 1;                   // [2 tiles]: Q_t's first dimensions are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_tm + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = 1 << a.lg2G;
  const int qpt = 128 >> a.lg2G;  // queries per Q tile
  // Grid (query block, KV head, sequence), heaviest blocks first; with the key split (key range, query
  // block, KV head), so that the ranges of one block are dispatched together, heaviest blocks first.
  const int qb = a.nqb - 1 - static_cast<int>(KSPLIT ? blockIdx.y : blockIdx.x);
  const int qrow0 = qb * 2 * qpt;      // first query row of the CTA (local)
  const int q0 = sp_pos(a.sp, qrow0);  // its position; the 2 * qpt rows share one zig-zag block
  const int g = KSPLIT ? blockIdx.z : blockIdx.y;
  const int seqi = KSPLIT ? 0 : static_cast<int>(blockIdx.z);
  const int tok0 = seqi * a.rows;  // query / output rows of this sequence
  const int kv0 = seqi * a.S;      // K/V rows of this sequence
  const int ntot = (q0 + 2 * qpt - 1) / TA_BK + 1;  // key tiles up to the block's last position
  const int nsplit = KSPLIT ? ta_nsplit(ntot, a.kchunk) : 1;
  const int chunk = KSPLIT ? static_cast<int>(blockIdx.x) : 0;
  if (chunk >= nsplit) return;  // the whole CTA: this block has fewer key ranges
  const int kt0 = chunk * ta_split_per(ntot, nsplit);  // first key tile of this CTA's range
  const int ntiles = min(ntot, kt0 + ta_split_per(ntot, nsplit)) - kt0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < TA_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 2);  // one commit per MMA issuer
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(drain, 2);
    mbar_init(&q_tm[0], 4);
    mbar_init(&q_tm[1], 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // Q, K and V come from the previous kernel

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    // The whole warp runs the loop (warp-uniform addresses); one elected lane issues the copies.
    const bool leader = elect_one();
    uint32_t issued = 0, issued_par = 0;  // bit s: stage s has loads in flight / their parity
    if (leader) {
      mbar_arrive_expect_tx(q_full, 4 * TA_QCHUNK);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < 2; ++c)
          tma_load_3d(sQ + (t * 2 + c) * TA_QCHUNK, &tmQ, q_full, c * 64, g * G, tok0 + qrow0 + t * qpt);
    }
    __syncwarp();
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % TA_STAGES;
      const uint32_t ph = (j / TA_STAGES) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag))) break;
      uint8_t* sst = sKV + st * TA_STAGE;
      if (leader) {
        mbar_arrive_expect_tx(&k_full[st], 2 * TA_KCHUNK);
        // a 64-key tile never straddles a zig-zag block (blocks are multiples of 64 tokens)
        const int krow = kv0 + sp_row(a.sp, (kt0 + j) * TA_BK);
        for (int c = 0; c < 2; ++c) tma_load_3d(sst + c * TA_KCHUNK, &tmK, &k_full[st], c * 64, g, krow);
        mbar_arrive_expect_tx(&v_full[st], 2 * TA_KCHUNK);
        for (int c = 0; c < 2; ++c)
          tma_load_3d(sst + (2 + c) * TA_KCHUNK, &tmV, &v_full[st], c * 64, g, krow);
      }
      __syncwarp();
      issued |= 1u << st;
      issued_par = (issued_par & ~(1u << st)) | (ph << st);
    }
    // every issued copy must land before the CTA exits
    mbar_wait_drain(q_full, 0);
    for (int st = 0; st < TA_STAGES; ++st)
      if (issued & (1u << st)) {
        mbar_wait_drain(&k_full[st], (issued_par >> st) & 1u);
        mbar_wait_drain(&v_full[st], (issued_par >> st) & 1u);
      }
  } else if (warp == 1 || warp == 2) {
    // ---------------------------------------------------------------- MMA issuers
    // Warp 1 issues the UMMAs of query tile 0, warp 2 those of tile 1: a single issuing thread
    // needs about 50 cycles per UMMA, more than a 64-key S UMMA takes to execute, so one issuer
    // per tile keeps the tensor pipe fed.  The two touch disjoint TMEM (S_t, P_t, O_t) and only
    // read the shared K/V stages; each waits for the same K/V barriers and releases a stage with its
    // own commit (kv_empty counts two).  Each whole warp runs its loop (warp-uniform descriptors) and
    // one elected lane issues.
    const int t = warp - 1;
    const bool leader = elect_one();
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, TA_BK);
    constexpr uint32_t idesc_pv = idesc_bf16_f32_bmn(128, HD);
    // S_t(j) = Q_t K_j^T into S buffer j & 1 of tile t
    auto issue_s = [&](int j) {
      const uint8_t* kb = sKV + (j % TA_STAGES) * TA_STAGE;
      const uint32_t d = tmem + t * 128 + (j & 1) * 64;
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const int c = ks >> 2;
          const uint64_t db = sdesc_kmajor_sw128(smem_u32(kb + c * TA_KCHUNK)) + 2 * (ks & 3);
          if (ks < ta_q_tmem_ksteps<HD>()) {
            mma_f16_ts(d, tmem + 256 + t * 128 + HD + ks * 8, db, idesc_s, ks > 0 ? 1u : 0u);
          } else {
            const uint64_t da = sdesc_kmajor_sw128(smem_u32(sQ + (t * 2 + c) * TA_QCHUNK)) + 2 * (ks & 3);
            mma_f16_ss(d, da, db, idesc_s, ks > 0 ? 1u : 0u);
          }
        }
        mma_commit(&s_full[t * 2 + (j & 1)]);
      }
      __syncwarp();
    };
    // The path from the softmax's p_ready(j) to S_t(j+2) being ready bounds the loop: O_t += P_t(j) V_j
    // and S_t(j+2) are issued back to back with no barrier wait between them.  The K/V waits for later
    // tiles are taken while this warp waits for the softmax anyway.
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, abort_flag) && mbar_wait(&k_full[0], 0, abort_flag) &&
                                          (ntiles < 2 || mbar_wait(&k_full[1 % TA_STAGES], 0, abort_flag)) &&
                                          (ta_q_tmem_ksteps<HD>() == 0 || mbar_wait(&q_tm[t], 0, abort_flag)));
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; ok && j < ntiles; ++j) {
      const int st = j % TA_STAGES;
      if (j + 1 < ntiles) {
        // K_{j+1} has landed (waited for in the previous iteration).  S buffer (j+1)&1 still holds
        // P_t(j-1), read by O_t += P_t(j-1) V.  tcgen05.mma ops issued by this thread execute in issue
        // order, so S_t(j+1) (issued after that P V) overwrites P_t(j-1) only after it has been read:
        // no wait, the tensor pipe stays full.  The softmax finished reading S_t(j-1) before it
        // signalled p_ready for tile j-1, which this thread consumed.
        tc_fence_after();
        issue_s(j + 1);
      }
      const int j2 = j + 2;
      if (!__all_sync(0xffffffffu,
                      (j2 >= ntiles || mbar_wait(&k_full[j2 % TA_STAGES], (j2 / TA_STAGES) & 1, abort_flag)) &&
                          mbar_wait(&v_full[st], (j / TA_STAGES) & 1, abort_flag) &&
                          mbar_wait(&p_ready[t * 2 + (j & 1)], (j >> 1) & 1, abort_flag)))
        break;
      tc_fence_after();
      const uint32_t vb = smem_u32(sKV + st * TA_STAGE + 2 * TA_KCHUNK);
      const uint32_t d = tmem + 256 + t * 128;
      const uint32_t pa = tmem + t * 128 + (j & 1) * 64;
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < TA_BK / 16; ++ks) {
          const uint64_t db = sdesc_mnmajor_sw128(vb + ks * 2048, TA_KCHUNK);
          mma_f16_ts(d, pa + ks * 8, db, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&pv_done[t]);
        mma_commit(&kv_empty[st]);  // this tile's reads of stage st (S_t(j), P_t(j) V_j) issued
      }
      __syncwarp();
    }
    if (leader) mma_commit(drain);
    __syncwarp();
    mbar_wait_drain(drain, 0);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int query = q0 + t * qpt + (row >> a.lg2G);
    const int head = g * G + (row & (G - 1));
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * 128;
    const float sc = a.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    if constexpr (ta_q_tmem_ksteps<HD>() > 0) {
      // Q_t row `row`, dimensions [0, 64): the first 128-byte chunk of the row in shared memory (128B
      // swizzle: 16-byte unit u of row r sits at unit u ^ (r & 7)), copied as bf16 pairs into the
      // columns after O_t, the layout of a TMEM A operand.
      ok = mbar_wait(q_full, 0, abort_flag);
      if (ok) {
        const uint8_t* qrow = sQ + t * 2 * TA_QCHUNK + row * 128;
        uint32_t qv[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 w = *reinterpret_cast<const uint4*>(qrow + ((u ^ (row & 7)) << 4));
          qv[4 * u] = w.x;
          qv[4 * u + 1] = w.y;
          qv[4 * u + 2] = w.z;
          qv[4 * u + 3] = w.w;
        }
        tmem_st_32x32b_x32(tO + HD, qv);
        tmem_st_wait();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_tm[t]);
    }
    for (int j = 0; ok && j < ntiles; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[t * 2 + b], (j >> 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v[64];
      tmem_ld_32x32b_x32(tS + b * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld_32x32b_x32(tS + b * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      // keys of this tile visible to this row (every range starts at or before the block's first
      // position, so each row sees at least the first key of its range)
      const int valid = query - (kt0 + j) * TA_BK + 1;
      if (valid < TA_BK) {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          if (e >= valid) v[e] = __float_as_uint(-INFINITY);
      }
      // row max: four independent partial maxima (no 64-long dependency chain)
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 64; e += 2)
        mx4[(e >> 1) & 3] = max3f(mx4[(e >> 1) & 3], __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
      const float m_tile = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sc;
      const bool need = m_tile > m_used + TA_RESCALE_THRESHOLD;
      bool prev_pv_waited = false;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t += P_t V of the previous tile must have landed before O_t is rescaled
        if (!mbar_wait(&pv_done[t], (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        prev_pv_waited = true;
        const float alpha = need ? ex2_approx(m_used - m_tile) : 1.f;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + c * 32, o);
        }
        tmem_st_wait();
        l *= alpha;
      }
      if (need) m_used = m_tile;
      uint32_t pk[32];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial row sums (two packed pairs)
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float x0, x1;
        fma2_sc(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]), sc, -m_used, x0, x1);
        // a sixteenth of the exponentials on the FMA pipe, the rest on MUFU
        const bool fma_exp = HD == 96 && (e & TA_FMA_EXP_MASK) == TA_FMA_EXP_MASK;
        const float p0 = fma_exp ? exp2_fma(x0) : ex2_approx(x0);
        const float p1 = fma_exp ? exp2_fma(x1) : ex2_approx(x1);
        add2_acc(ls[2 * (e & 1)], ls[2 * (e & 1) + 1], p0, p1);
        pk[e] = pack_bf16x2(p0, p1);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      if (j == ntiles - 1 && j > 0 && !prev_pv_waited) {
        // pv_done is a parity barrier: a wait is only exact while at most one completion is
        // outstanding.  The epilogue waits for O_t += P_t(last) V; completing the wait for the
        // second-to-last one here (before P_t(last) is handed over, so nothing later can be issued)
        // leaves exactly one outstanding.
        if (!mbar_wait(&pv_done[t], (j - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
      }
      tmem_st_32x32b_x32(tS + b * 64, pk);  // P_t(j) over the S columns just read
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t * 2 + b]);
    }
    const bool fin = ok && mbar_wait(&pv_done[t], (ntiles - 1) & 1, abort_flag);
    if (KSPLIT && fin && nsplit > 1) {
      // one key range of a split block: unnormalised O, the max its exponentials are taken against
      // (log2 units) and the row sum, for attn_split_combine_kernel
      tc_fence_after();
      float* pp = a.part + ((static_cast<size_t>(chunk) * a.rows + qrow0 + (query - q0)) * a.n_q + head) * (HD + 4);
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o32[32];
        tmem_ld_32x32b_x32(tO + c * 32, o32);
        tmem_ld_wait();
        float4* d4 = reinterpret_cast<float4*>(pp + c * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          d4[q] = make_float4(__uint_as_float(o32[4 * q]), __uint_as_float(o32[4 * q + 1]),
                              __uint_as_float(o32[4 * q + 2]), __uint_as_float(o32[4 * q + 3]));
      }
      *reinterpret_cast<float4*>(pp + HD) = make_float4(m_used, l, 0.f, 0.f);
    } else if (fin) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* dst = out + static_cast<size_t>(tok0 + qrow0 + (query - q0)) * a.ld_out + head * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o32[32];
        tmem_ld_32x32b_x32(tO + c * 32, o32);
        tmem_ld_wait();
        uint32_t o[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          o[e] = pack_bf16x2(__uint_as_float(o32[2 * e]) * inv, __uint_as_float(o32[2 * e + 1]) * inv);
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) d4[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0 && *abort_flag && a.err) atomicCAS(a.err, 0, DEV_ERR_TIMEOUT_ATTN_TC);
}

// Merges the key ranges of split query blocks (AttnTcArgs::kchunk): for each (query, head) row,
// M = max_s m_s, O = sum_s 2^(m_s - M) O_s, L = sum_s 2^(m_s - M) l_s, out = bf16(O / L), with the ranges
// taken in order, so the result does not depend on which CTA finished first.  Grid (query block, KV head,
// 8-dimension segment); thread = (query, head) row of the block, which reads one 32-byte sector of each
// range's partial row.  Blocks of one range have nothing to merge.
template <int HD>
__global__ void __launch_bounds__(256) attn_split_combine_kernel(__nv_bfloat16* __restrict__ out, const AttnTcArgs a) {
  pdl_trigger();
  // Every CTA waits for the attention grid, also those with nothing to merge: the next kernel waits only
  // for this grid, and reads the rows the attention kernel wrote directly.
  pdl_wait();
  const int G = 1 << a.lg2G;
  const int qpt = 128 >> a.lg2G;
  const int qb = a.nqb - 1 - static_cast<int>(blockIdx.x);
  const int qrow0 = qb * 2 * qpt;
  const int q0 = sp_pos(a.sp, qrow0);
  const int ntot = (q0 + 2 * qpt - 1) / TA_BK + 1;
  const int nsplit = ta_nsplit(ntot, a.kchunk);
  if (nsplit == 1) return;
  const int c = static_cast<int>(blockIdx.z) * 8;  // first dimension of the segment
  const size_t stride = static_cast<size_t>(a.rows) * a.n_q * (HD + 4);
  for (int p = threadIdx.x; p < 2 * qpt * G; p += blockDim.x) {
    const int row = qrow0 + (p >> a.lg2G);
    const int head = static_cast<int>(blockIdx.y) * G + (p & (G - 1));
    const float* p0 = a.part + (static_cast<size_t>(row) * a.n_q + head) * (HD + 4);
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, p0[s * stride + HD]);
    float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nsplit; ++s) {
      const float* ps = p0 + s * stride;
      const float w = exp2f(ps[HD] - mx);
      L += w * ps[HD + 1];
      const float4 v0 = *reinterpret_cast<const float4*>(ps + c);
      const float4 v1 = *reinterpret_cast<const float4*>(ps + c + 4);
      o[0] += w * v0.x; o[1] += w * v0.y; o[2] += w * v0.z; o[3] += w * v0.w;
      o[4] += w * v1.x; o[5] += w * v1.y; o[6] += w * v1.z; o[7] += w * v1.w;
    }
    const float inv = 1.f / L;
    uint4 pk;
    pk.x = pack_bf16x2(o[0] * inv, o[1] * inv);
    pk.y = pack_bf16x2(o[2] * inv, o[3] * inv);
    pk.z = pack_bf16x2(o[4] * inv, o[5] * inv);
    pk.w = pack_bf16x2(o[6] * inv, o[7] * inv);
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * a.ld_out + head * HD + c) = pk;
  }
}

}  // namespace mk
