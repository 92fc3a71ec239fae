/*
 * minicpm5_mk -- C ABI of the B200 (sm_100a) MiniCPM5 prefill-score path.
 *
 * The reference reaches its device program through one op,
 *   jax_op("minicpm5_mk::forward", mk_jax.mk_forward)          plugin/minicpm5_mk/model.py:57-66
 * called from MiniCPM5MegakernelForCausalLM._mk_call            plugin/minicpm5_mk/model.py:737-753
 * with (ids, embed, cos, sin, final_norm, 16 weight stacks, bs, seq, quant, n_q, n_kv, head_dim,
 * eps, attn) and returning (max(8, bs), H) bf16 final-normed last-token hidden rows
 * (plugin/minicpm5_mk/mk_jax.py:624-665).  This library replaces that op.  The weights are bound
 * once (mk_bind_weights, the counterpart of the `_mk_build` device copy, model.py:623-698) and
 * each forward passes only the ids, a caller-owned workspace and the outputs.
 *
 * Conventions
 *   - Plain C types only; every device buffer is owned by the caller (e.g. the torch caching
 *     allocator).  The library owns the handle and its host-side descriptors.
 *   - No exceptions cross the ABI: every call returns an mk_status.
 *   - All launches are asynchronous on the given stream; no call synchronises the host except
 *     mk_get_error (which reads the device error word).
 *   - One handle per device; calls on one handle are serialised by the caller.
 *   - bf16 = IEEE bfloat16 stored as uint16_t; "stream" is a cudaStream_t passed as void*.
 */
#ifndef MINICPM5_MK_H_
#define MINICPM5_MK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mk_status {
  MK_OK = 0,
  MK_ERR_BAD_SHAPE = 1,      /* unsupported or inconsistent sizes (e.g. seq % 128, head_dim not 96/128) */
  MK_ERR_BAD_ALIGN = 2,      /* a pointer is not 16-byte aligned */
  MK_ERR_CUDA = 3,           /* a CUDA runtime / driver call failed */
  MK_ERR_DEVICE_TIMEOUT = 4, /* a kernel gave up a bounded wait (see mk_get_error) */
  MK_ERR_BAD_ARG = 5,        /* null handle / pointer, bad enum value */
  MK_ERR_NOT_BOUND = 6,      /* mk_forward before mk_bind_weights */
  MK_ERR_BAD_TOKEN = 7,      /* a token id outside [0, vocab) was seen */
  MK_ERR_WORKSPACE = 8,      /* workspace smaller than mk_workspace_size */
  MK_ERR_TOO_LARGE = 9       /* request exceeds a fixed capacity of the library (see the entry point) */
} mk_status;

/* Model configuration: plugin/minicpm5_mk/model.py:561-567 plus the MiniCPM muP scalars.
 *   x = scale_emb * embed[ids];  x += residual_scale * branch;  logits = logit_scale * h @ lm_head^T
 * weight_bits: format of the projection weights -- 8 (or 0): int8 weight-only, per-output-channel f32
 * scales (the reference's `_quantize_w`, plugin/minicpm5_mk/mk_weights.py:113-123); 16: bf16 weights,
 * unquantised (the scales are then 1.0). */
typedef struct mk_config {
  int32_t num_layers, hidden, inter, n_q, n_kv, head_dim, vocab, max_seq;
  float eps, rope_theta, scale_emb, residual_scale, logit_scale;
  int32_t weight_bits;
} mk_config;

/* Device pointers of the prepared weights (layout written by minicpm5_mk/mk_weights.py):
 *   embed, lm_head : bf16 [vocab, hidden]
 *   final_norm     : f32  [hidden]
 *   rope_cos/sin   : f32  [max_seq, head_dim/2]
 *   w_qkv  W [L, (n_q+2 n_kv) head_dim, hidden]   s_qkv  f32 [L, (n_q+2 n_kv) head_dim]
 *   w_o    W [L, hidden, n_q head_dim]            s_o    f32 [L, hidden]
 *   w_gu   W [L, 2 inter, hidden] (gate/up rows alternating: row 2i gate i, row 2i+1 up i)
 *                                                 s_gu   f32 [L, 2 inter]
 *   w_down W [L, hidden, inter]                   s_down f32 [L, hidden]
 * W is int8 or bf16 as mk_config.weight_bits says.  The Q rows carry 1/sqrt(head_dim); RMSNorm gains
 * are folded into the weight columns. */
typedef struct mk_weight_ptrs {
  const void* embed;
  const void* lm_head;
  const float* final_norm;
  const float* rope_cos;
  const float* rope_sin;
  const void* w_qkv;
  const float* s_qkv;
  const void* w_o;
  const float* s_o;
  const void* w_gu;
  const float* s_gu;
  const void* w_down;
  const float* s_down;
} mk_weight_ptrs;

typedef struct mk_handle mk_handle;

/* Human-readable name of a status code (static string). */
const char* mk_status_string(mk_status s);

/* Library version (major * 10000 + minor * 100 + patch). */
int32_t mk_version(void);

/* Create a handle on `device` (the CUDA device ordinal).  Replaces the op creation in
 * plugin/minicpm5_mk/model.py:57-66 (`_get_op`). */
mk_status mk_create(const mk_config* cfg, int32_t device, mk_handle** out);

/* Bind the prepared weights (device pointers stay owned by the caller and must outlive the
 * handle's use).  Builds the TMA descriptors of the weight stacks.  Counterpart of the device
 * copy in `_mk_build` (plugin/minicpm5_mk/model.py:623-698). */
mk_status mk_bind_weights(mk_handle* h, const mk_weight_ptrs* w);

/* Bytes of workspace mk_forward needs for (bs, seq). */
mk_status mk_workspace_size(const mk_handle* h, int32_t bs, int32_t seq, size_t* bytes);

/* Whole-model prefill-score forward of `bs` equal-length sequences of length `seq`
 * (replaces mk_forward, plugin/minicpm5_mk/mk_jax.py:624-665, and vLLM's lm_head + greedy sampler
 * for those rows).
 *   d_ids       int32 [bs * seq], sequence-major
 *   d_workspace >= mk_workspace_size bytes, 256-byte aligned
 *   d_hidden    optional bf16 [bs, hidden]: final-normed last-token hidden rows (the reference op's output)
 *   d_logits    optional f32 [bs, vocab]: last-token logits (logit_scale applied)
 *   d_top1      optional int32 [bs]: greedy token (argmax of the logits, ties -> lowest id)
 * seq must be a multiple of 128 and <= max_seq; bs >= 1. */
mk_status mk_forward(mk_handle* h, const int32_t* d_ids, int32_t bs, int32_t seq, void* d_workspace,
                     size_t workspace_bytes, void* d_hidden, float* d_logits, int32_t* d_top1, void* stream);

/* Number of kernel launches one mk_forward(bs, seq) issues (for launch accounting). */
int32_t mk_launches_per_forward(const mk_handle* h, int32_t bs, int32_t seq);

/* Per-stage device time of one forward, measured with CUDA events recorded on `stream` between
 * the launches (the interval after a launch runs up to the next launch's start, so gaps are
 * charged to the stage before them).  Index by mk_stage. */
typedef enum mk_stage {
  MK_STAGE_EMBED = 0,      /* embedding gather (+ row sums of squares) */
  MK_STAGE_QKV = 1,        /* QKV projection with RMSNorm and RoPE, layers 0..L-2 */
  MK_STAGE_ATTN = 2,       /* causal prefill attention, layers 0..L-2 */
  MK_STAGE_O = 3,          /* o_proj with the residual update */
  MK_STAGE_GATE_UP = 4,    /* gate/up projection with SiLU * up */
  MK_STAGE_DOWN = 5,       /* down projection with the residual update */
  MK_STAGE_LAST_LAYER = 6, /* the last layer (K/V for every position, the rest for the last one) */
  MK_STAGE_HEAD = 7,       /* final norm, lm_head and argmax */
  MK_STAGE_KV_GATHER = 8,  /* sequence parallel: K/V packing and the caller's all-gather, every layer */
  MK_STAGES = 9
} mk_stage;

typedef struct mk_stage_times {
  float ms[MK_STAGES];         /* summed device milliseconds per stage */
  int32_t launches[MK_STAGES]; /* kernel launches per stage */
} mk_stage_times;

/* mk_forward with per-stage timing: the same launches on the same stream, with CUDA events
 * between them.  Synchronises the stream before returning and fills *times. */
mk_status mk_forward_timed(mk_handle* h, const int32_t* d_ids, int32_t bs, int32_t seq, void* d_workspace,
                           size_t workspace_bytes, void* d_hidden, float* d_logits, int32_t* d_top1, void* stream,
                           mk_stage_times* times);

/* ---------------------------------------------------------------- sequence parallelism
 * One sequence over `world` GPUs, one rank (process) per GPU (counterpart of `core_forward_sp`,
 * plugin/minicpm5_mk/mk_jax.py:440-489, generalised from 2 TensorCores to `world` GPUs).  The
 * sequence is cut into zig-zag blocks: in every group of 2 * world blocks, rank r owns block r and
 * block 2 * world - 1 - r (`sp_global_block`, plugin/minicpm5_mk/mk_attn.py:721-724).  Each rank runs
 * the projections and MLPs on its own rows and attention for its own queries.  Once per layer the
 * ranks all-gather their K/V rows (rank by rank) through the caller's collective.
 *
 * The all-gather callback is issued on `stream`, in the same order on every rank: it gathers
 * `bytes_per_rank` bytes from `d_send` of every rank into `d_recv` (rank r's bytes at offset
 * r * bytes_per_rank), ordered after the work already on the stream and before the work issued
 * after it returns (an NCCL all-gather on that stream does this).  It returns 0 on success. */
typedef int32_t (*mk_allgather_fn)(void* ctx, const void* d_send, void* d_recv, size_t bytes_per_rank, void* stream);

/* Zig-zag block length in tokens for (seq, world), 0 if the shape cannot be split: the largest of
 * 512, 256, 128, 64 with seq % (2 * world * blk) == 0 that holds whole attention query blocks. */
int32_t mk_sp_block(const mk_handle* h, int32_t seq, int32_t world);

/* Whether mk_forward_sp cuts the long causal key ranges of a rank's attention over several CTAs
 * (enabled by default).  A rank owns few query blocks and their key ranges are very unequal (at 8 ranks
 * one CTA would walk all of an 8192-token sequence's keys while the average SM has a fifth of that), so
 * when a replay of the grid's dispatch says it pays, ranges are cut into near-equal parts whose partial
 * results (unnormalised output, running max, row sum) a second kernel merges in a fixed order.  The merge
 * rounds differently from a single pass, so with a split the logits agree with mk_forward to float
 * rounding (the same greedy id in the tests) rather than bit for bit; disabled, mk_forward_sp is
 * bit-identical to mk_forward.  Set it before mk_workspace_size_sp: the split keeps its partial results
 * in the workspace.  No counterpart in the reference (its sequence parallelism spans the two
 * TensorCores of one chip). */
mk_status mk_set_sp_key_split(mk_handle* h, int32_t enabled);

/* Bytes of workspace mk_forward_sp needs on each rank. */
mk_status mk_workspace_size_sp(const mk_handle* h, int32_t seq, int32_t world, size_t* bytes);

/* Sequence-parallel prefill-score forward of one sequence of `seq` tokens.
 *   d_ids   int32 [seq], the whole sequence, on every rank
 *   d_hidden / d_logits / d_top1 as in mk_forward (bs = 1); written on rank 0 only, which owns the
 *           last position
 *   times   optional per-stage device times (as mk_forward_timed; synchronises the stream)
 * Returns MK_ERR_BAD_ARG for a bad rank / world or a null callback, MK_ERR_BAD_SHAPE when
 * mk_sp_block is 0, MK_ERR_CUDA when the callback fails. */
mk_status mk_forward_sp(mk_handle* h, const int32_t* d_ids, int32_t seq, int32_t rank, int32_t world,
                        mk_allgather_fn allgather, void* allgather_ctx, void* d_workspace, size_t workspace_bytes,
                        void* d_hidden, float* d_logits, int32_t* d_top1, void* stream, mk_stage_times* times);

/* Read and clear the library's device error word (synchronises the device).  *device_err
 * receives the raw code (0 = none); the return value maps it to an mk_status. */
mk_status mk_get_error(mk_handle* h, int32_t* device_err);

void mk_destroy(mk_handle* h);

/* ---------------------------------------------------------------- isolated kernels
 * The per-stage kernels of the forward, exposed for parity tests and the isolated-kernel
 * benchmarks.  They use the current device and build their descriptors per call. */

/* GEMM epilogue modes. */
typedef enum mk_gemm_mode {
  MK_GEMM_ROWSCALE = 0, /* out = bf16(acc * row_scale[m] * col_scale[n])                     */
  MK_GEMM_RESID = 1,    /* out = bf16(out + resid_scale * acc * col_scale[n])   (in place)   */
  MK_GEMM_SWIGLU = 2,   /* out[m, i] = bf16(silu(g_i) * u_i), rows 2i / 2i+1 = gate / up; out width N/2 */
  MK_GEMM_COLSCALE = 3, /* out = bf16(acc * col_scale[n])                                    */
  MK_GEMM_RESID32 = 4   /* resid32 += resid_scale * acc * col_scale[n] (f32, in place); out = bf16(resid32) */
} mk_gemm_mode;

/* W8A16 GEMM: acc[m, n] = sum_k a[m, k] * w[n, k]; a bf16 [M, lda], w int8 [N, K].
 * N % 128 == 0, K % 64 == 0, lda % 8 == 0, ldo % 8 == 0.
 * resid32 (f32 [M, ld_resid32], RESID32 mode only, else NULL) is the f32 residual stream.
 * Replaces `fused_qkv` (plugin/minicpm5_mk/mk_mlp.py:161-206), `linear` (mk_jax.py:233-269) and the
 * gate/up half of `fused_mlp` (mk_mlp.py:68-145). */
mk_status mk_gemm_w8a16(const void* a, int32_t M, int32_t K, int32_t lda, const int8_t* w, const float* col_scale,
                        int32_t N, int32_t mode, const float* row_scale, float resid_scale, void* out, int32_t ldo,
                        float* resid32, int32_t ld_resid32, void* stream);

/* Fused epilogue work of one W8A16 GEMM launch, as the forward's projections use it.  Zero / NULL fields
 * switch a part off.
 *   rowsq     f32 [M, rowsq_ld]: per-(token, 128-channel tile) sums of squares of the f32 residual.
 *             ROWSCALE / SWIGLU with rowsq_np > 0 read them: rstd[m] = 1/sqrt(sum of the first rowsq_np
 *             entries of row m / norm_dim + eps) replaces row_scale (the fused RMSNorm of `fused_qkv`,
 *             plugin/minicpm5_mk/mk_mlp.py:161-206, `rms_norm_unit`, mk_jax.py:32-36).
 *             RESID32 writes them: rowsq[m * rowsq_ld + n / 128] = sum over the tile's 128 channels of the
 *             updated residual squared (rowsq_ld >= N / 128).
 *   rope_*    ROWSCALE only: columns [0, rope_cols) are heads of head_dim columns whose rotation pairs
 *             (i, i + head_dim/2) are stored as adjacent columns (2j, 2j + 1); each pair is rotated by the
 *             angle of position rope_pos_base + m % rope_seq (tables f32 [*, head_dim/2]) before the bf16
 *             rounding (RoPE of plugin/minicpm5_mk/mk_attn.py:572-589).  rope_cols % 32 == 0. */
typedef struct mk_gemm_fusion {
  float* rowsq;
  int32_t rowsq_ld, rowsq_np, norm_dim;
  float eps;
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_cols, head_dim, rope_seq, rope_pos_base;
  int32_t weight_bits; /* 8 (or 0): w is int8; 16: w is bf16 [N, K] */
} mk_gemm_fusion;

/* mk_gemm_w8a16 with the fused epilogue work above (fusion may be NULL: then it is mk_gemm_w8a16;
 * row_scale may be NULL when rowsq_np > 0). */
mk_status mk_gemm_w8a16_fused(const void* a, int32_t M, int32_t K, int32_t lda, const void* w,
                              const float* col_scale, int32_t N, int32_t mode, const float* row_scale,
                              float resid_scale, void* out, int32_t ldo, float* resid32, int32_t ld_resid32,
                              const mk_gemm_fusion* fusion, void* stream);

/* Causal GQA prefill attention over bs sequences of length seq.  qkv bf16 [bs*seq, ld_qkv] with
 * Q heads at column q_col, K at k_col, V at v_col (each head head_dim wide); out bf16
 * [bs*seq, ld_out] (head h at column h*head_dim).  Scores are multiplied by `softmax_scale`
 * (1.0 when Q already carries 1/sqrt(head_dim)).  n_q / n_kv must be 1, 2, 4 or 8.
 * Replaces `super_gqa_v2` (plugin/minicpm5_mk/mk_attn.py:557-710). */
mk_status mk_attention_prefill(const void* qkv, int32_t bs, int32_t seq, int32_t n_q, int32_t n_kv,
                               int32_t head_dim, int32_t ld_qkv, int32_t q_col, int32_t k_col, int32_t v_col,
                               float softmax_scale, void* out, int32_t ld_out, void* stream);

/* In-place RoPE on n_heads heads starting at column col0 of each of `rows` rows (row r at position
 * pos_base + r % seq).  Tables f32 [*, head_dim/2].  (RoPE of plugin/minicpm5_mk/mk_attn.py:572-589,
 * math of benchmark/f32_golden.py:57-59,88-89.) */
mk_status mk_rope(void* x, int32_t rows, int32_t ld, int32_t col0, int32_t n_heads, int32_t head_dim,
                  const float* rope_cos, const float* rope_sin, int32_t seq, int32_t pos_base, void* stream);

/* rstd[t] = 1/sqrt(mean(x[t, :H]^2) + eps) for the f32 residual stream x [T, ld]
 * (`rms_norm_unit`, plugin/minicpm5_mk/mk_jax.py:32-36). */
mk_status mk_rms_rstd(const float* x, int32_t T, int32_t H, int32_t ld, float eps, float* rstd, void* stream);

/* x32[t] = scale * embed[ids[t]] (f32) and xb[t] = bf16(x32[t])  (plugin/minicpm5_mk/mk_jax.py:532). */
mk_status mk_embed(const int32_t* ids, int32_t T, const void* embed, int32_t V, int32_t H, float scale, float* x32,
                   void* xb, void* stream);

/* Top-k log-probabilities of each row of f32 logits [bs, ld] (first V entries):
 * logprobs[b, r] = logits[b, ids[b, r]] - logsumexp(logits[b, :V]) for the k largest logits in
 * descending order (equal logits: lower id first).  ids int32 [bs, k], logprobs f32 [bs, k];
 * 1 <= k <= 64.  Replaces the golden's log_softmax + top-k (benchmark/f32_golden.py:100-102) that the
 * reference's gate scorer compares (benchmark/gate.py:16-121). */
mk_status mk_topk_logprobs(const float* logits, int32_t bs, int32_t V, int32_t ld, int32_t k, int32_t* ids,
                           float* logprobs, void* stream);

/* logits[b] = h[b] @ lm_head^T (f32), top1[b] = argmax (ties -> lowest id) for h f32 [bs, H].
 * part_val/part_idx: scratch of bs * mk_lm_head_parts() entries each.
 * (vLLM LogitsProcessor + greedy sampler after the reference op.) */
int32_t mk_lm_head_parts(void);
mk_status mk_lm_head_argmax(const float* h, int32_t bs, int32_t H, const void* lm_head, int32_t V, float* logits,
                            float* part_val, int32_t* part_idx, int32_t* top1, void* stream);

/* ---------------------------------------------------------------- allocation-free variant
 * No counterpart in the reference.  Same computation and results as mk_lm_head_argmax, for callers
 * that cannot allocate device memory at call time -- for example a serving engine that has already
 * reserved almost all of the GPU for weights and its KV cache, or a host runtime calling through a
 * thin FFI without access to the framework's caching allocator, where a cudaMalloc / cudaFree pair per
 * call could fail or stall every stream on the device.  The caller passes only the inputs and the
 * outputs; the per-block argmax partials live in a fixed array inside the library.
 *   - At most MK_LM_HEAD_NOALLOC_MAX_ROWS rows per call; larger bs returns MK_ERR_TOO_LARGE.
 *   - The array (about 148 KiB) exists on every GPU that loads the library, until process exit.
 *   - The first call on a device looks up the array's device address (with that device current);
 *     make that first call before any stream capture on the device.
 *   - Nothing in the array needs to start at zero: every slot a call reads was written earlier in
 *     the same call.  Calls share the array, so calls that overlap on the GPU (different streams, or
 *     different host threads on one device) race; serialise them on one stream.
 *   - Calls no cudaMalloc, cudaFree or allocating library routine. */
#define MK_LM_HEAD_NOALLOC_MAX_ROWS 64
mk_status mk_lm_head_argmax_noalloc(const float* h, int32_t bs, int32_t H, const void* lm_head, int32_t V,
                                    float* logits, int32_t* top1, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINICPM5_MK_H_ */
