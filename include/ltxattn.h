/*
 * ltxattn.h -- C ABI of libltxattn_cuda, the B200 (sm_100a) fused attention of
 * the LTX 2.5 diffusion transformer.
 *
 * This is the drop-in boundary behind the reference's attention seam.  In
 * loading-awesome/LTX-2.5-Swift the seam is `Sources/LTXAttention`
 * (`AttentionBackend.swift:13-15`, an empty placeholder) and the attention
 * core it stands in for is the SDPA switch of
 * `Sources/LTXModules/DiTAttention.swift:369-382`, together with the split
 * RoPE applied just before it (`:364-367`, `:206-234`).  A Swift caller binds
 * this header through a SwiftPM system-library target whose module map names
 * it (ltx-2.5-swift_b200/swift/CLTXAttnCUDA/module.modulemap).
 *
 * Conventions
 *  - Plain pointers and sizes only.  Device pointers are CUDA device memory;
 *    `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Tensors are [B, H, T, D] views with element strides for B, H and T; the
 *    D stride is 1.  The reference's `split` (`DiTAttention.swift:346-348`)
 *    is a transposed view of [B, T, H*D]: strides (T*H*D, D, H*D).  It is
 *    accepted as is, with no copy.
 *  - The caller owns every buffer, including outputs, the log-sum-exp and the
 *    workspace.  The library allocates no device memory per call.
 *  - Calls are asynchronous with respect to the host and ordered on `stream`.
 *    They are re-entrant; distinct host threads may use distinct streams.
 *  - No exception crosses the ABI.  Every entry returns an ltxattn_status;
 *    ltxattn_last_error() gives this thread's message for the last failure.
 *  - There is no CPU fallback.  A shape the kernels do not cover returns
 *    LTXATTN_ERR_UNSUPPORTED (the reference's own warning against a silent
 *    fallback is at `DiTAttention.swift:284-287`).
 */
#ifndef LTXATTN_H
#define LTXATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LTXATTN_ABI_VERSION 3

/* Entry points are the only symbols the library exports. */
#if defined(__GNUC__)
#define LTXATTN_API __attribute__((visibility("default")))
#else
#define LTXATTN_API
#endif

typedef enum ltxattn_status {
  LTXATTN_OK = 0,
  LTXATTN_ERR_SHAPE = 1,       /* sizes disagree; mirrors DiTAttention.Failure.shape (:109) */
  LTXATTN_ERR_DTYPE = 2,       /* dtype not F32 / BF16 */
  LTXATTN_ERR_ALIGN = 3,       /* pointer or stride not 16-byte aligned where TMA needs it */
  LTXATTN_ERR_UNSUPPORTED = 4, /* head_dim or size outside what the kernels cover */
  LTXATTN_ERR_CUDA = 5,        /* a CUDA runtime call failed */
  LTXATTN_ERR_NCCL = 6,        /* an NCCL call failed or NCCL is not loadable */
  LTXATTN_ERR_TIMEOUT = 7,     /* a device-side bounded wait gave up */
  LTXATTN_ERR_WORKSPACE = 8,   /* workspace missing or smaller than required */
  LTXATTN_ERR_ARG = 9          /* NULL where a pointer is required, bad enum, bad range */
} ltxattn_status;

typedef enum ltxattn_dtype {
  LTXATTN_F32 = 0,  /* float32: the `.explicit` arm's arithmetic, parity gate */
  LTXATTN_BF16 = 1  /* bfloat16 storage, fp32 accumulation: the render/training dtype */
} ltxattn_dtype;

/* A [B, H, T, D] view.  Strides are in elements; the D stride is 1. */
typedef struct ltxattn_tensor {
  void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
} ltxattn_tensor;

/* One split-RoPE table pair, DiTAttention.Rotary (`DiTAttention.swift:98-105`):
 * cos and sin are [B, H, T, D/2] in the activation dtype (the reference narrows
 * them to x.dtype before use, `:231-232`).  A zero stride_b / stride_h shares
 * the table across batch / heads.  `tokens` is how many rows the table holds.
 * cos == NULL means "no rotary". */
typedef struct ltxattn_rotary {
  const void* cos;
  const void* sin;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
  int32_t tokens;
} ltxattn_rotary;

/* Forward arguments: out = softmax(scale * rope(q) rope(k)^T + mask) v.
 *
 *  - heads [head_begin, head_begin + head_count) are computed (head_count 0 =
 *    all heads); the views cover all `heads`.  This is how a rank of a
 *    head-sharded job runs its block of a shared tensor.
 *  - key_mask: [B, kv_len] uint8, nonzero = valid, or NULL.  Masked keys get
 *    exactly zero weight; a batch row with no valid key attends to every key
 *    unmasked, the rule of `GemmaTextEncoder.swift:306-319`.
 *  - q_rotary rotates q; k_rotary rotates k; k_rotary.cos == NULL with
 *    q_rotary given rotates k with the q table (`keyRotary ?? rotary`,
 *    `DiTAttention.swift:366`).  k_rotary without q_rotary is ignored, as in
 *    the reference (`:364`).
 *  - lse: [B, H, q_len] float32, natural-log log-sum-exp of the scaled
 *    logits, or NULL.  The backward needs it.
 *  - workspace: device scratch of ltxattn_fwd_workspace() bytes (may be 0).
 *  - num_splits: 0 = choose: short query sequences split every 256-row
 *    query block's KV range across CTAs, and dense calls whose last wave of
 *    blocks would leave most SMs idle split only those last blocks; n > 0
 *    splits every block n ways.  The choice changes only the summation order.
 *  - causal, window, kv_heads: the Gemma text encoder's self-attention
 *    (`GemmaTextEncoder.swift:218-233,292-323`); all zero for the DiT.  causal
 *    (requires q_len == kv_len): query i attends key j only if j <= i; window
 *    > 0: also i - j < window (a sliding layer).  A query row these rules and
 *    key_mask leave without keys attends every key instead (the reference's
 *    un-masking of fully masked rows).  kv_heads (0 = heads) must divide heads:
 *    k and v are [B, kv_heads, kv_len, D] and query head h reads kv head
 *    h / (heads / kv_heads); grouped heads take no rotary (rotate before).
 *  - gate: the per-head output gate of `DiTAttention.swift:395-399`, fused
 *    into the store of out: the `to_gate_logits` output [B, q_len, heads] in
 *    the activation dtype T (element strides gate_stride_b / _t / _h; any
 *    layout), or NULL.  out = T(T(O) * g), g = 2 * T(sigmoid(float(logit)))
 *    per query row and head (the sigmoid in fp32 and cast back, `:240-242`;
 *    the doubling is exact).  lse is not gated.  The backward wants the
 *    un-gated out, so a training forward keeps gate NULL and gates outside. */
typedef struct ltxattn_fwd_args {
  int32_t dtype;
  int32_t batch, heads, q_len, kv_len, head_dim;
  int32_t head_begin, head_count;
  ltxattn_tensor q, k, v, out;
  float scale;
  const uint8_t* key_mask;
  int64_t key_mask_stride_b;
  ltxattn_rotary q_rotary, k_rotary;
  float* lse;
  int64_t lse_stride_b, lse_stride_h;
  void* workspace;
  size_t workspace_bytes;
  int32_t num_splits;
  int32_t causal;
  int32_t window;
  int32_t kv_heads;
  /* ABI 3 */
  const void* gate;
  int64_t gate_stride_b, gate_stride_t, gate_stride_h;
} ltxattn_fwd_args;

/* Backward arguments: gradients of sum(dout * out) with respect to q, k and v
 * (the un-rotated inputs when rotaries are given; the bf16 roundings inside
 * RoPE pass gradients straight through, as autodiff does).  P is recomputed
 * from the forward's saved `lse`; no score matrix is stored.  This replaces
 * MLX's VJP of the fused SDPA under gradient checkpointing
 * (`LoRATrainingStep.swift:283-304`, `GradientCheckpoint.swift:48-67`). */
typedef struct ltxattn_bwd_args {
  int32_t dtype;
  int32_t batch, heads, q_len, kv_len, head_dim;
  int32_t head_begin, head_count;
  ltxattn_tensor q, k, v, out, dout;
  const float* lse;
  int64_t lse_stride_b, lse_stride_h;
  ltxattn_tensor dq, dk, dv;
  float scale;
  const uint8_t* key_mask;
  int64_t key_mask_stride_b;
  ltxattn_rotary q_rotary, k_rotary;
  void* workspace;
  size_t workspace_bytes;
} ltxattn_bwd_args;

/* Replaces `MLXFast.scaledDotProductAttention(queries:keys:values:scale:mask:)`
 * and the `.explicit` arm (`DiTAttention.swift:373-382`), fused with the RoPE
 * of `:364-367`. */
LTXATTN_API int ltxattn_fwd(const ltxattn_fwd_args* args, void* stream);

/* Device scratch bytes ltxattn_fwd needs for these arguments. */
LTXATTN_API size_t ltxattn_fwd_workspace(const ltxattn_fwd_args* args);

/* What ltxattn_fwd will launch for these arguments (introspection for
 * benchmarks and logs; no counterpart in the reference). */
typedef struct ltxattn_fwd_plan_info {
  int32_t kernel;       /* 0: fp32 path; 1: tiled bf16 forward (one CTA per unit); 2: persistent bf16
                           forward for kv_len <= 128; 3: persistent bf16 forward over whole units
                           (no causal or window band, at least one wave of units) */
  int32_t splits;       /* KV splits of the split units (1: none) */
  int64_t units;        /* 256-row query blocks x heads x batch (bf16) or 128-row blocks (fp32) */
  int64_t split_units;  /* how many of them run split */
  int32_t launches;     /* kernel launches of one call: RoPE pre-pass + attention + combine */
} ltxattn_fwd_plan_info;
LTXATTN_API int ltxattn_fwd_plan(const ltxattn_fwd_args* args, ltxattn_fwd_plan_info* info);

/* ltxattn_fwd for callers that cannot allocate device memory -- for example a
 * host whose device memory is owned by another framework's allocator, or a
 * render loop that must not allocate between steps.  No counterpart in the
 * reference.  args->workspace is ignored: scratch comes from a fixed 32 MiB
 * device array inside the library (held on every GPU that loads it until
 * exit), and arguments needing more (ltxattn_fwd_workspace) are refused with
 * LTXATTN_ERR_WORKSPACE.  Allocates nothing.  The first call on a device
 * looks the array up for that device; make it before any stream capture.
 * All calls share the array, so calls that overlap on the GPU race: keep them
 * ordered (one stream, or explicit events). */
LTXATTN_API int ltxattn_fwd_noalloc(const ltxattn_fwd_args* args, void* stream);

/* ---- head-sharded forward with the all-gather fused into its epilogue ---- */

/* Every rank's full output tensor and signal words, mapped on the calling
 * device (CUDA IPC over NVLink).  signals[d] is rank d's array of 16 uint32
 * words, zero at allocation: [0, 8) count the output tiles that arrived from
 * each source rank, [8, 16) hold the last call each rank has entered. */
typedef struct ltxattn_gather_peers {
  int32_t world;          /* ranks, 2 to 8 */
  int32_t rank;           /* this rank */
  void* out[8];           /* rank d's output [B, H, T, D] (out[rank] == args->out.data) */
  uint32_t* signals[8];   /* rank d's 16 signal words */
  uint32_t epoch;         /* 1, 2, 3, ...: one per call, the same on every rank */
  int32_t reserved;
} ltxattn_gather_peers;

/* ltxattn_fwd of this rank's head block (args->head_begin / head_count; every
 * rank passes the same shape and head_count), whose epilogue also stores each
 * output tile into every other rank's output with peer stores over NVLink, so
 * the all-gather overlaps the attention tile by tile (the head-parallel
 * counterpart of the call followed by ltxattn_allgather_heads; no counterpart in
 * the reference, which runs one device).  Stream-ordered: the work queued after
 * it sees every rank's heads in args->out.  Before storing into the peers'
 * outputs the call waits until every rank has entered the same epoch (so a
 * rank's earlier work on its output has completed); every cross-device wait is
 * bounded and reports LTXATTN_ERR_TIMEOUT through ltxattn_device_status.  bf16
 * only; the call runs the tiled kernel (KV splits as planned, their combine
 * storing to the peers too; a call planned for a persistent kernel runs tiled
 * and unsplit); the output must be 16-byte aligned with strides that are
 * multiples of 8 elements; not for stream capture (the epoch is a launch
 * argument). */
LTXATTN_API int ltxattn_fwd_gather(const ltxattn_fwd_args* args, const ltxattn_gather_peers* peers, void* stream);

/* Replaces the autodiff VJP of the SDPA core (LoRA training backward). */
LTXATTN_API int ltxattn_bwd(const ltxattn_bwd_args* args, void* stream);

/* Device scratch bytes ltxattn_bwd needs for these arguments. */
LTXATTN_API size_t ltxattn_bwd_workspace(const ltxattn_bwd_args* args);

/* ---- projections ---------------------------------------------------------- */

/* Arguments of ltxattn_linear: out = T(T(x W^T) + bias), the bf16 matmul (fp32
 * accumulation, one rounding) and then the bias added in bf16.
 *  - x [m, k] rows of x_stride elements; weight [n, k] (the checkpoint's
 *    [out, in] layout) rows of weight_stride; out [m, n] rows of out_stride.
 *  - bias [n] or NULL.
 *  - n a multiple of 8, k of 64; rows 16-byte aligned.
 *  - workspace: NULL, or device scratch of ltxattn_linear_workspace() bytes
 *    (256-byte aligned).  That size is non-zero for a narrow output whose
 *    column tiles would leave most SMs idle (the gate logits: 32 columns);
 *    with the workspace such a call splits K across CTAs into fp32 partials
 *    and adds them in a fixed order before the bias and the roundings (the
 *    same function; only the fp32 summation order differs). */
typedef struct ltxattn_linear_args {
  int32_t dtype; /* LTXATTN_BF16 */
  int32_t m, n, k;
  const void* x;
  int64_t x_stride;
  const void* weight;
  int64_t weight_stride;
  const void* bias;
  void* out;
  int64_t out_stride;
  void* workspace;
  size_t workspace_bytes;
} ltxattn_linear_args;

/* Replaces `DiTAttention.linear` (`DiTAttention.swift:178-188`) without the LoRA
 * overlay: to_q, to_k, to_v, to_out.0 and to_gate_logits of the attention module
 * (q and k then take ltxattn_qk_prep for the norm, the head split and RoPE). */
LTXATTN_API int ltxattn_linear(const ltxattn_linear_args* args, void* stream);

/* Device scratch bytes ltxattn_linear can use for these arguments (0: none). */
LTXATTN_API size_t ltxattn_linear_workspace(const ltxattn_linear_args* args);

/* Arguments of ltxattn_head_gate: out = T(T(x) * g) per head, g = 2 * T(sigmoid(logit)).
 *  - x, out: [B, H, T, D] views (out may view the merged [B, T, H * D] buffer).
 *  - gate: the to_gate_logits output [B, T, H] (element strides), or NULL for a
 *    plain copy (the merge alone).  head_dim a multiple of 8. */
typedef struct ltxattn_head_gate_args {
  int32_t dtype;
  int32_t batch, heads, tokens, head_dim;
  ltxattn_tensor x, out;
  const void* gate;
  int64_t gate_stride_b, gate_stride_t, gate_stride_h;
} ltxattn_head_gate_args;

/* Replaces the per-head gate and merge (`DiTAttention.swift:395-403`) for the
 * STG passthrough (`:349-356`), whose output is the value stream rather than an
 * attention output (ltxattn_fwd applies the same gate in its own store). */
LTXATTN_API int ltxattn_head_gate(const ltxattn_head_gate_args* args, void* stream);

/* ---- split RoPE on its own ------------------------------------------------ */

/* Arguments of ltxattn_rope: out = split-RoPE(x, rotary).
 *  - dtype, batch, heads, tokens, head_dim: the shape of x and out.
 *  - x, out: [B, H, T, D] views; out may be x itself (in place) but must not
 *    otherwise overlap it.
 *  - rotary: the table pair, [1|B, 1|H, >= tokens, D/2] in the activation dtype. */
typedef struct ltxattn_rope_args {
  int32_t dtype;
  int32_t batch;
  int32_t heads;
  int32_t tokens;
  int32_t head_dim;
  ltxattn_tensor x;
  ltxattn_tensor out;
  ltxattn_rotary rotary;
} ltxattn_rope_args;

/* Replaces `applySplitRoPE` (`DiTAttention.swift:206-234`) for a caller that
 * rotates a tensor outside the attention call (ltxattn_fwd rotates q and k
 * itself).  bf16: every product and every sum rounds to bf16, as for a bf16
 * MLX tensor times a bf16 table. */
LTXATTN_API int ltxattn_rope(const ltxattn_rope_args* args, void* stream);

/* ---- query / key preparation ---------------------------------------------- */

/* Arguments of ltxattn_qk_prep: out = split-RoPE(split(rmsNorm(x, weight))).
 *  - dtype, batch, tokens, heads, head_dim: x is [B, tokens, heads * head_dim]
 *    (the projection output, unit stride along the inner dim), out the
 *    [B, heads, tokens, head_dim] view the attention consumes.
 *  - x_stride_b, x_stride_t: element strides of x.
 *  - weight: the norm weight [heads * head_dim] (activation dtype); eps its epsilon.
 *  - rotary: per-head tables as for ltxattn_fwd, or cos = NULL for none (the
 *    attention then gets q / k already rotated and is called without tables).
 * heads * head_dim must be a multiple of 512 and at most 8192. */
typedef struct ltxattn_qk_prep_args {
  int32_t dtype;
  int32_t batch;
  int32_t tokens;
  int32_t heads;
  int32_t head_dim;
  const void* x;
  int64_t x_stride_b;
  int64_t x_stride_t;
  const void* weight;
  float eps;
  ltxattn_rotary rotary;
  ltxattn_tensor out;
} ltxattn_qk_prep_args;

/* Replaces the query / key preparation of `DiTAttention.callAsFunction`
 * (`DiTAttention.swift:358-367`): `rmsNorm` over the whole inner dim (`:190-204`),
 * the head split (`:346-348`) and `applySplitRoPE` (`:206-234`), in one pass. */
LTXATTN_API int ltxattn_qk_prep(const ltxattn_qk_prep_args* args, void* stream);

/* q and k preparations (same dtype and inner width; token counts may differ,
 * as in a cross-attention) in one launch; each result is exactly what
 * ltxattn_qk_prep gives for its arguments. */
LTXATTN_API int ltxattn_qk_prep_pair(const ltxattn_qk_prep_args* q, const ltxattn_qk_prep_args* k, void* stream);

/* ---- rotary tables -------------------------------------------------------- */

/* Arguments of ltxattn_rotary_tables: the per-head split-RoPE tables of one
 * stream (DiTForward.rotary).
 *  - dtype: of the tables (LTXATTN_BF16 for a bf16 model: the reference narrows
 *    its fp32 tables to the activation dtype at use).
 *  - n_pos (1..4), tokens: positions is a device array [n_pos][tokens][2] of
 *    fp32 (lo, hi) bounds per positional dimension (videoPositions /
 *    audioPositions, or IC-LoRA reference positions).
 *  - max_pos[d]: the normaliser of dimension d; theta: the frequency base.
 *  - inner, heads: the attention's inner width and head count; the tables are
 *    [heads, tokens, inner / 2 / heads] (cos and sin, device memory). */
typedef struct ltxattn_rotary_table_args {
  int32_t dtype;
  int32_t n_pos;
  int32_t tokens;
  int32_t inner;
  int32_t heads;
  double theta;
  float max_pos[4];
  const float* positions;
  void* cos;
  void* sin;
} ltxattn_rotary_table_args;

/* Replaces `DiTForward.rotary` (`DiTForward.swift:641-678`, with frequencyGrid
 * `:455-466`): fp64 frequency grid, fp32 angles, leading identity pairs,
 * positional dimension fastest, split per head. */
LTXATTN_API int ltxattn_rotary_tables(const ltxattn_rotary_table_args* args, void* stream);

/* ---- head-parallel all-gather (NCCL over NVLink) ------------------------- */

/* Opaque NCCL communicator owned by the library. */
typedef struct ltxattn_comm ltxattn_comm;

/* Fill 128 bytes with a fresh NCCL unique id (rank 0 calls this and shares
 * the bytes with the other ranks out of band). */
LTXATTN_API int ltxattn_comm_unique_id(uint8_t id[128]);

/* Create the communicator for `rank` of `nranks` on CUDA device `device`. */
LTXATTN_API int ltxattn_comm_init(ltxattn_comm** comm, int32_t nranks, int32_t rank, const uint8_t id[128],
                      int32_t device);
LTXATTN_API int ltxattn_comm_destroy(ltxattn_comm* comm);

/* All-gather head blocks: rank r holds send = [B, heads_per_rank, T, D]
 * (contiguous) for heads [r*heads_per_rank, (r+1)*heads_per_rank); every rank
 * receives recv = [B, nranks*heads_per_rank, T, D] (contiguous).  The
 * reference has no collective; this is only used where a caller needs every
 * head (e.g. a non-sharded to_out, `DiTAttention.swift:402-404`). */
typedef struct ltxattn_gather_args {
  int32_t dtype;
  int32_t batch, heads_per_rank, tokens, head_dim;
  const void* send;
  void* recv;
} ltxattn_gather_args;

LTXATTN_API int ltxattn_allgather_heads(const ltxattn_gather_args* args, ltxattn_comm* comm, void* stream);

/* Row-parallel to_out over the head shards (`DiTAttention.swift:401-404` with
 * heads sharded across ranks): rank r holds its heads' slice of the merged
 * attention output x [m, k] (k = heads_per_rank * head_dim) and the matching
 * column block of to_out.0.weight ([n, k] rows of weight_stride, e.g. the full
 * weight's pointer advanced by r * k with weight_stride = heads * head_dim).
 * Each rank's GEMM writes its fp32 partial product into the workspace
 * (m * n floats, ltxattn_out_project_workspace bytes, 256-byte aligned), an
 * NCCL all-reduce sums the partials over the ranks in place, and every rank
 * stores out = T(T(sum) + bias), the roundings of DiTAttention.linear
 * (`:178-188`) applied once to the full sum.  With one rank the result is
 * bit-identical to ltxattn_linear on the same arguments.  n a multiple of 8,
 * k of 64.  The reference is single-device; this serves a head-parallel job
 * whose next layer needs the whole to_out output on every rank. */
typedef struct ltxattn_out_project_args {
  int32_t dtype; /* LTXATTN_BF16 */
  int32_t m, n, k;
  const void* x;
  int64_t x_stride;
  const void* weight;
  int64_t weight_stride;
  const void* bias;
  void* out;
  int64_t out_stride;
  void* workspace;
  size_t workspace_bytes;
} ltxattn_out_project_args;

LTXATTN_API size_t ltxattn_out_project_workspace(const ltxattn_out_project_args* args);

/* Every rank's receive planes, output and signal words for
 * ltxattn_out_project_fused, mapped on the calling device (CUDA IPC over
 * NVLink).  recv[d]: rank d's `world` fp32 planes of [m, n] (plane s holds the
 * partial from rank s); out[d]: rank d's [m, n] bf16 output (row stride
 * args->out_stride); signals[d]: rank d's 16 signal words, zero at
 * allocation. */
typedef struct ltxattn_reduce_peers {
  int32_t world;
  int32_t rank;
  float* recv[8];
  void* out[8];
  uint32_t* signals[8];
  uint32_t epoch;         /* 1, 2, 3, ...: one per call, the same on every rank */
  int32_t reserved;
} ltxattn_reduce_peers;

/* The row-parallel to_out with its reduction done over peer memory instead of
 * an NCCL all-reduce (no counterpart in the reference, which runs one device).
 * Rows are owned in blocks of 128 (rank t / rows_per_owner); the GEMM's
 * epilogue stores each fp32 partial row straight into its owner's receive plane
 * for this rank; after a bounded handshake each owner adds its rows' planes in
 * rank order, applies the bias and the roundings of DiTAttention.linear, and
 * stores the bf16 rows into every rank's output; a second bounded handshake
 * ends the call with the whole output on every rank.  Same arithmetic as
 * ltxattn_out_project_allreduce (fp32 partials added in rank order, then
 * T(T(sum) + b)).  args->workspace is unused; args->out must be
 * peers->out[rank]; not for stream capture (the epoch is a launch argument). */
LTXATTN_API int ltxattn_out_project_fused(const ltxattn_out_project_args* args, const ltxattn_reduce_peers* peers,
                                          void* stream);
LTXATTN_API int ltxattn_out_project_allreduce(const ltxattn_out_project_args* args, ltxattn_comm* comm,
                                              void* stream);

/* The rank count and this rank's index as NCCL itself reports them
 * (ncclCommCount / ncclCommUserRank), for checking a launch's world size.
 * No counterpart in the reference. */
LTXATTN_API int ltxattn_comm_size(const ltxattn_comm* comm, int32_t* nranks, int32_t* rank);

/* ---- device discovery ----------------------------------------------------- */

/* Replaces `LTXHardware.Machine.detect` (`Machine.swift:31-36`) and the Metal
 * library locator (`MetalLibrary.swift:25-128`) for a CUDA device. */
typedef struct ltxattn_device_info {
  char name[256];
  int32_t device;
  int32_t cc_major, cc_minor;
  int32_t sm_count;
  int64_t total_memory_bytes;
  int64_t free_memory_bytes;
  int32_t max_smem_per_block_optin;
  int32_t l2_bytes;
  int32_t sm_clock_khz;
  int32_t mem_clock_khz;
  int32_t mem_bus_width_bits;
  int32_t supported; /* 1 when the kernels here run on it (sm_100) */
} ltxattn_device_info;

LTXATTN_API int ltxattn_device_count(int32_t* count);
LTXATTN_API int ltxattn_device_query(int32_t device, ltxattn_device_info* info);

/* ---- memory planning ------------------------------------------------------ */

/* Whether an attention working set fits the current device: the counterpart of
 * `LTXHardware.MemoryPlan` (`MemoryPlan.swift:27-34,62-74`).  The reference fits
 * its fused-path activation bytes to MLX allocator peaks (4.67e5 B per video
 * token); here the bytes are the exact buffers of one call at this shape: q, k,
 * v, out and the fp32 lse, the library's workspace for the call
 * (ltxattn_fwd_workspace), and with `training` the backward's dout, dq, dk, dv
 * and ltxattn_bwd_workspace.  A self-attention shape (q, k, v of `tokens`
 * rows) is planned; `rotary` = 1 when the call rotates q and k. */
typedef struct ltxattn_memory_plan_args {
  int32_t dtype;
  int32_t batch, heads, tokens, head_dim;
  int32_t rotary;
  int32_t training;
  int64_t resident_bytes;   /* already held on the device (weights; the reference's DiT is 42.06e9) */
  int64_t available_bytes;  /* 0: the current device's free memory (cudaMemGetInfo) */
  double margin_fraction;   /* MemoryPlan.plan's margin (0.15 there) */
} ltxattn_memory_plan_args;

typedef struct ltxattn_memory_plan_info {
  int64_t tensor_bytes;     /* q, k, v, out, lse */
  int64_t workspace_bytes;  /* ltxattn_fwd_workspace of the call */
  int64_t backward_bytes;   /* dout, dq, dk, dv and ltxattn_bwd_workspace (0 unless training) */
  int64_t peak_bytes;       /* resident + the three above */
  int64_t available_bytes;
  int64_t headroom_bytes;   /* available - peak * (1 + margin), as MemoryPlan.headroomBytes */
  int32_t fits;             /* headroom > 0 */
  double bytes_per_token;   /* attention bytes per batch row token: the counterpart of 4.67e5 */
} ltxattn_memory_plan_info;

LTXATTN_API int ltxattn_memory_plan(const ltxattn_memory_plan_args* args, ltxattn_memory_plan_info* info);

/* ---- status --------------------------------------------------------------- */

/* Message for this thread's most recent failure ("" if none). */
LTXATTN_API const char* ltxattn_last_error(void);

/* Read (and, when `clear` is nonzero, reset) the current device's kernel
 * error word.  Synchronises the device.  Returns LTXATTN_ERR_TIMEOUT when a
 * kernel's bounded wait gave up since the last clear; *site receives the
 * encoded wait site (may be NULL). */
LTXATTN_API int ltxattn_device_status(int32_t clear, int32_t* site);

/* Failure-detection self-test (no counterpart in the reference): launches one
 * CTA on `stream` that waits, with the same bounded wait as the attention
 * kernels, on an mbarrier nothing ever arrives at.  After limit_us
 * microseconds (1 .. 1000000) the wait gives up, records LTXATTN_ERR_TIMEOUT
 * with site 99 in the device error word, and the CTA frees its tensor memory
 * and exits normally; no fault, and the context stays usable.  Returns
 * LTXATTN_OK once launched; ltxattn_device_status then reports the timeout. */
LTXATTN_API int ltxattn_selftest_wait_timeout(uint32_t limit_us, void* stream);

/* Library state: the device error word's address and the no-allocation
 * forward's scratch address are looked up once per device and kept for the
 * life of the process.  Do not keep using the library on a device after
 * cudaDeviceReset (or any teardown of the device's primary context) in the
 * same process: those addresses then no longer belong to the new context. */
LTXATTN_API int ltxattn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LTXATTN_H */
