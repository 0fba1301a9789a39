// ltxattn_internal.h -- parameter blocks and launchers shared by the kernel
// files and the C-ABI layer.  Not installed; the public surface is
// include/ltxattn.h.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ltx {

// Device error word encoding: (site << 8) | code.
constexpr int kErrNone = 0;
constexpr int kErrTimeout = 1;

constexpr int kTileM = 128;            // query rows per CTA (UMMA M)
constexpr int kTileN = 128;            // keys per KV tile (UMMA N of QK^T)
constexpr int kMaxKvLen = 131072;      // 1024 KV tiles
constexpr int kMaxKvTiles = kMaxKvLen / kTileN;
constexpr int kMaxSplits = 32;
constexpr int kFwdBlockM = 2 * kTileM;  // query rows per forward CTA (two Q tiles)

// Forward, bf16 tcgen05 path.
struct FwdParams {
  CUtensorMap tm_q;  // [D, Lq, Hq, B] box {64, 128, 1, 1}, 128B swizzle
  CUtensorMap tm_k;  // [D, Lk, Hk, B] box {64, 128, 1, 1}
  CUtensorMap tm_v;  // [D, Lk, Hk, B] box {64, 128, 1, 1}
  CUtensorMap tm_o;  // [D, Lq, H, B] box {64, 128, 1, 1}: the output of unsplit units
  CUtensorMap tm_part;  // fp32 [D, 256, n_tail, splits] box {32, 128, 1, 1}: partials of split units
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  float* lse;  // natural log, may be null
  int64_t lse_sb, lse_sh;
  const uint8_t* mask;  // [B, Lk] or null
  int64_t mask_sb;
  int mask_vec;  // every mask row is 16-byte aligned (vector loads)
  int Lq, Lk;
  int head_begin;   // global index of local head 0 (out / lse / mask addressing)
  int q_head_off;   // head coordinate of local head 0 in tm_q
  int kv_head_off;  // head coordinate of local head 0 in tm_k / tm_v
  int n_kv_tiles;
  // Work units are (256-row query block, local head, batch), q_block fastest.
  // Units [0, n_full) run whole, one CTA each; each of the n_tail units after
  // them runs as num_splits CTAs over shares of its KV tiles (1-D grid of
  // n_full + n_tail * num_splits CTAs, so the split CTAs fill the last wave).
  int q_blocks, Hc;
  int n_full, n_tail;
  int num_splits;
  int group;   // query heads per kv head: kv head = (kv_head_off + local head) / group
  int causal;  // key j attends query i only if j <= i (q_len == kv_len)
  int window;  // > 0: also i - j < window
  float scale_log2;  // softmax scale * log2(e)
  float* part_lse;   // [splits][n_tail][256] log2 domain (n_tail > 0)
  const __nv_bfloat16* gate;  // [B, Lq, H] gate logits or null (global head index)
  int64_t g_sb, g_st, g_sh;
  // Fused all-gather (ltxattn_fwd_gather): peer_n > 0 makes the epilogue also
  // store each output tile with TMA into the outputs of the other ranks
  // (tm_peer[i]: the output of the i-th other rank, same geometry as tm_o).
  int peer_n;
  int* err;
  CUtensorMap tm_peer[7];
};

// Cross-device entry / arrival handshakes of ltxattn_fwd_gather (signal words:
// [0, 8) "rank d's tiles of this epoch have landed here", [8, 16) "rank d has
// entered this epoch").
struct GatherSync {
  unsigned int* sig[8];
  int n, rank;
  unsigned int epoch;
  int word;  // gather_done's words: [word, word + 8) (0, or 8 for a second handshake of one call)
  int* err;
};
cudaError_t launch_gather_enter(const GatherSync& g, cudaStream_t s);
cudaError_t launch_gather_done(const GatherSync& g, cudaStream_t s);

// Forward, fp32 SIMT path (parity path for the float32 dtype).
struct F32Params {
  const float* q;
  const float* k;
  const float* v;
  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  int q_head_off, kv_head_off;  // head index of local head 0 in q / k,v
  float* out;
  int64_t o_sb, o_sh, o_st;
  float* lse;
  int64_t lse_sb, lse_sh;
  const uint8_t* mask;
  int64_t mask_sb;
  int Lq, Lk, head_begin;
  float scale;
  int group, causal, window;  // as FwdParams
  const float* gate;          // as FwdParams (fp32 logits)
  int64_t g_sb, g_st, g_sh;
};

// Split-RoPE pre-pass: y[b][hl][t][:] = rope(x[b][head_begin+hl][t][:]) into a
// contiguous buffer.
struct RopeParams {
  const void* x;
  int64_t x_sb, x_sh, x_st;
  const void* cos;
  const void* sin;
  int64_t t_sb, t_sh, t_st;
  void* y;  // [B][Hc][T][D] view, local head index
  int64_t y_sb, y_sh, y_st;
  int B, Hc, T, D, head_begin;
};

// q / k preparation (rmsNorm over the inner dim, head split, split RoPE): see qkprep.cu.
struct QkPrepParams {
  const void* x;  // [B, tokens, inner] rows, unit stride along inner
  int64_t x_sb, x_st;
  const void* w;  // [inner] norm weight (activation dtype)
  float eps;
  const void* cos;  // per-head tables or null (no rotation)
  const void* sin;
  int64_t t_sb, t_sh, t_st;
  void* out;  // [B, H, tokens, D] view
  int64_t o_sb, o_sh, o_st;
  int B, tokens, inner, D;
  int vec;  // every row, weight, table and output address is 16-byte aligned (vector loads and stores)
  int* err;  // device error word (bounded waits)
};
cudaError_t launch_qk_prep(const QkPrepParams& p, bool bf16, cudaStream_t s);
cudaError_t launch_qk_prep_pair(const QkPrepParams& p0, const QkPrepParams& p1, bool bf16, cudaStream_t s);

// Rotary tables (DiTForward.rotary): see rotary.cu.
struct RotaryTableParams {
  const float* positions;  // [n_pos][tokens][2] fp32 (lo, hi)
  void* cos;               // [heads][tokens][inner/2/heads], activation dtype
  void* sin;
  double theta;
  float max_pos[4];
  int n_pos, tokens, inner, heads, count, pad;
};
cudaError_t launch_rotary_tables(const RotaryTableParams& p, bool bf16, cudaStream_t s);

struct CombineParams {
  const float* part_o;
  const float* part_lse;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  float* lse;
  int64_t lse_sb, lse_sh;
  int Hc, Lq, D, num_splits, head_begin;
  int q_blocks, n_full, n_tail;  // the forward's unit split (FwdParams)
  const __nv_bfloat16* gate;     // as FwdParams
  int64_t g_sb, g_st, g_sh;
  int peer_n;                    // fused all-gather: the rows also go to these outputs (same strides)
  __nv_bfloat16* peer_out[7];
};

// Backward.  Every pointer and tensor map is based at local head 0 (the
// C-ABI layer offsets the caller's views by head_begin), so kernels index
// heads by blockIdx.y directly.
struct BwdParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;  // [D, T, Hc, B] box {64, 128, 1, 1}
  const float* lse2;                    // [B][Hc][Lq_pad]: lse*log2(e) (bf16) or lse (f32); +inf pad
  const float* delta;                   // [B][Hc][Lq_pad]: rowsum(dO o O); 0 pad
  int Lq_pad;
  void* dq;
  int64_t dq_sb, dq_sh, dq_st;
  void* dk;
  int64_t dk_sb, dk_sh, dk_st;
  void* dv;
  int64_t dv_sb, dv_sh, dv_st;
  const uint8_t* mask;
  int64_t mask_sb;
  const void* qcos;  // transpose rotation of dq (null = none), activation dtype
  const void* qsin;
  int64_t qt_sb, qt_sh, qt_st;
  const void* kcos;  // transpose rotation of dk
  const void* ksin;
  int64_t kt_sb, kt_sh, kt_st;
  int rope_vec;  // both tables' rows are 16-byte aligned (bf16 path: vector table reads)
  // fp32 path: plain strided inputs (no tensor maps)
  const float* q;
  const float* k;
  const float* v;
  const float* dout;
  int64_t q_sb, q_sh, q_st, k_sb, k_sh, k_st, v_sb, v_sh, v_st, do_sb, do_sh, do_st;
  int Lq, Lk;
  int n_q_tiles, n_kv_tiles;
  float scale, scale_log2;
  int* err;
};

struct BwdPrepParams {
  const void* o;
  int64_t o_sb, o_sh, o_st;
  const void* dout;
  int64_t do_sb, do_sh, do_st;
  const float* lse;
  int64_t lse_sb, lse_sh;
  float* lse2;
  float* delta;
  int B, Hc, Lq, Lq_pad, D;
  int log2_domain;  // 1: lse2 = lse*log2(e) (bf16 kernels); 0: natural lse (fp32 kernels)
  int f32;          // o / dout are float32
};

// Launch with programmatic stream serialization: the kernel's CTAs may start
// while the previous kernel in the stream finishes (their prologue overlaps
// its tail) and must call grid_dep_wait() before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Launchers (return cudaError_t of the launch).
// Once-per-device kernel attributes (cached); call before launch_fwd_bf16.
cudaError_t prepare_fwd_bf16(int D, size_t smem_bytes);
cudaError_t launch_fwd_bf16(const FwdParams& p, int D, size_t smem_bytes, cudaStream_t s);
size_t fwd_bf16_smem_bytes(int D, int Lk, bool has_mask);
// Persistent forward for kv_len <= 128 (one KV tile); see fwd_short_sm100.cu.
cudaError_t prepare_fwd_short(int D);
cudaError_t launch_fwd_short(const FwdParams& p, int D, int units, int sms, cudaStream_t s);
// Persistent forward for unbanded calls of at least one wave: `ctas` CTAs walk
// the p.n_full units round-robin; see fwd_persist_sm100.cu.  With a key mask the
// shared memory holds every batch row's mask bits and live-tile list.
size_t fwd_persist_smem_bytes(int D, int batch, int kv_tiles, bool has_mask);
constexpr size_t kMaxDynamicSmem = 232448;  // sm_100 per-block opt-in limit (227 KB)
cudaError_t prepare_fwd_persist(int D, size_t smem);
cudaError_t launch_fwd_persist(const FwdParams& p, int D, int ctas, size_t smem, cudaStream_t s);
cudaError_t launch_combine(const CombineParams& p, cudaStream_t s);
cudaError_t launch_fwd_f32(const F32Params& p, int D, int Hc, int B, cudaStream_t s);
// Rotate one tensor (b == nullptr) or two in one launch.
cudaError_t launch_rope(const RopeParams* a, const RopeParams* b, bool bf16, cudaStream_t s);
cudaError_t launch_bwd_prep(const BwdPrepParams& p, cudaStream_t s);
size_t bwd_dq_smem_bytes(int D, int Lk, bool has_mask);
size_t bwd_dkdv_smem_bytes(int D, int Lk, bool has_mask);
// Once-per-device kernel attributes (cached); call before launch_bwd_bf16.
cudaError_t prepare_bwd_bf16(int D, size_t smem_dq, size_t smem_dkdv);
cudaError_t launch_bwd_bf16(const BwdParams& p, int D, int Hc, int B, size_t smem_dq, size_t smem_dkdv,
                            cudaStream_t s);
cudaError_t launch_bwd_f32(const BwdParams& p, int D, int Hc, int B, cudaStream_t s);

// Device error word of this module (one per device).
int* device_error_word();

}  // namespace ltx

struct ltxattn_linear_args;

namespace ltx {

// The row-parallel to_out's local steps (proj_sm100.cu): the GEMM's fp32
// accumulator into `partial` [m, n] (no bias, no rounding), and, after the
// reduction across ranks, out = T(T(sum) + bias) (sum: `splits` partial planes
// split_stride floats apart, added in order).
int linear_partial_f32(const ltxattn_linear_args* a, float* partial, cudaStream_t st);
int bias_round(const float* sum, int splits, int64_t split_stride, const void* bias, void* out, int64_t out_stride,
               int m, int n, cudaStream_t st, int n_peer_out = 0, void* const* peer_out = nullptr);
// The fused reduce-scatter's GEMM (ltxattn_out_project_fused): row t's fp32
// partial goes to plane `rank` of the receive planes of rank t / rows_per_owner
// (planes[d]: rank d's [world][m][n] planes, slot_stride floats apart).
struct OwnerPlanes {
  int world, rank, rows_per_owner;
  int64_t slot_stride;
  float* planes[8];
};
int linear_partial_f32_to_owners(const ltxattn_linear_args* a, float* const* planes, int world, int rank,
                                 int rows_per_owner, int64_t slot_stride, cudaStream_t st);

}  // namespace ltx
