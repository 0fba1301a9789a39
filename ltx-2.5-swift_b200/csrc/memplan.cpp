// memplan.cpp -- ltxattn_memory_plan: will an attention working set fit this
// CUDA device?  The counterpart, for the fused attention on a B200, of the
// reference's Sources/LTXHardware/MemoryPlan.swift.
//
// The reference fits its fused-path activation memory to two MLX allocator
// measurements on an M3 Ultra (MemoryPlan.swift:27-34: 4.67e5 bytes per video
// token above the weights, linear) and admits a render when the peak phase,
// grown by a safety margin, is below the available memory (:62-74).  Here the
// attention's device bytes are not fitted: they are the exact sizes of the
// buffers one call needs -- q, k, v, out and the log-sum-exp, plus the
// library's own workspace for those arguments (ltxattn_fwd_workspace, and
// for training the backward's dout, dq, dk, dv and ltxattn_bwd_workspace) --
// and the available bytes are the device's free memory (cudaMemGetInfo)
// unless the caller gives a figure.  The margin and the headroom keep the
// reference's meaning: headroom = available - peak * (1 + margin).
#include <cuda_runtime.h>

#include <cmath>

#include "../../include/ltxattn.h"

namespace ltx {
int set_error_message(int status, const char* msg);
}

extern "C" {

int ltxattn_memory_plan(const ltxattn_memory_plan_args* a, ltxattn_memory_plan_info* info) {
  if (a == nullptr || info == nullptr) return ltx::set_error_message(LTXATTN_ERR_ARG, "args or info is NULL");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1)
    return ltx::set_error_message(LTXATTN_ERR_SHAPE, "ltxattn_memory_plan: batch, heads and tokens must be >= 1");
  if (a->resident_bytes < 0 || a->available_bytes < 0 || !(a->margin_fraction >= 0.0))
    return ltx::set_error_message(LTXATTN_ERR_ARG,
                                  "ltxattn_memory_plan: resident and available bytes and the margin must be >= 0");
  const int64_t es = a->dtype == LTXATTN_BF16 ? 2 : 4;
  const int64_t B = a->batch, H = a->heads, T = a->tokens, D = a->head_dim;
  const int64_t act = B * H * T * D * es;  // one [B, H, T, D] tensor

  // the library's workspace for exactly this call (the pointers are never read:
  // planning looks at shapes and at which options are present)
  static char placeholder[16];
  ltxattn_fwd_args f{};
  f.dtype = a->dtype;
  f.batch = a->batch;
  f.heads = a->heads;
  f.q_len = f.kv_len = a->tokens;
  f.head_dim = a->head_dim;
  f.scale = 1.0f;
  if (a->rotary) {
    f.q_rotary.cos = f.q_rotary.sin = placeholder;
    f.q_rotary.tokens = a->tokens;
  }
  ltxattn_fwd_plan_info pi;
  if (const int rc = ltxattn_fwd_plan(&f, &pi)) return rc;  // a shape the forward refuses
  const size_t fws = ltxattn_fwd_workspace(&f);
  int64_t bws = 0;
  if (a->training) {
    ltxattn_bwd_args b{};
    b.dtype = a->dtype;
    b.batch = a->batch;
    b.heads = a->heads;
    b.q_len = b.kv_len = a->tokens;
    b.head_dim = a->head_dim;
    b.scale = 1.0f;
    b.q_rotary = f.q_rotary;
    bws = (int64_t)ltxattn_bwd_workspace(&b);
  }

  info->tensor_bytes = 4 * act + B * H * T * 4;  // q, k, v, out + fp32 lse
  info->workspace_bytes = (int64_t)fws;
  info->backward_bytes = a->training ? 4 * act + bws : 0;  // dout, dq, dk, dv + backward workspace
  const int64_t attention = info->tensor_bytes + info->workspace_bytes + info->backward_bytes;
  info->peak_bytes = a->resident_bytes + attention;
  int64_t avail = a->available_bytes;
  if (avail == 0) {
    size_t free_b = 0, total_b = 0;
    const cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();  // not left behind for a later launch check to find
      return ltx::set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
    }
    avail = (int64_t)free_b;
  }
  info->available_bytes = avail;
  info->headroom_bytes = avail - (int64_t)std::llround((double)info->peak_bytes * (1.0 + a->margin_fraction));
  info->fits = info->headroom_bytes > 0 ? 1 : 0;
  info->bytes_per_token = (double)attention / (double)(B * T);
  return LTXATTN_OK;
}

}  // extern "C"
