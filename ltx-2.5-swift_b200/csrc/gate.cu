// gate.cu -- ltxattn_head_gate: the per-head output gate and the merge of
// DiTAttention.swift:395-403 for a tensor that did not come out of the
// attention kernel (whose store applies the same gate itself): the STG
// passthrough, where a fully perturbed block returns the projected values
// v in place of the attention output (DiTAttention.swift:349-356).
//
//   out[b, h, t, :] = T(T(x[b, h, t, :]) * g),  g = 2 * T(sigmoid(logit[b, t, h]))
//
// with the sigmoid in fp32 and cast back to the activation dtype T
// (:236-242); without logits, out = x (the merge alone).  `out` may view the
// merged [B, T, H * D] buffer, so the transpose of :401-403 is the store's
// addressing.  One thread moves 8 elements (16 bytes of bf16).
#include <cstdio>

#include "../../include/ltxattn.h"
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {

int set_error_message(int status, const char* msg);

namespace {

struct HeadGateParams {
  const void* x;
  int64_t x_sb, x_sh, x_st;
  void* out;
  int64_t o_sb, o_sh, o_st;
  const void* gate;
  int64_t g_sb, g_st, g_sh;
  int B, H, T, D;
  int64_t total8;  // B * H * T * D / 8
};

template <bool kBf16>
__global__ void __launch_bounds__(256) head_gate_kernel(const HeadGateParams p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.total8) return;
  const int d8 = p.D / 8;
  const int d = (int)(i % d8) * 8;
  int64_t r = i / d8;
  const int t = (int)(r % p.T);
  r /= p.T;
  const int h = (int)(r % p.H);
  const int b = (int)(r / p.H);
  if constexpr (kBf16) {
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x) + b * p.x_sb + h * p.x_sh + t * p.x_st + d;
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + b * p.o_sb + h * p.o_sh + t * p.o_st + d;
    uint4 v = *reinterpret_cast<const uint4*>(x);
    if (p.gate != nullptr) {
      const float logit = __bfloat162float(
          static_cast<const __nv_bfloat16*>(p.gate)[b * p.g_sb + (int64_t)t * p.g_st + (int64_t)h * p.g_sh]);
      const float g = gate_bf16(logit);
      const uint32_t g2 = pack_bf16x2(g, g);
      v.x = bmul2(v.x, g2);
      v.y = bmul2(v.y, g2);
      v.z = bmul2(v.z, g2);
      v.w = bmul2(v.w, g2);
    }
    *reinterpret_cast<uint4*>(o) = v;
  } else {
    const float* x = static_cast<const float*>(p.x) + b * p.x_sb + h * p.x_sh + t * p.x_st + d;
    float* o = static_cast<float*>(p.out) + b * p.o_sb + h * p.o_sh + t * p.o_st + d;
    float g = 1.f;
    if (p.gate != nullptr)
      g = gate_f32(static_cast<const float*>(p.gate)[b * p.g_sb + (int64_t)t * p.g_st + (int64_t)h * p.g_sh]);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = p.gate != nullptr ? __fmul_rn(x[e], g) : x[e];
  }
}

int fail_gate(int status, const char* msg) { return set_error_message(status, msg); }

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

}  // namespace
}  // namespace ltx

extern "C" {

int ltxattn_head_gate(const ltxattn_head_gate_args* a, void* stream) {
  using namespace ltx;
  if (a == nullptr) return fail_gate(LTXATTN_ERR_ARG, "args is NULL");
  if (a->dtype != LTXATTN_BF16 && a->dtype != LTXATTN_F32)
    return fail_gate(LTXATTN_ERR_DTYPE, "ltxattn_head_gate: dtype must be LTXATTN_BF16 or LTXATTN_F32");
  if (a->batch < 1 || a->heads < 1 || a->tokens < 1 || a->head_dim < 8 || a->head_dim % 8)
    return fail_gate(LTXATTN_ERR_SHAPE, "ltxattn_head_gate: sizes must be >= 1 and head_dim a multiple of 8");
  if (a->x.data == nullptr || a->out.data == nullptr)
    return fail_gate(LTXATTN_ERR_ARG, "ltxattn_head_gate: x and out are required");
  const int es = a->dtype == LTXATTN_BF16 ? 2 : 4;
  const int64_t q = 16 / es;
  const ltxattn_tensor* v[2] = {&a->x, &a->out};
  for (const ltxattn_tensor* t : v) {
    if (t->stride_b < 0 || t->stride_h < 0 || t->stride_t < 0)
      return fail_gate(LTXATTN_ERR_SHAPE, "ltxattn_head_gate: negative stride");
    if (!aligned(t->data, 16) || t->stride_b % q || t->stride_h % q || t->stride_t % q)
      return fail_gate(LTXATTN_ERR_ALIGN, "ltxattn_head_gate: x and out rows must be 16-byte aligned");
  }
  if (a->gate != nullptr && (a->gate_stride_b < 0 || a->gate_stride_t < 0 || a->gate_stride_h < 0))
    return fail_gate(LTXATTN_ERR_SHAPE, "ltxattn_head_gate: gate has a negative stride");
  HeadGateParams p;
  p.x = a->x.data;
  p.x_sb = a->x.stride_b;
  p.x_sh = a->x.stride_h;
  p.x_st = a->x.stride_t;
  p.out = a->out.data;
  p.o_sb = a->out.stride_b;
  p.o_sh = a->out.stride_h;
  p.o_st = a->out.stride_t;
  p.gate = a->gate;
  p.g_sb = a->gate_stride_b;
  p.g_st = a->gate_stride_t;
  p.g_sh = a->gate_stride_h;
  p.B = a->batch;
  p.H = a->heads;
  p.T = a->tokens;
  p.D = a->head_dim;
  p.total8 = (int64_t)a->batch * a->heads * a->tokens * (a->head_dim / 8);
  const int64_t blocks = (p.total8 + 255) / 256;
  if (blocks > 0x7fffffff) return fail_gate(LTXATTN_ERR_UNSUPPORTED, "ltxattn_head_gate: tensor too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == LTXATTN_BF16)
    head_gate_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(p);
  else
    head_gate_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_gate(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  return LTXATTN_OK;
}

}  // extern "C"
