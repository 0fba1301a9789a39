// rope.cu -- split-RoPE pre-pass (DiTAttention.swift:206-234).
//
//   out[..., :D/2] = x1*cos - x2*sin ;  out[..., D/2:] = x2*cos + x1*sin
//
// bf16: every product and sum is rounded to bf16, the arithmetic of a bf16
// MLX tensor times a bf16 table (the tables are narrowed to the activation
// dtype first, :231-232).  Each op is evaluated in fp32 and rounded once, so
// no product is fused into the following add.
// fp32: the same four products and two sums in fp32, unfused.
// inverse = 1 applies the transpose rotation (g1*c + g2*s, g2*c - g1*s) in
// fp32 without rounding: the gradient w.r.t. the un-rotated input.
//
// Reads a strided [B, H, T, D] view, writes a contiguous [B, Hc, T, D] buffer
// (the library's workspace), 8 rotary pairs per thread.
#include "ltxattn_internal.h"

namespace ltx {
namespace {

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void st(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

template <typename T, bool kBf16>
__global__ void __launch_bounds__(256) rope_kernel(const RopeParams p) {
  const int half = p.D / 2;
  const int groups = half / 8;  // 8 pairs per thread
  const int64_t total = (int64_t)p.B * p.Hc * p.T * groups;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= total) return;
  const int g = (int)(gid % groups);
  const int t = (int)((gid / groups) % p.T);
  const int hl = (int)((gid / ((int64_t)groups * p.T)) % p.Hc);
  const int b = (int)(gid / ((int64_t)groups * p.T * p.Hc));
  const int h = p.head_begin + hl;
  const T* x = static_cast<const T*>(p.x) + (int64_t)b * p.x_sb + (int64_t)h * p.x_sh + (int64_t)t * p.x_st;
  const T* c = static_cast<const T*>(p.cos) + (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st;
  const T* s = static_cast<const T*>(p.sin) + (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st;
  T* y = static_cast<T*>(p.y) + (((int64_t)b * p.Hc + hl) * p.T + t) * p.D;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = g * 8 + e;
    const float x1 = ld(x, i), x2 = ld(x, i + half);
    const float cc = ld(c, i), ss = ld(s, i);
    float o1, o2;
    if (p.inverse) {
      o1 = __fadd_rn(__fmul_rn(x1, cc), __fmul_rn(x2, ss));
      o2 = __fsub_rn(__fmul_rn(x2, cc), __fmul_rn(x1, ss));
    } else if (kBf16) {
      o1 = bf(__fsub_rn(bf(__fmul_rn(x1, cc)), bf(__fmul_rn(x2, ss))));
      o2 = bf(__fadd_rn(bf(__fmul_rn(x2, cc)), bf(__fmul_rn(x1, ss))));
    } else {
      o1 = __fsub_rn(__fmul_rn(x1, cc), __fmul_rn(x2, ss));
      o2 = __fadd_rn(__fmul_rn(x2, cc), __fmul_rn(x1, ss));
    }
    st(y, i, o1);
    st(y, i + half, o2);
  }
}

template <typename T, bool kBf16>
cudaError_t launch(const RopeParams& p, cudaStream_t s) {
  const int64_t total = (int64_t)p.B * p.Hc * p.T * (p.D / 16);
  const int blocks = (int)((total + 255) / 256);
  if (blocks > 0) rope_kernel<T, kBf16><<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope_bf16(const RopeParams& p, cudaStream_t s) { return launch<__nv_bfloat16, true>(p, s); }
cudaError_t launch_rope_f32(const RopeParams& p, cudaStream_t s) { return launch<float, false>(p, s); }

}  // namespace ltx
