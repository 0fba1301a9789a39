// rope.cu -- split-RoPE pre-pass (DiTAttention.swift:206-234).
//
//   out[..., :D/2] = x1*cos - x2*sin ;  out[..., D/2:] = x2*cos + x1*sin
//
// bf16: every product and sum is rounded to bf16, the arithmetic of a bf16
// MLX tensor times a bf16 table (the tables are narrowed to the activation
// dtype first, :231-232).  The vector path uses the bf16x2 instructions
// (rope_bf16x8); the scalar path evaluates each op in fp32 and rounds once;
// both give the same bits.  No product is fused into the following add.
// fp32: the same four products and two sums in fp32, unfused.
//
// Reads a strided [B, H, T, D] view, writes a [B, Hc, T, D] view (the
// library's workspace, or the caller's output for ltxattn_rope; in place is
// allowed: each thread reads both halves of its pairs before writing them).
// One launch can rotate two tensors (q and k).  Each thread handles 8 rotary
// pairs; when every address of a job is 16-byte aligned the pairs move as one
// 16-byte load/store per operand (bf16), else element by element.
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void rot(float x1, float x2, float c, float s, bool bf16, float& o1, float& o2) {
  if (bf16) {
    o1 = bf(__fsub_rn(bf(__fmul_rn(x1, c)), bf(__fmul_rn(x2, s))));
    o2 = bf(__fadd_rn(bf(__fmul_rn(x2, c)), bf(__fmul_rn(x1, s))));
  } else {
    o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
}

// Grid: x covers (token, 8-pair group) of one (head, batch), y = local head,
// z = batch for job a followed by batch for job b.  Groups per row are 4 or 8
// (D = 64 / 128), so the decode is shifts, not divisions.  Each kernel inlines
// its body once per job with that job's parameter block, so every field is a
// fixed-offset parameter load (selecting a block through a pointer would make
// each thread copy both blocks to local memory).
__device__ __forceinline__ bool locate(const RopeParams& p, int& hl, int& t, int& g) {
  hl = blockIdx.y;
  if (hl >= p.Hc) return false;
  const int shift = p.D == 128 ? 3 : 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  g = idx & ((1 << shift) - 1);
  t = idx >> shift;
  return t < p.T;
}

__device__ __forceinline__ void rope_vec_job(const RopeParams& p, int b) {
  int hl, t, g;
  if (!locate(p, hl, t, g)) return;
  const int half = p.D / 2;
  const int h = p.head_begin + hl;
  const __nv_bfloat16* x =
      static_cast<const __nv_bfloat16*>(p.x) + (int64_t)b * p.x_sb + (int64_t)h * p.x_sh + (int64_t)t * p.x_st + g * 8;
  const int64_t toff = (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st + g * 8;
  const uint4 vx1 = __ldg(reinterpret_cast<const uint4*>(x));
  const uint4 vx2 = __ldg(reinterpret_cast<const uint4*>(x + half));
  const uint4 vc = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.cos) + toff));
  const uint4 vs = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.sin) + toff));
  uint4 o1v, o2v;
  rope_bf16x8(vx1, vx2, vc, vs, o1v, o2v);
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y) + (int64_t)b * p.y_sb + (int64_t)hl * p.y_sh +
                     (int64_t)t * p.y_st + g * 8;
  *reinterpret_cast<uint4*>(y) = o1v;
  *reinterpret_cast<uint4*>(y + half) = o2v;
}

__global__ void __launch_bounds__(256) rope_bf16_vec_kernel(const RopeParams a, const RopeParams c2) {
  grid_dep_launch_dependents();  // the attention kernel after this one may start its prologue
  const int z = blockIdx.z;
  if (z < a.B)
    rope_vec_job(a, z);
  else
    rope_vec_job(c2, z - a.B);
}

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

template <typename T>
__device__ __forceinline__ void rope_scalar_job(const RopeParams& p, int b) {
  int hl, t, g;
  if (!locate(p, hl, t, g)) return;
  const int half = p.D / 2;
  const int h = p.head_begin + hl;
  const bool bf16 = sizeof(T) == 2;
  const T* x = static_cast<const T*>(p.x) + (int64_t)b * p.x_sb + (int64_t)h * p.x_sh + (int64_t)t * p.x_st;
  const T* c = static_cast<const T*>(p.cos) + (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st;
  const T* s = static_cast<const T*>(p.sin) + (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st;
  T* y = static_cast<T*>(p.y) + (int64_t)b * p.y_sb + (int64_t)hl * p.y_sh + (int64_t)t * p.y_st;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = g * 8 + e;
    float o1, o2;
    rot(ld(x, i), ld(x, i + half), ld(c, i), ld(s, i), bf16, o1, o2);
    st(y, i, o1);
    st(y, i + half, o2);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_scalar_kernel(const RopeParams a, const RopeParams c2) {
  grid_dep_launch_dependents();  // the attention kernel after this one may start its prologue
  const int z = blockIdx.z;
  if (z < a.B)
    rope_scalar_job<T>(a, z);
  else
    rope_scalar_job<T>(c2, z - a.B);
}

bool vec_ok(const RopeParams& p) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  auto m8 = [](int64_t s) { return (s % 8) == 0; };
  return al(p.x) && al(p.cos) && al(p.sin) && al(p.y) && m8(p.x_sb) && m8(p.x_sh) && m8(p.x_st) && m8(p.t_sb) &&
         m8(p.t_sh) && m8(p.t_st) && m8(p.y_sb) && m8(p.y_sh) && m8(p.y_st);
}

}  // namespace

// Rotate one or two tensors (b may be null) in one launch.
cudaError_t launch_rope(const RopeParams* a, const RopeParams* b, bool bf16, cudaStream_t s) {
  const RopeParams none{};
  const RopeParams& pb = b ? *b : none;
  const int rows_a = a->T * (a->D / 16), rows_b = b ? b->T * (b->D / 16) : 0;
  const int xs = ((rows_a > rows_b ? rows_a : rows_b) + 255) / 256;
  const int ys = (b && b->Hc > a->Hc) ? b->Hc : a->Hc;
  const int zs = a->B + (b ? b->B : 0);
  if (xs == 0 || ys > 65535 || zs > 65535) return xs == 0 ? cudaSuccess : cudaErrorInvalidConfiguration;
  const dim3 grid(xs, ys, zs);
  if (bf16) {
    if (vec_ok(*a) && (!b || vec_ok(*b)))
      rope_bf16_vec_kernel<<<grid, 256, 0, s>>>(*a, pb);
    else
      rope_scalar_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(*a, pb);
  } else {
    rope_scalar_kernel<float><<<grid, 256, 0, s>>>(*a, pb);
  }
  return cudaGetLastError();
}

}  // namespace ltx
