// qkprep.cu -- the query / key preparation between a projection and the
// attention, in one pass (DiTAttention.swift:358-367):
//
//   q = rmsNorm(q_raw, weight)      over the whole inner dim (:190-204), eps
//   qh = split(q)                   [B, T, H*D] -> [B, H, T, D]      (:346-348)
//   qh = applySplitRoPE(qh, rotary) per-head tables                  (:206-234)
//
// rmsNorm follows the MLX kernel's arithmetic: the mean square accumulates in
// fp32, r = 1 / sqrt(mean + eps), each element is normalised in fp32 and cast
// to the activation dtype, then multiplied by the weight (also cast):
//   y = T(w * T(x * r)).
// RoPE then rounds every product and sum to bf16 (rope_bf16x8), or runs in
// plain fp32 for fp32 activations.
//
// One block per token row; inner / 16 threads hold 16 elements each.  The
// mean square reduces in a fixed order (warp shuffles, then warp partials in
// warp order), so results are deterministic.  The normalised row is staged in
// shared memory so that each thread can take 8 rotary pairs (d, d + D/2) of
// one head; the outputs go straight into the [B, H, T, D] view.
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename T>
__device__ __forceinline__ float tof(T v);
template <>
__device__ __forceinline__ float tof<float>(float v) { return v; }
template <>
__device__ __forceinline__ float tof<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ float cast_t(float v);
template <>
__device__ __forceinline__ float cast_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ float cast_t<__nv_bfloat16>(float v) { return bf16r(v); }

template <typename T>
__device__ __forceinline__ void store_t(T* p, float v);
template <>
__device__ __forceinline__ void store_t<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_t<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(512) qk_prep_kernel(const QkPrepParams p) {
  extern __shared__ uint8_t smem_raw[];
  T* srow = reinterpret_cast<T*>(smem_raw);                  // the normalised row
  float* wsum = reinterpret_cast<float*>(smem_raw + (size_t)p.inner * sizeof(T));  // per-warp partials
  const int row = blockIdx.x;  // b * T + t
  const int b = row / p.tokens, t = row - (row / p.tokens) * p.tokens;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* x = static_cast<const T*>(p.x) + (int64_t)b * p.x_sb + (int64_t)t * p.x_st;
  const T* w = static_cast<const T*>(p.w);

  // 1. mean square of the row (fp32), fixed reduction order
  float xv[16], wv[16];
  bool loaded = false;
  if constexpr (sizeof(T) == 2) {
    if (p.vec) {  // 16-byte rows: two vector loads each for x and the weight
      const uint4* xs = reinterpret_cast<const uint4*>(x + tid * 16);
      const uint4* ws = reinterpret_cast<const uint4*>(w + tid * 16);
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const uint4 a = xs[v], c = __ldg(ws + v);
        const uint32_t au[4] = {a.x, a.y, a.z, a.w}, cu[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          xv[8 * v + 2 * k] = __uint_as_float(au[k] << 16);
          xv[8 * v + 2 * k + 1] = __uint_as_float(au[k] & 0xffff0000u);
          wv[8 * v + 2 * k] = __uint_as_float(cu[k] << 16);
          wv[8 * v + 2 * k + 1] = __uint_as_float(cu[k] & 0xffff0000u);
        }
      }
      loaded = true;
    }
  }
  if (!loaded) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      xv[e] = tof<T>(x[tid * 16 + e]);
      wv[e] = tof<T>(w[tid * 16 + e]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) ss = fmaf(xv[e], xv[e], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) wsum[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += wsum[i];
  const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)p.inner), p.eps));

  // 2. y = T(w * T(x * r)) into shared memory
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int i = tid * 16 + e;
    const float n = cast_t<T>(__fmul_rn(xv[e], r));
    store_t<T>(srow + i, __fmul_rn(wv[e], n));
  }
  __syncthreads();

  // 3. head split (+ split RoPE): thread tid takes 8 pairs (d, d + D/2) of one head
  const int half = p.D / 2;
  const int groups = half / 8;  // 8-pair groups per head
  const int h = tid / groups, j0 = (tid - h * groups) * 8;
  const T* y1 = srow + h * p.D + j0;
  const T* y2 = y1 + half;
  T* o = static_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)t * p.o_st + j0;
  if (p.cos == nullptr) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o[e] = y1[e];
      o[half + e] = y2[e];
    }
    return;
  }
  const int64_t toff = (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st + j0;
  const T* cs = static_cast<const T*>(p.cos) + toff;
  const T* sn = static_cast<const T*>(p.sin) + toff;
  if constexpr (sizeof(T) == 2) {
    if (p.vec) {
      const uint4 a1 = *reinterpret_cast<const uint4*>(y1), a2 = *reinterpret_cast<const uint4*>(y2);
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(cs)), s = __ldg(reinterpret_cast<const uint4*>(sn));
      uint4 o1, o2;
      rope_bf16x8(a1, a2, c, s, o1, o2);
      *reinterpret_cast<uint4*>(o) = o1;
      *reinterpret_cast<uint4*>(o + half) = o2;
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a1 = tof<T>(y1[e]), a2 = tof<T>(y2[e]), c = tof<T>(cs[e]), s = tof<T>(sn[e]);
    const float o1 = cast_t<T>(__fsub_rn(cast_t<T>(__fmul_rn(a1, c)), cast_t<T>(__fmul_rn(a2, s))));
    const float o2 = cast_t<T>(__fadd_rn(cast_t<T>(__fmul_rn(a2, c)), cast_t<T>(__fmul_rn(a1, s))));
    store_t<T>(o + e, o1);
    store_t<T>(o + half + e, o2);
  }
}

}  // namespace

cudaError_t launch_qk_prep(const QkPrepParams& p, bool bf16, cudaStream_t s) {
  const int rows = p.B * p.tokens;
  if (rows == 0) return cudaSuccess;
  const int threads = p.inner / 16;
  const size_t smem = (size_t)p.inner * (bf16 ? 2 : 4) + 32 * sizeof(float);
  if (bf16)
    qk_prep_kernel<__nv_bfloat16><<<rows, threads, smem, s>>>(p);
  else
    qk_prep_kernel<float><<<rows, threads, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ltx
