// rotary.cu -- split-RoPE tables on the device (DiTForward.rotary,
// DiTForward.swift:641-678, with frequencyGrid :455-466).
//
// For token t and rotary pair j of the full inner/2 pairs:
//   j < pad:  (cos, sin) = (1, 0)                      leading identity pairs
//   else      k = j - pad, i = k / n_pos, d = k % n_pos (positional dim fastest)
//             freq[i] = (float)(theta^(i/(count-1)) * pi/2)   fp64, last exponent 1
//             middle  = (lo + hi) / 2,  frac = middle / max_pos[d]     fp32
//             angle   = freq[i] * (frac * 2 - 1)                      fp32
//             (cos, sin) = (cosf(angle), sinf(angle))                 fp32
// and pair j of head j / per lands at out[h][t][j % per], per = inner/2/heads.
// Every fp32 step is a separately rounded operation (no contraction), as the
// reference's array ops are; cosf/sinf are CUDA's accurate functions, so the
// fp32 tables agree with a host libm to within its and CUDA's ulp bounds.
#include "ltxattn_internal.h"

namespace ltx {
namespace {

template <typename T>
__device__ __forceinline__ void put(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void put<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void put<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// One block per token; the block's threads walk the inner/2 pairs.
template <typename T>
__global__ void __launch_bounds__(256) rotary_tables_kernel(const RotaryTableParams p) {
  const int t = blockIdx.x;
  const int half = p.inner / 2;
  const int per = half / p.heads;
  const int count = p.count;
  const double step = 1.0 / (double)(count - 1);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    float c = 1.f, s = 0.f;
    if (j >= p.pad) {
      const int k = j - p.pad, i = k / p.n_pos, d = k - (k / p.n_pos) * p.n_pos;
      const double e = (i == count - 1) ? 1.0 : (double)i * step;
      const float freq = (float)(pow(p.theta, e) * 3.14159265358979323846 / 2.0);
      const float lo = p.positions[((int64_t)d * p.tokens + t) * 2];
      const float hi = p.positions[((int64_t)d * p.tokens + t) * 2 + 1];
      const float middle = __fdiv_rn(__fadd_rn(lo, hi), 2.0f);
      const float frac = __fdiv_rn(middle, p.max_pos[d]);
      const float ang = __fmul_rn(freq, __fsub_rn(__fmul_rn(frac, 2.0f), 1.0f));
      sincosf(ang, &s, &c);
    }
    const int64_t o = ((int64_t)(j / per) * p.tokens + t) * per + (j % per);
    put(static_cast<T*>(p.cos), o, c);
    put(static_cast<T*>(p.sin), o, s);
  }
}

}  // namespace

cudaError_t launch_rotary_tables(const RotaryTableParams& p, bool bf16, cudaStream_t s) {
  if (p.tokens <= 0) return cudaSuccess;
  if (bf16)
    rotary_tables_kernel<__nv_bfloat16><<<p.tokens, 256, 0, s>>>(p);
  else
    rotary_tables_kernel<float><<<p.tokens, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ltx
