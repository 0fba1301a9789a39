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
// RoPE then rounds every product and sum to bf16 (bf16x2 arithmetic), or runs
// in plain fp32 for fp32 activations.
//
// Thread i of a row holds elements [16i, 16i + 16): 16 values of one half of
// one head (D / 16 threads per head, so a head's lower and upper halves sit
// D / 32 lanes apart in the same warp and RoPE pairs meet by warp shuffle).
// The mean square reduces in a fixed order (each thread's even and odd
// products in two sequential f32x2 lanes, warp shuffles, then warp partials in
// warp order), so results are deterministic.  Blocks walk rows with a grid stride; each thread keeps its
// weight slice in registers, loads the next row's x before working on the
// current one, and issues the current row's table loads before the reduction,
// so a block has two rows' loads in flight and one barrier per row.
#include <algorithm>

#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

#ifndef LTX_QK_MIN_BLOCKS_BF16
#define LTX_QK_MIN_BLOCKS_BF16 1
#endif

// 16 consecutive elements of one row: two (bf16) or four (fp32) 16-byte words.
template <typename T>
struct Raw16 {
  uint4 w[sizeof(T)];
};

template <typename T>
__device__ __forceinline__ void load16(Raw16<T>& r, const T* src, bool vec) {
  if (vec) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < (int)sizeof(T); ++i) r.w[i] = s4[i];
  } else {
    T* d = reinterpret_cast<T*>(r.w);
#pragma unroll
    for (int e = 0; e < 16; ++e) d[e] = src[e];
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* dst, const Raw16<T>& r, bool vec) {
  if (vec) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < (int)sizeof(T); ++i) d4[i] = r.w[i];
  } else {
    const T* d = reinterpret_cast<const T*>(r.w);
#pragma unroll
    for (int e = 0; e < 16; ++e) dst[e] = d[e];
  }
}

// y = T(w * T(x * r)), then split RoPE (lower half  out = y c - y' s,  upper
// half  out = y c + y' s,  y' = the partner lane's value of the same pair;
// products and sums rounded to T), stored to the thread's 16 output elements.
template <typename T>
__device__ __forceinline__ void finish_row(const Raw16<T>& xc, const Raw16<T>& wr, float r, bool rope,
                                           const Raw16<T>& cr, const Raw16<T>& sr, bool lower, int partner,
                                           T* out, bool vec) {
  Raw16<T> yr;
  if constexpr (sizeof(T) == 2) {
    // pairs: T(x r) by one f32x2 multiply and one packing conversion, then
    // T(w * that) as one bf16x2 multiply (the product of two bf16 values is
    // exact in fp32, so a single rounding gives the same bits)
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xc.w);
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(wr.w);
    uint32_t* yw = reinterpret_cast<uint32_t*>(yr.w);
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 xr = mul2(make_float2(__uint_as_float(xw[k] << 16), __uint_as_float(xw[k] & 0xffff0000u)), r2);
      yw[k] = bmul2(pack_bf16x2(xr.x, xr.y), ww[k]);
    }
  } else {
    T* y = reinterpret_cast<T*>(yr.w);
    const T* w = reinterpret_cast<const T*>(wr.w);
    const T* xe = reinterpret_cast<const T*>(xc.w);
#pragma unroll
    for (int e = 0; e < 16; ++e) y[e] = __fmul_rn(w[e], __fmul_rn(xe[e], r));
  }
  Raw16<T> outr = yr;
  if (rope) {
    Raw16<T> pr;
#pragma unroll
    for (int i = 0; i < (int)sizeof(T); ++i) {
      pr.w[i].x = __shfl_xor_sync(0xffffffffu, yr.w[i].x, partner);
      pr.w[i].y = __shfl_xor_sync(0xffffffffu, yr.w[i].y, partner);
      pr.w[i].z = __shfl_xor_sync(0xffffffffu, yr.w[i].z, partner);
      pr.w[i].w = __shfl_xor_sync(0xffffffffu, yr.w[i].w, partner);
    }
    if constexpr (sizeof(T) == 2) {
      const uint32_t* a = reinterpret_cast<const uint32_t*>(yr.w);
      const uint32_t* a2 = reinterpret_cast<const uint32_t*>(pr.w);
      const uint32_t* c = reinterpret_cast<const uint32_t*>(cr.w);
      const uint32_t* sn = reinterpret_cast<const uint32_t*>(sr.w);
      uint32_t* o = reinterpret_cast<uint32_t*>(outr.w);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t ac = bmul2(a[i], c[i]), ps = bmul2(a2[i], sn[i]);
        o[i] = lower ? bsub2(ac, ps) : badd2(ac, ps);
      }
    } else {
      const float* a = reinterpret_cast<const float*>(yr.w);
      const float* a2 = reinterpret_cast<const float*>(pr.w);
      const float* c = reinterpret_cast<const float*>(cr.w);
      const float* sn = reinterpret_cast<const float*>(sr.w);
      float* o = reinterpret_cast<float*>(outr.w);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float ac = __fmul_rn(a[e], c[e]), ps = __fmul_rn(a2[e], sn[e]);
        o[e] = lower ? __fsub_rn(ac, ps) : __fadd_rn(ac, ps);
      }
    }
  }
  store16<T>(out, outr, vec);
}

// Sum of squares of the thread's 16 values, then over the warp (fixed order:
// even and odd elements in two f32x2 lanes, in sequence, then their sum).
template <typename T>
__device__ __forceinline__ float warp_sumsq(const Raw16<T>& xc) {
  float ss;
  if constexpr (sizeof(T) == 2) {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xc.w);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 v = make_float2(__uint_as_float(xw[k] << 16), __uint_as_float(xw[k] & 0xffff0000u));
      acc = fma2(v, v, acc);
    }
    ss = acc.x + acc.y;
  } else {
    const float* xe = reinterpret_cast<const float*>(xc.w);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 v = make_float2(xe[2 * k], xe[2 * k + 1]);
      acc = fma2(v, v, acc);
    }
    ss = acc.x + acc.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return ss;
}

// Register path (any alignment): x of the next row is loaded into registers
// before the current row is worked on.
template <typename T>
__global__ void __launch_bounds__(512, sizeof(T) == 2 ? LTX_QK_MIN_BLOCKS_BF16 : 1) qk_prep_kernel(const QkPrepParams p) {
  grid_dep_launch_dependents();  // the attention kernel after this one may start its prologue
  __shared__ __align__(16) float wsum[2][16];  // per-warp partials, alternating by row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int rows = p.B * p.tokens;
  const int e0 = tid * 16;
  const int h = e0 / p.D, d0 = e0 - h * p.D;
  const int half = p.D / 2;
  const bool lower = d0 < half;  // holds x1 of its pairs (x2 sits D / 32 lanes up)
  const int j0 = lower ? d0 : d0 - half;
  const int partner = p.D / 32;
  const bool rope = p.cos != nullptr;

  Raw16<T> wr;  // the weight slice, kept packed
  load16<T>(wr, static_cast<const T*>(p.w) + e0, p.vec);

  int row = blockIdx.x;
  Raw16<T> xr;
  if (row < rows) {
    const int b = row / p.tokens, t = row - b * p.tokens;
    load16<T>(xr, static_cast<const T*>(p.x) + (int64_t)b * p.x_sb + (int64_t)t * p.x_st + e0, p.vec);
  }
  int par = 0;
  for (; row < rows; row += gridDim.x, par ^= 1) {
    const int b = row / p.tokens, t = row - b * p.tokens;
    Raw16<T> cr, sr;
    if (rope) {
      const int64_t toff = (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st + j0;
      load16<T>(cr, static_cast<const T*>(p.cos) + toff, p.vec);
      load16<T>(sr, static_cast<const T*>(p.sin) + toff, p.vec);
    }
    const Raw16<T> xc = xr;  // this row's x, packed
    const int nrow = row + gridDim.x;
    if (nrow < rows) {
      const int nb = nrow / p.tokens, nt = nrow - nb * p.tokens;
      load16<T>(xr, static_cast<const T*>(p.x) + (int64_t)nb * p.x_sb + (int64_t)nt * p.x_st + e0, p.vec);
    }
    const float ss = warp_sumsq<T>(xc);
    if (lane == 0) wsum[par][warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nwarps; ++i) tot += wsum[par][i];
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)p.inner), p.eps));
    T* out = static_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)t * p.o_st + d0;
    finish_row<T>(xc, wr, r, rope, cr, sr, lower, partner, out, p.vec);
  }
}

// Bulk path (16-byte aligned rows): thread 0 streams whole x rows into a ring
// of `stages` shared-memory rows with 1-D bulk copies (cp.async.bulk, one
// mbarrier per stage), so each block keeps up to `stages` rows in flight; a
// stage is refilled as soon as the block's per-row barrier shows that every
// thread has read it.  Waits are bounded; a wait that gives up ends every
// thread of the block at that row's barrier, and thread 0 drains the copies
// still in flight before the block exits.
// The bulk path for one tensor, run by blocks [0, G) of the job (blk is this
// block's index among them); inlined into the single and the paired kernels.
template <typename T>
__device__ __forceinline__ void qk_prep_bulk_body(const QkPrepParams& p, int stages, int blk, int G,
                                                  uint8_t* smem_raw, float (*wsum)[16], int& abort_flag) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int rows = p.B * p.tokens;
  const uint32_t row_bytes = (uint32_t)p.inner * sizeof(T);
  T* ring = reinterpret_cast<T*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)stages * row_bytes);
  const int e0 = tid * 16;
  const int h = e0 / p.D, d0 = e0 - h * p.D;
  const int half = p.D / 2;
  const bool lower = d0 < half;
  const int j0 = lower ? d0 : d0 - half;
  const int partner = p.D / 32;
  const bool rope = p.cos != nullptr;
  auto row_src = [&](int r) {
    const int b = r / p.tokens, t = r - b * p.tokens;
    return static_cast<const T*>(p.x) + (int64_t)b * p.x_sb + (int64_t)t * p.x_st;
  };

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(full + s, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // pipeline slots whose copy thread 0 has issued (slot k: row blk + k * G)
  if (tid == 0) {
    for (; issued < stages && blk + issued * G < rows; ++issued) {
      mbar_arrive_expect_tx(full + issued, row_bytes);
      bulk_load(ring + (size_t)issued * p.inner, row_src(blk + issued * G), row_bytes, full + issued);
    }
  }
  Raw16<T> wr;
  load16<T>(wr, static_cast<const T*>(p.w) + e0, true);

  // mean = tot / inner: for a power-of-two width the product with 1 / inner is
  // the same correctly rounded value (the exact quotient is a scaling by 2^-k)
  const bool inner_pow2 = (p.inner & (p.inner - 1)) == 0;
  const float inv_inner = 1.0f / (float)p.inner;
  int i = 0, par = 0;
  int b = blk / p.tokens, t = blk - b * p.tokens;  // (batch, token) of `row`, advanced without a division
  int s = 0;                                       // ring stage of slot i (i % stages) ...
  uint32_t ph = 0;                                 // ... and its phase parity ((i / stages) & 1)
  for (int row = blk; row < rows; row += G, ++i, par ^= 1) {
    if (i > 0) {
      t += G;
      while (t >= p.tokens) {
        t -= p.tokens;
        ++b;
      }
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    Raw16<T> cr, sr;
    if (rope) {
      const int64_t toff = (int64_t)b * p.t_sb + (int64_t)h * p.t_sh + (int64_t)t * p.t_st + j0;
      load16<T>(cr, static_cast<const T*>(p.cos) + toff, true);
      load16<T>(sr, static_cast<const T*>(p.sin) + toff, true);
    }
    const bool ok = mbar_wait(full + s, ph, (volatile int*)&abort_flag, p.err, 40);
    Raw16<T> xc;
    if (ok) {
      const uint4* src = reinterpret_cast<const uint4*>(ring + (size_t)s * p.inner + e0);
#pragma unroll
      for (int k = 0; k < (int)sizeof(T); ++k) xc.w[k] = src[k];
    } else {
#pragma unroll
      for (int k = 0; k < (int)sizeof(T); ++k) xc.w[k] = make_uint4(0u, 0u, 0u, 0u);
    }
    const float ss = warp_sumsq<T>(xc);
    if (lane == 0) wsum[par][warp] = ss;
    if (!__syncthreads_and(ok)) break;
    // every thread has read stage s: refill it with slot i + stages
    if (tid == 0 && issued == i + stages && blk + issued * G < rows) {
      mbar_arrive_expect_tx(full + s, row_bytes);
      bulk_load(ring + (size_t)s * p.inner, row_src(blk + issued * G), row_bytes, full + s);
      ++issued;
    }
    // the warp partials in warp order (16-byte reads, the same sums)
    float tot = 0.f;
    {
      const float4* w4 = reinterpret_cast<const float4*>(wsum[par]);
      int k = 0;
      for (; k + 4 <= nwarps; k += 4) {
        const float4 a = w4[k >> 2];
        tot += a.x;
        tot += a.y;
        tot += a.z;
        tot += a.w;
      }
      for (; k < nwarps; ++k) tot += wsum[par][k];
    }
    const float mean = inner_pow2 ? __fmul_rn(tot, inv_inner) : __fdiv_rn(tot, (float)p.inner);
    const float r = 1.0f / sqrtf(__fadd_rn(mean, p.eps));
    T* out = static_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)t * p.o_st + d0;
    finish_row<T>(xc, wr, r, rope, cr, sr, lower, partner, out, true);
  }
  // never leave with a bulk copy still writing this block's shared memory
  if (tid == 0)
    for (int k = i; k < issued; ++k) drain_wait(full + k % stages, (uint32_t)(k / stages) & 1u);
}


template <typename T>
__global__ void __launch_bounds__(512) qk_prep_bulk_kernel(const QkPrepParams p, int stages) {
  grid_dep_launch_dependents();  // the attention kernel after this one may start its prologue
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(16) float wsum[2][16];
  __shared__ int abort_flag;
  qk_prep_bulk_body<T>(p, stages, blockIdx.x, gridDim.x, smem_raw, wsum, abort_flag);
}

// q and k in one launch: blocks [0, g0) prepare p0, the rest p1.
template <typename T>
__global__ void __launch_bounds__(512) qk_prep_bulk_pair_kernel(const QkPrepParams p0, const QkPrepParams p1,
                                                                 int stages, int g0) {
  grid_dep_launch_dependents();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ __align__(16) float wsum[2][16];
  __shared__ int abort_flag;
  if ((int)blockIdx.x < g0)
    qk_prep_bulk_body<T>(p0, stages, blockIdx.x, g0, smem_raw, wsum, abort_flag);
  else
    qk_prep_bulk_body<T>(p1, stages, blockIdx.x - g0, gridDim.x - g0, smem_raw, wsum, abort_flag);
}

}  // namespace

cudaError_t launch_qk_prep(const QkPrepParams& p, bool bf16, cudaStream_t s) {
  const int rows = p.B * p.tokens;
  if (rows == 0) return cudaSuccess;
  const int threads = p.inner / 16;
  int dev = 0, sms = 148, per_sm = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // bulk path: as many row stages (<= 8) as fit in 47 KB of dynamic shared memory
  const size_t row_bytes = (size_t)p.inner * (bf16 ? 2 : 4);
  const int stages = (int)std::min<size_t>(8, (47 * 1024) / (row_bytes + 8));
  cudaError_t e;
  if (p.vec && stages >= 2) {
    const size_t smem = (size_t)stages * (row_bytes + 8);
    e = bf16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_bulk_kernel<__nv_bfloat16>, threads, smem)
             : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_bulk_kernel<float>, threads, smem);
    if (e != cudaSuccess) return e;
    const int grid = std::min(rows, std::max(1, per_sm) * sms);
    if (bf16)
      qk_prep_bulk_kernel<__nv_bfloat16><<<grid, threads, smem, s>>>(p, stages);
    else
      qk_prep_bulk_kernel<float><<<grid, threads, smem, s>>>(p, stages);
    return cudaGetLastError();
  }
  e = bf16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_kernel<__nv_bfloat16>, threads, 0)
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_kernel<float>, threads, 0);
  if (e != cudaSuccess) return e;
  const int grid = std::min(rows, std::max(1, per_sm) * sms);
  if (bf16)
    qk_prep_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(p);
  else
    qk_prep_kernel<float><<<grid, threads, 0, s>>>(p);
  return cudaGetLastError();
}

// q and k (same dtype and inner width; token counts may differ) in one launch;
// shapes the bulk path cannot take run as two launches.
cudaError_t launch_qk_prep_pair(const QkPrepParams& p0, const QkPrepParams& p1, bool bf16, cudaStream_t s) {
  const int64_t rows0 = (int64_t)p0.B * p0.tokens, rows1 = (int64_t)p1.B * p1.tokens;
  const size_t row_bytes = (size_t)p0.inner * (bf16 ? 2 : 4);
  const int stages = (int)std::min<size_t>(8, (47 * 1024) / (row_bytes + 8));
  if (rows0 == 0 || rows1 == 0 || !p0.vec || !p1.vec || stages < 2 || p0.inner != p1.inner) {
    cudaError_t e = launch_qk_prep(p0, bf16, s);
    return e != cudaSuccess ? e : launch_qk_prep(p1, bf16, s);
  }
  const int threads = p0.inner / 16;
  int dev = 0, sms = 148, per_sm = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = (size_t)stages * (row_bytes + 8);
  cudaError_t e = bf16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_bulk_pair_kernel<__nv_bfloat16>, threads, smem)
                       : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_prep_bulk_pair_kernel<float>, threads, smem);
  if (e != cudaSuccess) return e;
  const int grid = (int)std::min<int64_t>(rows0 + rows1, (int64_t)std::max(1, per_sm) * sms);
  if (grid < 2) {
    e = launch_qk_prep(p0, bf16, s);
    return e != cudaSuccess ? e : launch_qk_prep(p1, bf16, s);
  }
  // blocks in proportion to rows, at least one per job and none beyond a job's rows
  int g0 = (int)((grid * rows0 + (rows0 + rows1) / 2) / (rows0 + rows1));
  g0 = (int)std::min<int64_t>(std::max(1, std::min(g0, grid - 1)), rows0);
  const int g1 = (int)std::min<int64_t>(grid - g0, rows1);
  if (bf16)
    qk_prep_bulk_pair_kernel<__nv_bfloat16><<<g0 + g1, threads, smem, s>>>(p0, p1, stages, g0);
  else
    qk_prep_bulk_pair_kernel<float><<<g0 + g1, threads, smem, s>>>(p0, p1, stages, g0);
  return cudaGetLastError();
}

}  // namespace ltx
