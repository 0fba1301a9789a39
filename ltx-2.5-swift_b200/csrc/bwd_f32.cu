// bwd_f32.cu -- float32 attention backward on the CUDA cores.
//
// The float32 twin of bwd_sm100.cu (same closed-form VJP, same two-kernel
// deterministic split, P recomputed from the saved natural-log lse), for the
// float32 dtype where tcgen05 has no exact kind.  Accurate expf throughout.
//
//   bwd_f32_dq_kernel    32 query rows per CTA (8 per warp), loop over 64-key tiles
//   bwd_f32_dkdv_kernel  32 key rows per CTA (8 per warp), loop over 64-query tiles
// Shared-memory rows of the streamed operand are padded by one word so the
// per-lane dot products are bank-conflict free.
#include "ltxattn_internal.h"

namespace ltx {
namespace {

constexpr int kRows = 32, kCols = 64, kRpw = 8;

template <int D>
__device__ __forceinline__ void rope_inverse_lane(float (&g)[D / 32], const float* c, const float* s, int lane) {
  // lane owns d = lane + 32e; pairs (d, d + D/2) sit in e and e + D/64
#pragma unroll
  for (int e = 0; e < D / 64; ++e) {
    const int i = lane + 32 * e;
    const float cc = c[i], ss = s[i];
    const float g1 = g[e], g2 = g[e + D / 64];
    g[e] = __fadd_rn(__fmul_rn(g1, cc), __fmul_rn(g2, ss));
    g[e + D / 64] = __fsub_rn(__fmul_rn(g2, cc), __fmul_rn(g1, ss));
  }
}

__device__ __forceinline__ bool unmasked_row(const BwdParams& p, int b) {
  int local = 0;
  if (p.mask)
    for (int j = threadIdx.x; j < p.Lk; j += blockDim.x) local |= (p.mask[(int64_t)b * p.mask_sb + j] != 0);
  return __syncthreads_or(local) == 0;  // true: no valid key -> attend to all
}

template <int D>
__global__ void __launch_bounds__(128) bwd_f32_dq_kernel(const BwdParams p) {
  extern __shared__ float sm[];
  float* sQ = sm;                        // [kRows][D]
  float* sDO = sQ + kRows * D;           // [kRows][D]
  float* sK = sDO + kRows * D;           // [kCols][D+1]
  float* sV = sK + kCols * (D + 1);      // [kCols][D+1]
  float* sDS = sV + kCols * (D + 1);     // [4][kRpw][kCols]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = blockIdx.y, b = blockIdx.z, q0 = blockIdx.x * kRows;
  const bool use_mask = p.mask != nullptr && !unmasked_row(p, b);
  const float* qb = p.q + (int64_t)b * p.q_sb + (int64_t)hl * p.q_sh;
  const float* gb = p.dout + (int64_t)b * p.do_sb + (int64_t)hl * p.do_sh;
  const float* kb = p.k + (int64_t)b * p.k_sb + (int64_t)hl * p.k_sh;
  const float* vb = p.v + (int64_t)b * p.v_sb + (int64_t)hl * p.v_sh;
  for (int i = threadIdx.x; i < kRows * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    const bool in = q0 + r < p.Lq;
    sQ[i] = in ? qb[(int64_t)(q0 + r) * p.q_st + d] : 0.f;
    sDO[i] = in ? gb[(int64_t)(q0 + r) * p.do_st + d] : 0.f;
  }
  constexpr int kPer = D / 32;
  float lse[kRpw], del[kRpw], acc[kRpw][kPer];
  const int64_t lrow = ((int64_t)b * gridDim.y + hl) * p.Lq_pad + q0 + warp * kRpw;
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    lse[r] = p.lse2[lrow + r];  // natural-log lse; +inf on padded rows
    del[r] = p.delta[lrow + r];
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[r][e] = 0.f;
  }
  float* myDS = sDS + warp * kRpw * kCols;
  for (int kv0 = 0; kv0 < p.Lk; kv0 += kCols) {
    __syncthreads();
    for (int i = threadIdx.x; i < kCols * D; i += blockDim.x) {
      const int j = i / D, d = i % D;
      const bool in = kv0 + j < p.Lk;
      sK[j * (D + 1) + d] = in ? kb[(int64_t)(kv0 + j) * p.k_st + d] : 0.f;
      sV[j * (D + 1) + d] = in ? vb[(int64_t)(kv0 + j) * p.v_st + d] : 0.f;
    }
    __syncthreads();
    const int j0 = kv0 + lane, j1 = kv0 + lane + 32;
    const bool ok0 = j0 < p.Lk && (!use_mask || p.mask[(int64_t)b * p.mask_sb + j0] != 0);
    const bool ok1 = j1 < p.Lk && (!use_mask || p.mask[(int64_t)b * p.mask_sb + j1] != 0);
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      const float* qr = sQ + (warp * kRpw + r) * D;
      const float* gr = sDO + (warp * kRpw + r) * D;
      const float* k0 = sK + lane * (D + 1);
      const float* k1 = sK + (lane + 32) * (D + 1);
      const float* v0 = sV + lane * (D + 1);
      const float* v1 = sV + (lane + 32) * (D + 1);
      float s0 = 0.f, s1 = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        s0 = fmaf(qr[d], k0[d], s0);
        s1 = fmaf(qr[d], k1[d], s1);
        d0 = fmaf(gr[d], v0[d], d0);
        d1 = fmaf(gr[d], v1[d], d1);
      }
      const float p0 = ok0 ? expf(s0 * p.scale - lse[r]) : 0.f;
      const float p1 = ok1 ? expf(s1 * p.scale - lse[r]) : 0.f;
      myDS[r * kCols + lane] = p0 * (d0 - del[r]);
      myDS[r * kCols + lane + 32] = p1 * (d1 - del[r]);
    }
    __syncwarp();
    for (int j = 0; j < kCols; ++j) {
      float kk[kPer];
#pragma unroll
      for (int e = 0; e < kPer; ++e) kk[e] = sK[j * (D + 1) + lane + 32 * e];
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const float ds = myDS[r * kCols + j];
#pragma unroll
        for (int e = 0; e < kPer; ++e) acc[r][e] = fmaf(ds, kk[e], acc[r][e]);
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    const int row = q0 + warp * kRpw + r;
    if (row >= p.Lq) continue;
    float g[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) g[e] = acc[r][e] * p.scale;
    if (p.qcos)
      rope_inverse_lane<D>(g, static_cast<const float*>(p.qcos) + (int64_t)b * p.qt_sb + (int64_t)hl * p.qt_sh + (int64_t)row * p.qt_st,
                           static_cast<const float*>(p.qsin) + (int64_t)b * p.qt_sb + (int64_t)hl * p.qt_sh + (int64_t)row * p.qt_st,
                           lane);
    float* dst = static_cast<float*>(p.dq) + (int64_t)b * p.dq_sb + (int64_t)hl * p.dq_sh + (int64_t)row * p.dq_st;
#pragma unroll
    for (int e = 0; e < kPer; ++e) dst[lane + 32 * e] = g[e];
  }
}

template <int D>
__global__ void __launch_bounds__(128) bwd_f32_dkdv_kernel(const BwdParams p) {
  extern __shared__ float sm[];
  float* sK = sm;                        // [kRows][D]  (stationary keys)
  float* sV = sK + kRows * D;            // [kRows][D]
  float* sQ = sV + kRows * D;            // [kCols][D+1] (streamed queries)
  float* sG = sQ + kCols * (D + 1);      // [kCols][D+1]
  float* sP = sG + kCols * (D + 1);      // [4][kRpw][kCols]
  float* sS = sP + 4 * kRpw * kCols;     // [4][kRpw][kCols] dS^T
  float* sL = sS + 4 * kRpw * kCols;     // [kCols] lse
  float* sD = sL + kCols;                // [kCols] delta
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = blockIdx.y, b = blockIdx.z, k0r = blockIdx.x * kRows;
  const bool use_mask = p.mask != nullptr && !unmasked_row(p, b);
  const float* qb = p.q + (int64_t)b * p.q_sb + (int64_t)hl * p.q_sh;
  const float* gb = p.dout + (int64_t)b * p.do_sb + (int64_t)hl * p.do_sh;
  const float* kb = p.k + (int64_t)b * p.k_sb + (int64_t)hl * p.k_sh;
  const float* vb = p.v + (int64_t)b * p.v_sb + (int64_t)hl * p.v_sh;
  for (int i = threadIdx.x; i < kRows * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    const bool in = k0r + r < p.Lk;
    sK[i] = in ? kb[(int64_t)(k0r + r) * p.k_st + d] : 0.f;
    sV[i] = in ? vb[(int64_t)(k0r + r) * p.v_st + d] : 0.f;
  }
  constexpr int kPer = D / 32;
  bool kval[kRpw];
  float dv[kRpw][kPer], dk[kRpw][kPer];
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    const int key = k0r + warp * kRpw + r;
    kval[r] = key < p.Lk && (!use_mask || p.mask[(int64_t)b * p.mask_sb + key] != 0);
#pragma unroll
    for (int e = 0; e < kPer; ++e) dv[r][e] = dk[r][e] = 0.f;
  }
  const int64_t lrow = ((int64_t)b * gridDim.y + hl) * p.Lq_pad;
  float* myP = sP + warp * kRpw * kCols;
  float* myS = sS + warp * kRpw * kCols;
  for (int q0 = 0; q0 < p.Lq; q0 += kCols) {
    __syncthreads();
    for (int i = threadIdx.x; i < kCols * D; i += blockDim.x) {
      const int j = i / D, d = i % D;
      const bool in = q0 + j < p.Lq;
      sQ[j * (D + 1) + d] = in ? qb[(int64_t)(q0 + j) * p.q_st + d] : 0.f;
      sG[j * (D + 1) + d] = in ? gb[(int64_t)(q0 + j) * p.do_st + d] : 0.f;
    }
    for (int j = threadIdx.x; j < kCols; j += blockDim.x) {
      sL[j] = p.lse2[lrow + q0 + j];  // padded to whole 128-row tiles: in range
      sD[j] = p.delta[lrow + q0 + j];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kRpw; ++r) {
      const float* kr = sK + (warp * kRpw + r) * D;
      const float* vr = sV + (warp * kRpw + r) * D;
      const float* qa = sQ + lane * (D + 1);
      const float* qc = sQ + (lane + 32) * (D + 1);
      const float* ga = sG + lane * (D + 1);
      const float* gc = sG + (lane + 32) * (D + 1);
      float s0 = 0.f, s1 = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        s0 = fmaf(kr[d], qa[d], s0);
        s1 = fmaf(kr[d], qc[d], s1);
        d0 = fmaf(vr[d], ga[d], d0);
        d1 = fmaf(vr[d], gc[d], d1);
      }
      const float p0 = kval[r] ? expf(s0 * p.scale - sL[lane]) : 0.f;       // +inf lse on padding -> 0
      const float p1 = kval[r] ? expf(s1 * p.scale - sL[lane + 32]) : 0.f;
      myP[r * kCols + lane] = p0;
      myP[r * kCols + lane + 32] = p1;
      myS[r * kCols + lane] = p0 * (d0 - sD[lane]);
      myS[r * kCols + lane + 32] = p1 * (d1 - sD[lane + 32]);
    }
    __syncwarp();
    for (int j = 0; j < kCols; ++j) {
      float qq[kPer], gg[kPer];
#pragma unroll
      for (int e = 0; e < kPer; ++e) {
        qq[e] = sQ[j * (D + 1) + lane + 32 * e];
        gg[e] = sG[j * (D + 1) + lane + 32 * e];
      }
#pragma unroll
      for (int r = 0; r < kRpw; ++r) {
        const float pj = myP[r * kCols + j], sj = myS[r * kCols + j];
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          dv[r][e] = fmaf(pj, gg[e], dv[r][e]);
          dk[r][e] = fmaf(sj, qq[e], dk[r][e]);
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < kRpw; ++r) {
    const int key = k0r + warp * kRpw + r;
    if (key >= p.Lk) continue;
    float* dvp = static_cast<float*>(p.dv) + (int64_t)b * p.dv_sb + (int64_t)hl * p.dv_sh + (int64_t)key * p.dv_st;
#pragma unroll
    for (int e = 0; e < kPer; ++e) dvp[lane + 32 * e] = dv[r][e];
    float g[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) g[e] = dk[r][e] * p.scale;
    if (p.kcos)
      rope_inverse_lane<D>(g, static_cast<const float*>(p.kcos) + (int64_t)b * p.kt_sb + (int64_t)hl * p.kt_sh + (int64_t)key * p.kt_st,
                           static_cast<const float*>(p.ksin) + (int64_t)b * p.kt_sb + (int64_t)hl * p.kt_sh + (int64_t)key * p.kt_st,
                           lane);
    float* dkp = static_cast<float*>(p.dk) + (int64_t)b * p.dk_sb + (int64_t)hl * p.dk_sh + (int64_t)key * p.dk_st;
#pragma unroll
    for (int e = 0; e < kPer; ++e) dkp[lane + 32 * e] = g[e];
  }
}

template <int D>
cudaError_t launch_d(const BwdParams& p, int Hc, int B, cudaStream_t s) {
  const size_t sq = sizeof(float) * (2 * kRows * D + 2 * kCols * (D + 1) + 4 * kRpw * kCols);
  const size_t skv = sizeof(float) * (2 * kRows * D + 2 * kCols * (D + 1) + 8 * kRpw * kCols + 2 * kCols);
  cudaError_t e = cudaFuncSetAttribute(bwd_f32_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sq);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(bwd_f32_dkdv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)skv);
  if (e != cudaSuccess) return e;
  bwd_f32_dq_kernel<D><<<dim3((p.Lq + kRows - 1) / kRows, Hc, B), 128, sq, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  bwd_f32_dkdv_kernel<D><<<dim3((p.Lk + kRows - 1) / kRows, Hc, B), 128, skv, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_f32(const BwdParams& p, int D, int Hc, int B, cudaStream_t s) {
  return D == 128 ? launch_d<128>(p, Hc, B, s) : launch_d<64>(p, Hc, B, s);
}

}  // namespace ltx
