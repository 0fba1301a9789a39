// fwd_f32.cu -- float32 fused attention forward (CUDA cores).
//
// The float32 dtype is the reference's `.explicit` arithmetic
// (DiTAttention.swift:377-381: fp32 logits, softmax, PV) and BASELINE's parity
// gate (config 1, max abs error 1e-5).  tcgen05 has no fp32 kind (tf32 would
// miss 1e-5), so this path runs on the FP32 pipes with the same online-softmax
// structure as the bf16 kernel and accurate expf.
//
// CTA: 128 threads for 32 query rows of one (batch, head); each warp owns 8
// rows.  KV tiles of 64 keys are staged in shared memory (K rows padded by one
// word so the per-lane dot products are bank-conflict free).
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

constexpr int kRows = 32;
constexpr int kKeys = 64;
constexpr int kRowsPerWarp = 8;

template <int D>
__global__ void __launch_bounds__(128) fwd_f32_kernel(const F32Params p) {
  extern __shared__ float sm[];
  float* sQ = sm;                              // [kRows][D]
  float* sK = sQ + kRows * D;                  // [kKeys][D+1]
  float* sV = sK + kKeys * (D + 1);            // [kKeys][D]
  float* sP = sV + kKeys * D;                  // [4][kRowsPerWarp][kKeys]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * kRows;
  const int Lk = p.Lk;
  const float* qb = p.q + (int64_t)b * p.q_sb + (int64_t)(p.q_head_off + hl) * p.q_sh;
  const int kvh = (p.kv_head_off + hl) / p.group;  // grouped heads share a kv head
  const float* kb = p.k + (int64_t)b * p.k_sb + (int64_t)kvh * p.k_sh;
  const float* vb = p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh;
  const uint8_t* mrow = p.mask ? p.mask + (int64_t)b * p.mask_sb : nullptr;

  // unmask rule: a batch row with no valid key attends to every key
  int local = 0;
  if (mrow)
    for (int j = threadIdx.x; j < Lk; j += blockDim.x) local |= (mrow[j] != 0);
  const int any_valid = __syncthreads_or(local);
  const bool use_mask = mrow != nullptr && any_valid != 0;

  for (int i = threadIdx.x; i < kRows * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    sQ[i] = (q0 + r < p.Lq) ? qb[(int64_t)(q0 + r) * p.q_st + d] : 0.f;
  }
  // causal / sliding rows (GemmaTextEncoder.swift:292-323): row i attends key j
  // when j <= i and i - j < window; a row left with no such valid key attends
  // every key.  free_row[r]: this warp's row r is such an un-masked row.
  bool free_row[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) free_row[r] = false;
  // a batch row whose mask has no valid key leaves every query row without keys
  const bool batch_empty = mrow != nullptr && any_valid == 0;
  const bool banded = p.causal || p.window > 0 || batch_empty;
  if (batch_empty) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) free_row[r] = true;
  } else if (banded) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int row = q0 + warp * kRowsPerWarp + r;
      const int lo = p.window > 0 ? max(0, row - p.window + 1) : 0;
      const int hi = p.causal ? min(row, Lk - 1) : Lk - 1;
      int any = 0;
      for (int j = lo + lane; j <= hi; j += 32) any |= (!use_mask || mrow[j] != 0);
      free_row[r] = __any_sync(0xffffffffu, any) == 0;
    }
  }

  constexpr int kPer = D / 32;
  float m[kRowsPerWarp], l[kRowsPerWarp], o[kRowsPerWarp][kPer];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < kPer; ++e) o[r][e] = 0.f;
  }
  float* myP = sP + warp * kRowsPerWarp * kKeys;

  for (int kv0 = 0; kv0 < Lk; kv0 += kKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKeys * D; i += blockDim.x) {
      const int j = i / D, d = i % D;
      const bool in = kv0 + j < Lk;
      sK[j * (D + 1) + d] = in ? kb[(int64_t)(kv0 + j) * p.k_st + d] : 0.f;
      sV[j * D + d] = in ? vb[(int64_t)(kv0 + j) * p.v_st + d] : 0.f;
    }
    __syncthreads();
    const int j0 = kv0 + lane, j1 = kv0 + lane + 32;
    const bool ok0 = j0 < Lk && (!use_mask || mrow[j0] != 0);
    const bool ok1 = j1 < Lk && (!use_mask || mrow[j1] != 0);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const float* qr = sQ + (warp * kRowsPerWarp + r) * D;
      const float* k0 = sK + lane * (D + 1);
      const float* k1 = sK + (lane + 32) * (D + 1);
      float a0 = 0.f, a1 = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) {
        const float qd = qr[d];
        a0 = fmaf(qd, k0[d], a0);
        a1 = fmaf(qd, k1[d], a1);
      }
      bool k0ok = ok0, k1ok = ok1;
      if (banded) {
        const int row = q0 + warp * kRowsPerWarp + r;
        if (free_row[r]) {
          k0ok = j0 < Lk;
          k1ok = j1 < Lk;
        } else {
          k0ok = ok0 && (!p.causal || j0 <= row) && (p.window <= 0 || row - j0 < p.window);
          k1ok = ok1 && (!p.causal || j1 <= row) && (p.window <= 0 || row - j1 < p.window);
        }
      }
      const float s0 = k0ok ? a0 * p.scale : -INFINITY;
      const float s1 = k1ok ? a1 * p.scale : -INFINITY;
      float mt = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m[r], mt);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float corr = expf(m[r] - m_use);  // m[r] = -inf -> 0
      const float p0 = expf(s0 - m_use), p1 = expf(s1 - m_use);
      float ps = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[r] = l[r] * corr + ps;
      m[r] = m_new;
#pragma unroll
      for (int e = 0; e < kPer; ++e) o[r][e] *= corr;
      myP[r * kKeys + lane] = p0;
      myP[r * kKeys + lane + 32] = p1;
    }
    __syncwarp();
    for (int j = 0; j < kKeys; ++j) {
      float vv[kPer];
#pragma unroll
      for (int e = 0; e < kPer; ++e) vv[e] = sV[j * D + lane + 32 * e];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const float pj = myP[r * kKeys + j];
#pragma unroll
        for (int e = 0; e < kPer; ++e) o[r][e] = fmaf(pj, vv[e], o[r][e]);
      }
    }
    __syncwarp();
  }

#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int row = q0 + warp * kRowsPerWarp + r;
    if (row >= p.Lq) continue;
    const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
    float* orow = p.out + (int64_t)b * p.o_sb + (int64_t)(p.head_begin + hl) * p.o_sh + (int64_t)row * p.o_st;
    const float g = p.gate == nullptr ? 1.f
                    : gate_f32(p.gate[(int64_t)b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + hl) * p.g_sh]);
#pragma unroll
    for (int e = 0; e < kPer; ++e) orow[lane + 32 * e] = p.gate == nullptr ? o[r][e] * inv : (o[r][e] * inv) * g;
    if (p.lse != nullptr && lane == 0)
      p.lse[(int64_t)b * p.lse_sb + (int64_t)(p.head_begin + hl) * p.lse_sh + row] =
          l[r] > 0.f ? m[r] + logf(l[r]) : -INFINITY;
  }
}

template <int D>
size_t f32_smem() {
  return sizeof(float) * (kRows * D + kKeys * (D + 1) + kKeys * D + 4 * kRowsPerWarp * kKeys);
}

}  // namespace

cudaError_t launch_fwd_f32(const F32Params& p, int D, int Hc, int B, cudaStream_t s) {
  dim3 grid((p.Lq + kRows - 1) / kRows, Hc, B);
  cudaError_t e;
  if (D == 128) {
    const size_t smem = f32_smem<128>();
    e = cudaFuncSetAttribute(fwd_f32_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fwd_f32_kernel<128><<<grid, 128, smem, s>>>(p);
  } else {
    const size_t smem = f32_smem<64>();
    e = cudaFuncSetAttribute(fwd_f32_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fwd_f32_kernel<64><<<grid, 128, smem, s>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace ltx
