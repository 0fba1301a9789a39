// fwd_sm100.cu -- bf16 fused attention forward on tcgen05 (sm_100a).
//
// Computes, per (batch, head, 128-row query tile):
//     O = softmax(scale * Q K^T + mask) V,   lse = log sum exp(scale * Q K^T + mask)
// the function of DiTAttention.swift:369-382 (fused arm: MLXFast SDPA;
// explicit arm: fp32 logits -> softmax -> PV), online-softmax style with O(N)
// memory: no score matrix leaves the SM.
//
// CTA layout (192 threads, two CTAs per SM):
//   warps 0-3  softmax + correction + epilogue; thread i owns query row i,
//              which is TMEM lane i (warp w reads lane quadrant w)
//   warp 4     TMA producer (lane 0): Q once, then K_j / V_j per KV tile
//   warp 5     TMEM owner; lane 0 issues every tcgen05.mma
// TMEM (256 columns): S = Q K_j^T in columns [0,128) (fp32); P_j (bf16,
// packed two per column) overwrites S's first 64 columns and feeds the PV
// MMA straight from TMEM; O in columns [128, 128+D).
// Per KV tile j the MMA order is  QK_j -> (softmax j) -> PV_j -> QK_{j+1}:
// tcgen05 ops of one thread run in issue order, so QK_{j+1} never overwrites
// P_j before PV_j has read it, and the commit that publishes S_{j+1} also
// proves PV_j finished (so the softmax may rescale O).  The second CTA on the
// SM overlaps its softmax with this CTA's MMAs.
//
// Online softmax in the log2 domain with a lazy max: the running max m only
// moves when a tile's max exceeds it by more than 8 (a factor of 256), so O is
// rescaled rarely; exp2(s - m) then stays <= 256, which fp32 and bf16 carry
// exactly as well as values <= 1.  The final O / l is the same function.
//
// Keys: a tile whose keys are all masked is skipped outright (its weight is
// exactly zero); partial tiles and the ragged tail get -inf logits per
// column.  A batch row whose mask has no valid key attends to all keys
// (GemmaTextEncoder.swift:306-319).
//
// Split-KV (short query sequences): blockIdx.x = q_tile * num_splits + split;
// each split handles a contiguous share of the active KV tiles and writes an
// fp32 partial O (normalised by its own l) and its log2-domain lse; the
// combine kernel merges them.
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {

namespace {

constexpr int kThreads = 192;
constexpr uint32_t kChunkBytes = 128u * 128u;  // one 64-element-wide chunk of a 128-row tile
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLn2 = 0.69314718055994530942f;

template <int D>
struct Smem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTileBytes = kChunks * kChunkBytes;
  // [Q][K][V] tiles (1024-aligned), then control words
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffK = kTileBytes;
  static constexpr uint32_t kOffV = 2 * kTileBytes;
  static constexpr uint32_t kOffBar = 3 * kTileBytes;          // 8 mbarriers
  static constexpr uint32_t kOffCtl = kOffBar + 8 * 8;          // tmem slot, abort, n_tiles
  static constexpr uint32_t kOffTiles = kOffCtl + 16;           // uint16 [kMaxKvTiles]
  static constexpr uint32_t kOffBits = kOffTiles + 2 * kMaxKvTiles;  // uint32 mask bits
  static constexpr uint32_t kFixed = kOffBits;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 2) fwd_bf16_sm100_kernel(const __grid_constant__ FwdParams p) {
  using S = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm + S::kOffQ;
  uint8_t* sK = sm + S::kOffK;
  uint8_t* sV = sm + S::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kf = bars + 1;
  uint64_t* bar_ke = bars + 2;
  uint64_t* bar_vf = bars + 3;
  uint64_t* bar_ve = bars + 4;
  uint64_t* bar_s = bars + 5;
  uint64_t* bar_p = bars + 6;
  uint64_t* bar_o = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  int* n_tiles_slot = reinterpret_cast<int*>(sm + S::kOffCtl + 8);
  uint16_t* tiles = reinterpret_cast<uint16_t*>(sm + S::kOffTiles);
  uint32_t* mbits = reinterpret_cast<uint32_t*>(sm + S::kOffBits);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q_tile = blockIdx.x / p.num_splits;
  const int split = blockIdx.x % p.num_splits;
  const int hl = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = q_tile * kTileM;
  const int Lk = p.Lk;

  // ---------------- prologue ----------------
  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_kf, 1);
    mbar_init(bar_ke, 1);
    mbar_init(bar_vf, 1);
    mbar_init(bar_ve, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 128);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }

  // key-mask bits (padded with zero words to a whole tile)
  bool use_mask = p.mask != nullptr;
  int local_any = 0;
  if (use_mask) {
    const uint8_t* mrow = p.mask + (int64_t)b * p.mask_sb;
    const int nwords = p.n_kv_tiles * (kTileN / 32);
    for (int w = threadIdx.x; w < nwords; w += kThreads) {
      uint32_t bits = 0;
      const int k0 = w * 32;
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int key = k0 + i;
        if (key < Lk && mrow[key] != 0) bits |= 1u << i;
      }
      mbits[w] = bits;
      local_any |= (bits != 0);
    }
  }
  const int any_valid = __syncthreads_or(local_any);
  use_mask = use_mask && (any_valid != 0);

  // the list of KV tiles with at least one valid key
  if (warp == 0) {
    int count = 0;
    for (int j0 = 0; j0 < p.n_kv_tiles; j0 += 32) {
      const int j = j0 + lane;
      bool act = j < p.n_kv_tiles;
      if (act && use_mask) {
        const uint32_t* w4 = mbits + j * 4;
        act = (w4[0] | w4[1] | w4[2] | w4[3]) != 0u;
      }
      const unsigned bal = __ballot_sync(0xffffffffu, act);
      if (act) tiles[count + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
      count += __popc(bal);
    }
    if (lane == 0) *n_tiles_slot = count;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_all = *n_tiles_slot;
  const int t_begin = (int)(((int64_t)split * n_all) / p.num_splits);
  const int t_end = (int)(((int64_t)(split + 1) * n_all) / p.num_splits);
  const int n = t_end - t_begin;
  const int qh = p.q_head_off + hl;
  const int kvh = p.kv_head_off + hl;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n > 0) {
      int k_issued = 0, v_issued = 0;
      mbar_arrive_expect_tx(bar_q, S::kTileBytes);
#pragma unroll
      for (int c = 0; c < S::kChunks; ++c)
        tma_load_4d(&p.tm_q, bar_q, sQ + c * kChunkBytes, c * 64, q0, qh, b);
      for (int i = 0; i < n; ++i) {
        const int kv0 = (int)tiles[t_begin + i] * kTileN;
        if (i > 0 && !mbar_wait(bar_ke, (i - 1) & 1, abort_flag, p.err, 1)) break;
        mbar_arrive_expect_tx(bar_kf, S::kTileBytes);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c)
          tma_load_4d(&p.tm_k, bar_kf, sK + c * kChunkBytes, c * 64, kv0, kvh, b);
        ++k_issued;
        if (i > 0 && !mbar_wait(bar_ve, (i - 1) & 1, abort_flag, p.err, 2)) break;
        mbar_arrive_expect_tx(bar_vf, S::kTileBytes);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c)
          tma_load_4d(&p.tm_v, bar_vf, sV + c * kChunkBytes, c * 64, kv0, kvh, b);
        ++v_issued;
      }
      // never leave the CTA with a bulk copy still writing its shared memory
      drain_wait(bar_q, 0);
      if (k_issued > 0) drain_wait(bar_kf, (k_issued - 1) & 1);
      if (v_issued > 0) drain_wait(bar_vf, (v_issued - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n > 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idesc_pv = idesc_bf16_f32(128, D, 0, 1);
      const uint32_t tS = tmem;         // columns [0, 128)
      const uint32_t tO = tmem + 128;   // columns [128, 128 + D)
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
      if (mbar_wait(bar_q, 0, abort_flag, p.err, 3)) {
        for (int i = 0; i < n; ++i) {
          if (!mbar_wait(bar_kf, i & 1, abort_flag, p.err, 4)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
            umma_ss(tS, sdesc_sw128(aQ + off, 16, 1024), sdesc_sw128(aK + off, 16, 1024), idesc_qk,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(bar_ke);
          umma_commit(bar_s);
          if (!mbar_wait(bar_p, i & 1, abort_flag, p.err, 5)) break;
          if (!mbar_wait(bar_vf, i & 1, abort_flag, p.err, 6)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            // 16 keys = 16 rows of 128 B in each d-chunk; d-chunks are kChunkBytes apart
            umma_ts(tO, tS + kk * 8, sdesc_sw128(aV + kk * 16 * 128, kChunkBytes, 1024), idesc_pv,
                    (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_ve);
        }
      }
      umma_commit(bar_o);
      drain_wait(bar_o, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off;
    const uint32_t tO = tmem + 128 + lane_off;
    const float sl2 = p.scale_log2;
    const int row = q0 + threadIdx.x;
    float m = -INFINITY;  // running max, log2 domain (lazy)
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      if (!warp_wait(bar_s, i & 1, abort_flag, p.err, 7)) { ok = false; break; }
      tc_fence_after();
      float s[128];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(tS + 0, r0);
        tmem_ld32(tS + 32, r1);
        tmem_ld32(tS + 64, r2);
        tmem_ld32(tS + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s[c] = __uint_as_float(r0[c]);
          s[32 + c] = __uint_as_float(r1[c]);
          s[64 + c] = __uint_as_float(r2[c]);
          s[96 + c] = __uint_as_float(r3[c]);
        }
      }
      const int kv0 = (int)tiles[t_begin + i] * kTileN;
      if (use_mask || kv0 + kTileN > Lk) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint32_t bits = 0xffffffffu;
          if (use_mask) bits = mbits[kv0 / 32 + w];
          const int lim = Lk - (kv0 + 32 * w);
          if (lim < 32) bits &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!((bits >> c) & 1u)) s[32 * w + c] = -INFINITY;
        }
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
      const float m_cand = mx * sl2;
      const bool need = m_cand > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need && i > 0)) {
        const float alpha = need ? fast_exp2(m - m_cand) : 1.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
      }
      if (need) {
        l *= fast_exp2(m - m_cand);  // exp2(-inf) = 0 on the first tile
        m = m_cand;
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      float lt = 0.f;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = fast_exp2(fmaf(s[c], sl2, -m_use));
        lt += s[c];
      }
      l += lt;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[64 * h2 + 2 * e], s[64 * h2 + 2 * e + 1]);
        tmem_st32(tS + 32 * h2, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p);
    }

    // epilogue
    const bool have_o = ok && n > 0 && warp_wait(bar_o, 0, abort_flag, p.err, 8);
    tc_fence_after();
    const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
    const int B = gridDim.z, Hc = gridDim.y;
    if (p.num_splits == 1) {
      __nv_bfloat16* orow = p.out + (int64_t)b * p.o_sb + (int64_t)(p.head_begin + hl) * p.o_sh +
                            (int64_t)row * p.o_st;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (have_o) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row < p.Lq) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack_bf16x2(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
        }
      }
      if (p.lse != nullptr && row < p.Lq) {
        p.lse[(int64_t)b * p.lse_sb + (int64_t)(p.head_begin + hl) * p.lse_sh + row] =
            (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
      }
    } else {
      const int64_t prow = (((int64_t)split * B + b) * Hc + hl) * p.Lq + row;
      float* po = p.part_o + prow * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (have_o) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row < p.Lq) {
          float4* dst = reinterpret_cast<float4*>(po + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv_l, __uint_as_float(o[4 * e + 1]) * inv_l,
                                 __uint_as_float(o[4 * e + 2]) * inv_l, __uint_as_float(o[4 * e + 3]) * inv_l);
        }
      }
      if (row < p.Lq) p.part_lse[prow] = (have_o && l > 0.f) ? m + log2f(l) : -INFINITY;
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Merge split partials: lse = log2-sum-exp2 of the splits' lse, O = sum_s w_s O_s.
// One warp per output row.
template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.B * p.Hc * p.Lq;
  if (gw >= rows) return;
  const int row = (int)(gw % p.Lq);
  const int hl = (int)((gw / p.Lq) % p.Hc);
  const int b = (int)(gw / ((int64_t)p.Lq * p.Hc));
  float mx = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) mx = fmaxf(mx, p.part_lse[(int64_t)s * rows + gw]);
  constexpr int kPer = D / 32;
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
  float wsum = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < p.num_splits; ++s) {
      const float ls = p.part_lse[(int64_t)s * rows + gw];
      if (ls == -INFINITY) continue;
      const float w = exp2f(ls - mx);
      wsum += w;
      const float* po = p.part_o + ((int64_t)s * rows + gw) * D;
#pragma unroll
      for (int e = 0; e < kPer; ++e) acc[e] += w * po[lane + 32 * e];
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* orow = p.out + (int64_t)b * p.o_sb + (int64_t)(p.head_begin + hl) * p.o_sh + (int64_t)row * p.o_st;
#pragma unroll
  for (int e = 0; e < kPer; ++e) orow[lane + 32 * e] = __float2bfloat16_rn(acc[e] * inv);
  if (p.lse != nullptr && lane == 0)
    p.lse[(int64_t)b * p.lse_sb + (int64_t)(p.head_begin + hl) * p.lse_sh + row] =
        (wsum > 0.f) ? (mx + log2f(wsum)) * kLn2 : -INFINITY;
}

}  // namespace

size_t fwd_bf16_smem_bytes(int D, int Lk, bool has_mask) {
  const int n_tiles = (Lk + kTileN - 1) / kTileN;
  const size_t fixed = (D == 128) ? Smem<128>::kFixed : Smem<64>::kFixed;
  size_t bytes = 1024 /* alignment slack */ + fixed + (has_mask ? (size_t)n_tiles * 16 : 0);
  // at most two CTAs per SM: each holds 256 TMEM columns of the SM's 512
  const size_t two_per_sm_floor = 80 * 1024;
  return bytes < two_per_sm_floor ? two_per_sm_floor : bytes;
}

cudaError_t launch_fwd_bf16(const FwdParams& p, int D, int q_tiles, int Hc, int B, size_t smem,
                            cudaStream_t s) {
  dim3 grid(q_tiles * p.num_splits, Hc, B);
  cudaError_t e;
  if (D == 128) {
    e = cudaFuncSetAttribute(fwd_bf16_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fwd_bf16_sm100_kernel<128><<<grid, kThreads, smem, s>>>(p);
  } else {
    e = cudaFuncSetAttribute(fwd_bf16_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fwd_bf16_sm100_kernel<64><<<grid, kThreads, smem, s>>>(p);
  }
  return cudaGetLastError();
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t s) {
  const int64_t rows = (int64_t)p.B * p.Hc * p.Lq;
  const int64_t threads = rows * 32;
  const int blocks = (int)((threads + 255) / 256);
  if (p.D == 128)
    combine_kernel<128><<<blocks, 256, 0, s>>>(p);
  else
    combine_kernel<64><<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ltx
