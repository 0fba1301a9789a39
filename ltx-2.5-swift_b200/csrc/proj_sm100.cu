// proj_sm100.cu -- the DiT attention module's projections on tcgen05 (sm_100a).
//
// linear_kernel<BN, kF32Out>: DiTAttention.linear (DiTAttention.swift:178-188)
// without the LoRA overlay: out = T(T(x W^T) + b), the matmul's result in the
// activation dtype T and then the bias added in T -- the reference's two
// roundings (MLX's bf16 matmul accumulates in fp32 and rounds once).  Serves
// to_q, to_k, to_v, to_out.0 and to_gate_logits.  The kF32Out instance stores
// the fp32 accumulator itself (no bias, no rounding): the partial product of a
// row-parallel to_out, which is reduced across ranks before bias_round_kernel
// applies the bias and the roundings once.
//
// CTA: 256 threads, one (128-row block, BN columns) tile.  Warp 0 lane 0 is the
// TMA producer: 128-row x 64 slices of x and BN-row x 64 slices of W into
// kPStages shared-memory stages (128-byte swizzle, K-major, the UMMA operand
// layout).  Warp 1 owns TMEM and its lane 0 issues the tcgen05.mma (M 128,
// N BN, K 16: four per stage), freeing a stage with tcgen05.commit once its
// MMAs complete.  Warps 4-7 are the epilogue: thread i reads TMEM lane i (row
// i of the tile) in 32-column chunks.  No multicast load anywhere.  Every
// mbarrier wait is bounded; a wait that gives up records its site in the
// device error word and the CTA unwinds.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/ltxattn.h"
#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {

int set_error_message(int status, const char* msg);

namespace {

constexpr int kPBM = 128;     // rows per CTA (UMMA M)
constexpr int kPBK = 64;      // K per stage: one 128-byte swizzle row of bf16
constexpr int kPStages = 4;
constexpr int kPThreads = 256;

template <int BN, int NT>
struct PSmem {
  static constexpr uint32_t kA = kPBM * kPBK * 2;  // 16 KB
  static constexpr uint32_t kB = BN * kPBK * 2;
  static constexpr uint32_t kStage = kA + kB;
  // full[kPStages], empty[kPStages], acc_full[NT]
  static constexpr uint32_t kOffBar = kPStages * kStage;
  static constexpr uint32_t kOffCtl = kOffBar + (2 * kPStages + NT) * 8;  // tmem slot, abort flag
  static constexpr uint32_t kBytes = kOffCtl + 16;
  static constexpr uint32_t kDynamic = kBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = BN * NT < 32 ? 32 : BN * NT;
  static_assert(kA % 1024 == 0 && kB % 1024 == 0, "stages must keep 1024-byte swizzle atoms aligned");
  static_assert(BN * NT <= 512, "TMEM holds 512 fp32 columns");
};

// The projection of a launch.
struct ProjJob {
  CUtensorMap tm_x;  // [K, T, B] bf16, box {64, 128, 1}
  CUtensorMap tm_w;  // [K, N] bf16, box {64, BN}
  const __nv_bfloat16* bias;  // [N] or null
  int T, B, N, K;
  int tiles_t;     // ceil(T / 128)
  int col_groups;  // CTAs per row block
  int ctas;        // tiles_t * B * col_groups * splits
  int splits;      // K split into `splits` ranges of kb_per 64-wide blocks (fp32 partials)
  int kb_per;
  // linear: out[b][t][n] at out + b * o_sb + t * o_st + n (bf16), or split s's fp32 partial at
  // out_f32 + s * split_stride + t * o_st + n
  __nv_bfloat16* out;
  float* out_f32;
  int64_t o_sb, o_st, split_stride;
  // fused reduce-scatter (ltxattn_out_project_fused): peer_n > 0 sends the fp32
  // partial of row t to the receive planes of its owner, rank t / rows_per_owner,
  // at plane my_rank (peer_f32[d]: rank d's planes, slot_stride floats apart)
  int peer_n, my_rank, rows_per_owner;
  int64_t slot_stride;
  float* peer_f32[8];
  // rank d's plane for this rank as an fp32 [n, m] tensor map, box {32, 128}:
  // the owner-directed partials leave through shared memory with TMA stores
  CUtensorMap tm_owner[8];
};

struct ProjParams {
  ProjJob job[1];
  int* err;
};

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// y = T(T(acc) + b) for 32 accumulator columns (b null: T(acc)).  `valid` < 32:
// only the first `valid` columns exist (a ragged last column tile); the bias is
// read for those alone.
__device__ __forceinline__ void project_chunk(const uint32_t (&acc)[32], const __nv_bfloat16* bias, float (&y)[32],
                                              int valid = 32) {
  if (bias != nullptr && valid < 32) {
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float bc = c < valid ? __bfloat162float(bias[c]) : 0.f;
      y[c] = bf16_round(bf16_round(__uint_as_float(acc[c])) + bc);
    }
  } else if (bias != nullptr) {
    const uint4* b4 = reinterpret_cast<const uint4*>(bias);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 bw = b4[q];
      const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float b0 = __uint_as_float(bb[e] << 16), b1 = __uint_as_float(bb[e] & 0xffff0000u);
        const int c = 8 * q + 2 * e;
        y[c] = bf16_round(bf16_round(__uint_as_float(acc[c])) + b0);
        y[c + 1] = bf16_round(bf16_round(__uint_as_float(acc[c + 1])) + b1);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c) y[c] = bf16_round(__uint_as_float(acc[c]));
  }
}

// The main loop's two roles (producer: warp 0 lane 0; MMA issuer: warp 1 lane
// 0).  `subtiles` consecutive 256-column (BN-column) accumulators share one
// row block; accumulator s starts at TMEM column s * BN.
template <int BN, int NT>
__device__ __forceinline__ void mainloop_role(const ProjJob& J, int warp, int lane, int t0, int b, int n_base,
                                              int kb0, int kb_n, uint8_t* sm, uint64_t* full, uint64_t* empty,
                                              uint64_t* acc_full, uint32_t tmem, volatile int* abort_flag, int* err) {
  using S = PSmem<BN, NT>;
  if (warp == 0 && lane == 0) {
    int it = 0;
    bool ok = true;
    for (int s = 0; s < NT && ok; ++s) {
      const int n0 = n_base + s * BN;
      for (int kb = 0; kb < kb_n; ++kb, ++it) {
        const int st = it % kPStages, u = it / kPStages;
        if (it >= kPStages && !mbar_wait(empty + st, (u - 1) & 1, abort_flag, err, 41)) {
          ok = false;
          break;
        }
        uint8_t* sa = sm + st * S::kStage;
        mbar_arrive_expect_tx(full + st, S::kStage);
        tma_load_3d(&J.tm_x, full + st, sa, (kb0 + kb) * kPBK, t0, b);
        tma_load_2d(&J.tm_w, full + st, sa + S::kA, (kb0 + kb) * kPBK, n0);
      }
    }
    // never leave the CTA with a bulk copy still writing its shared memory
    for (int i = it < kPStages ? 0 : it - kPStages; i < it; ++i) drain_wait(full + i % kPStages, (i / kPStages) & 1);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(128, BN, 0, 0);
    const SDesc a0 = sdesc_split(smem_u32(sm), 16, 1024);
    const SDesc b0 = sdesc_split(smem_u32(sm) + S::kA, 16, 1024);
    const uint32_t stage_step = S::kStage >> 4;
    int it = 0;
    bool ok = true;
    for (int s = 0; s < NT; ++s) {
      const uint32_t d = tmem + s * BN;
      for (int kb = 0; kb < kb_n && ok; ++kb, ++it) {
        const int st = it % kPStages, u = it / kPStages;
        if (!mbar_wait(full + st, u & 1, abort_flag, err, 42)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t alo = a0.lo + st * stage_step, blo = b0.lo + st * stage_step;
#pragma unroll
        for (int kk = 0; kk < kPBK / 16; ++kk)  // k-step kk: 32 bytes further along each 128-byte row
          umma_ss2(d, alo + kk * 2, a0.hi, blo + kk * 2, b0.hi, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(empty + st);  // the stage is free once these MMAs have read it
      }
      umma_commit(acc_full + s);  // also issued after a timeout, so the epilogue's waits end
    }
    drain_wait(acc_full + NT - 1, 0);  // no MMA still running when the CTA tears down
  }
}

// ---------------------------------------------------------------------------
// linear: one CTA per (128-row block, BN columns)

template <int BN, bool kF32Out>
__global__ void __launch_bounds__(kPThreads, 1) linear_kernel(const __grid_constant__ ProjParams p) {
  using S = PSmem<BN, 1>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPStages;
  uint64_t* acc_full = bars + 2 * kPStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  const ProjJob& J = p.job[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA -> (K split, row block, column tile), column tile fastest
  const int tiles = J.tiles_t * J.B * J.col_groups;
  const int split = (int)blockIdx.x / tiles;
  const int tile = (int)blockIdx.x - split * tiles;
  const int cg = tile % J.col_groups;
  const int rb = tile / J.col_groups;
  const int b = rb / J.tiles_t, t0 = (rb % J.tiles_t) * kPBM;
  const int n_base = cg * BN;
  const int kb0 = split * J.kb_per;
  const int kb_n = min(J.kb_per, J.K / kPBK - kb0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * kPStages + 1; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&J.tm_x);
    tma_prefetch_desc(&J.tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    mainloop_role<BN, 1>(J, warp, lane, t0, b, n_base, kb0, kb_n, sm, full, empty, acc_full, tmem, abort_flag,
                         p.err);
  } else {
    const int r = threadIdx.x - 128;  // TMEM lane = tile row
    const int t = t0 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const bool have = warp_wait(acc_full, 0, abort_flag, p.err, 43);
    tc_fence_after();
    if (kF32Out && J.peer_n > 0) {
      // fused reduce-scatter: the tile's rows all belong to one owner (owners hold
      // whole 128-row blocks); each 32-column chunk is staged row-major in the
      // idle pipeline stages (128 rows x 128 bytes) and stored with TMA into the
      // owner's plane for this rank, so the NVLink writes go out as bulk copies
      const CUtensorMap* dst_map = &J.tm_owner[t0 / J.rows_per_owner];
      float* stg = reinterpret_cast<float*>(sm);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int n = n_base + c * 32;
        if (n >= J.N) break;  // warp-uniform
        uint32_t acc[32];
        if (have) {
          tmem_ld32(tmem + lane_off + c * 32, acc);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0u;
        }
        if (r == 0) bulk_wait_read();  // the previous chunk's copy has read the staging rows
        named_barrier(1, 128);
        uint4* row = reinterpret_cast<uint4*>(stg + r * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) row[q] = make_uint4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        fence_proxy_async_smem();
        named_barrier(1, 128);
        if (r == 0) {
          tma_store_4d(dst_map, stg, n, t0, 0, 0);
          bulk_commit();
        }
      }
      if (r == 0) bulk_wait_read();  // the CTA's shared memory must outlive the copies' reads
    } else if (have) {
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int n = n_base + c * 32;
        if (n >= J.N) break;  // a ragged last column tile (warp-uniform)
        const int valid = min(32, J.N - n);  // a multiple of 8
        uint32_t acc[32];
        tmem_ld32(tmem + lane_off + c * 32, acc);
        tmem_wait_ld();
        if (t < J.T && kF32Out) {
          // the fp32 accumulator itself (a partial sum that is reduced across ranks before
          // the bias and the roundings)
          float* plane = J.out_f32 + split * J.split_stride;
          if (J.peer_n > 0) plane = J.peer_f32[t / J.rows_per_owner] + (int64_t)J.my_rank * J.slot_stride;
          uint4* dst = reinterpret_cast<uint4*>(plane + (int64_t)t * J.o_st + n);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (4 * q < valid) dst[q] = make_uint4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        } else if (t < J.T) {
          float y[32];
          project_chunk(acc, J.bias != nullptr ? J.bias + n : nullptr, y, valid);
          uint4* dst = reinterpret_cast<uint4*>(J.out + (int64_t)b * J.o_sb + (int64_t)t * J.o_st + n);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (8 * q < valid)
              dst[q] = make_uint4(pack_bf16x2(y[8 * q], y[8 * q + 1]), pack_bf16x2(y[8 * q + 2], y[8 * q + 3]),
                                  pack_bf16x2(y[8 * q + 4], y[8 * q + 5]), pack_bf16x2(y[8 * q + 6], y[8 * q + 7]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// out[t][n] = T(T(sum[t][n]) + b[n]) with sum the `splits` fp32 partial planes
// added in split order: the roundings of DiTAttention.linear applied once the
// partial sums (K splits of one GPU, or the row-parallel ranks after their
// all-reduce) are complete.  One thread per 8 columns.
struct PeerRows {  // the same rows in other ranks' outputs (fused all-gather of the reduced rows)
  int n;
  __nv_bfloat16* out[7];
};

__global__ void __launch_bounds__(256) bias_round_kernel(const float* sum, int64_t s_st, int splits,
                                                         int64_t split_stride, const __nv_bfloat16* bias,
                                                         __nv_bfloat16* out, int64_t o_st, int M, int N,
                                                         const PeerRows peers) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int n8 = N / 8;
  if (i >= (int64_t)M * n8) return;
  const int t = (int)(i / n8), n = (int)(i % n8) * 8;
  float y[8];
  for (int s = 0; s < splits; ++s) {
    const float4* src = reinterpret_cast<const float4*>(sum + s * split_stride + (int64_t)t * s_st + n);
    const float4 a = src[0], c = src[1];
    const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = s == 0 ? v[e] : __fadd_rn(y[e], v[e]);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    y[e] = bf16_round(y[e]);
    if (bias != nullptr) y[e] = bf16_round(y[e] + __bfloat162float(bias[n + e]));
  }
  const uint4 packed =
      make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  *reinterpret_cast<uint4*>(out + (int64_t)t * o_st + n) = packed;
  for (int d = 0; d < peers.n; ++d) *reinterpret_cast<uint4*>(peers.out[d] + (int64_t)t * o_st + n) = packed;
}

// ---------------------------------------------------------------------------
// host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
    else
      (void)cudaGetLastError();
  });
  return fn;
}

int fail_msg(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return set_error_message(status, buf);
}

// x: [K, T, B] bf16 (element strides st for T, sb for B), box {64, 128, 1}
int map_rows(CUtensorMap* m, const void* ptr, int K, int T, int B, int64_t st, int64_t sb, const char* name) {
  EncodeTiledFn enc = encoder();
  if (!enc) return fail_msg(LTXATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int64_t s2 = B == 1 ? st * T : sb;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)st * 2, (cuuint64_t)s2 * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail_msg(LTXATTN_ERR_ALIGN, "%s: cuTensorMapEncodeTiled rejected the view (CUresult %d)", name, (int)r);
  return LTXATTN_OK;
}

// An fp32 [m, n] plane (row stride n) as a 4-D [n, m, 1, 1] tensor map, box
// {32, 128, 1, 1}, no swizzle: the owner-directed partial stores.
int map_plane_f32(CUtensorMap* mp, float* ptr, int n, int m) {
  EncodeTiledFn enc = encoder();
  if (!enc) return fail_msg(LTXATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)n, (cuuint64_t)m, 1, 1};
  cuuint64_t strides[3] = {(cuuint64_t)n * 4, (cuuint64_t)n * m * 4, (cuuint64_t)n * m * 4};
  cuuint32_t box[4] = {32, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail_msg(LTXATTN_ERR_ALIGN, "receive plane: cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return LTXATTN_OK;
}

// W: [K, N] bf16 (row stride sw elements), box {64, bn}
int map_weight(CUtensorMap* m, const void* ptr, int K, int N, int64_t sw, int bn, const char* name) {
  EncodeTiledFn enc = encoder();
  if (!enc) return fail_msg(LTXATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
  cuuint64_t strides[1] = {(cuuint64_t)sw * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)bn};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail_msg(LTXATTN_ERR_ALIGN, "%s: cuTensorMapEncodeTiled rejected the view (CUresult %d)", name, (int)r);
  return LTXATTN_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_fail(cudaError_t e, const char* what) {
  (void)cudaGetLastError();
  return fail_msg(LTXATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Dynamic shared memory above 48 KB is opted into once per device and kernel.
constexpr int kMaxDev = 64;
std::mutex g_mu;
bool g_attr_set[kMaxDev][10] = {};

template <typename K>
cudaError_t prepare_kernel(K kernel, int slot, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_attr_set[dev][slot]) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    g_attr_set[dev][slot] = true;
  }
  return cudaSuccess;
}

}  // namespace
}  // namespace ltx

using namespace ltx;

namespace {

// Column tile: the widest that divides n; otherwise 32 with a ragged last tile
// (the weight's missing rows read as zeros, only existing columns are stored).
int bn_for(int n) {
  if (n % 256 == 0) return 256;
  if (n % 128 == 0) return 128;
  if (n % 64 == 0) return 64;
  return 32;
}

template <int BN, bool kF32Out>
int launch_linear_bn(ProjParams& P, const ltxattn_linear_args* a, cudaStream_t st) {
  using S = PSmem<BN, 1>;
  ProjJob& J = P.job[0];
  if (int rc = map_weight(&J.tm_w, a->weight, a->k, a->n, a->weight_stride, BN, "weight")) return rc;
  J.col_groups = (a->n + BN - 1) / BN;
  J.ctas = J.tiles_t * J.col_groups * J.splits;
  const int slot = (BN == 256 ? 0 : BN == 128 ? 1 : BN == 64 ? 2 : 3) + (kF32Out ? 5 : 0);
  cudaError_t e = prepare_kernel(linear_kernel<BN, kF32Out>, slot, S::kDynamic);
  if (e != cudaSuccess) return launch_fail(e, "linear kernel attributes");
  linear_kernel<BN, kF32Out><<<J.ctas, kPThreads, S::kDynamic, st>>>(P);
  e = cudaGetLastError();
  if (e != cudaSuccess) return launch_fail(e, "linear launch");
  return LTXATTN_OK;
}

}  // namespace


namespace {

int sm_count_cached() {
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    (void)cudaGetLastError();
    return 148;
  }
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = 148;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

// K splits for a narrow output: when the tiles fill under half the SMs (e.g. the
// 32 gate logits of 3120 rows: 25 tiles), split the 64-wide K blocks into ranges
// of at least 4 so the CTAs cover the SMs; 1 = no split.
void plan_splits(int m, int n, int k, int* splits, int* kb_per) {
  const int bn = bn_for(n);
  const int tiles = ((m + kPBM - 1) / kPBM) * ((n + bn - 1) / bn);
  const int kb_total = k / kPBK;
  const int sms = sm_count_cached();
  *splits = 1;
  *kb_per = kb_total;
  if (2 * tiles > sms || kb_total < 8) return;
  const int want = std::min({sms / tiles, kb_total / 4, 16});
  if (want < 2) return;
  *kb_per = (kb_total + want - 1) / want;
  *splits = (kb_total + *kb_per - 1) / *kb_per;
}

size_t split_workspace(int m, int n, int splits) {
  return splits > 1 ? ((size_t)splits * m * n * sizeof(float) + 255) & ~size_t(255) : 0;
}

// ltxattn_linear, or (f32_out != null) the same GEMM storing its fp32
// accumulator, without bias or roundings, into f32_out [m, n] (row stride n).
int run_linear(const ltxattn_linear_args* a, float* f32_out, cudaStream_t st, const ltx::OwnerPlanes* owners = nullptr) {
  if (a == nullptr) return fail_msg(LTXATTN_ERR_ARG, "args is NULL");
  if (a->dtype != LTXATTN_BF16) return fail_msg(LTXATTN_ERR_DTYPE, "ltxattn_linear: bf16 only");
  if (a->m < 1 || a->n < 1 || a->k < 1) return fail_msg(LTXATTN_ERR_SHAPE, "ltxattn_linear: m, n and k must be >= 1");
  const int bn = bn_for(a->n);
  if (a->n % 8 != 0 || a->k % 64 != 0)
    return fail_msg(LTXATTN_ERR_UNSUPPORTED, "ltxattn_linear: n (%d) must be a multiple of 8 and k (%d) of 64", a->n,
                    a->k);
  if (!a->x || !a->weight || !a->out) return fail_msg(LTXATTN_ERR_ARG, "ltxattn_linear: x, weight and out are required");
  if (a->x_stride < a->k || a->weight_stride < a->k || a->out_stride < a->n)
    return fail_msg(LTXATTN_ERR_SHAPE, "ltxattn_linear: a row stride is shorter than its row");
  if (!al16(a->x) || !al16(a->weight) || !al16(a->out) || (a->bias && !al16(a->bias)) || (a->x_stride % 8) ||
      (a->weight_stride % 8) || (a->out_stride % 8))
    return fail_msg(LTXATTN_ERR_ALIGN, "ltxattn_linear: x, weight, bias and out need 16-byte aligned rows");
  ProjParams P{};
  P.err = device_error_word();
  if (!P.err) return fail_msg(LTXATTN_ERR_CUDA, "no device error word");
  ProjJob& J = P.job[0];
  if (int rc = map_rows(&J.tm_x, a->x, a->k, a->m, 1, a->x_stride, 0, "x")) return rc;
  J.bias = static_cast<const __nv_bfloat16*>(a->bias);
  J.T = a->m;
  J.B = 1;
  J.N = a->n;
  J.K = a->k;
  J.tiles_t = (a->m + kPBM - 1) / kPBM;
  J.out = static_cast<__nv_bfloat16*>(a->out);
  J.out_f32 = f32_out;
  J.o_sb = 0;
  J.o_st = f32_out != nullptr ? a->n : a->out_stride;
  J.splits = 1;
  J.kb_per = a->k / kPBK;
  J.split_stride = 0;
  if (owners != nullptr) {
    J.peer_n = owners->world;
    J.my_rank = owners->rank;
    J.rows_per_owner = owners->rows_per_owner;
    J.slot_stride = owners->slot_stride;
    for (int d = 0; d < owners->world; ++d) {
      J.peer_f32[d] = owners->planes[d];
      if (int rc = map_plane_f32(&J.tm_owner[d], owners->planes[d] + (int64_t)owners->rank * owners->slot_stride,
                                 a->n, a->m))
        return rc;
    }
  }
  if (f32_out == nullptr) {
    // a narrow output with a workspace: K splits into fp32 partials, then one
    // pass adds them in split order and applies the bias and the roundings
    int splits = 1, kb_per = 0;
    plan_splits(a->m, a->n, a->k, &splits, &kb_per);
    const size_t need = split_workspace(a->m, a->n, splits);
    if (splits > 1 && a->workspace != nullptr && a->workspace_bytes >= need &&
        (reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0) {
      J.splits = splits;
      J.kb_per = kb_per;
      J.out_f32 = static_cast<float*>(a->workspace);
      J.o_st = a->n;
      J.split_stride = (int64_t)a->m * a->n;
      int rc;
      switch (bn) {
        case 256: rc = launch_linear_bn<256, true>(P, a, st); break;
        case 128: rc = launch_linear_bn<128, true>(P, a, st); break;
        case 64: rc = launch_linear_bn<64, true>(P, a, st); break;
        default: rc = launch_linear_bn<32, true>(P, a, st); break;
      }
      if (rc) return rc;
      return ltx::bias_round(J.out_f32, splits, J.split_stride, a->bias, a->out, a->out_stride, a->m, a->n, st);
    }
  }
  if (f32_out != nullptr) {
    switch (bn) {
      case 256: return launch_linear_bn<256, true>(P, a, st);
      case 128: return launch_linear_bn<128, true>(P, a, st);
      case 64: return launch_linear_bn<64, true>(P, a, st);
      default: return launch_linear_bn<32, true>(P, a, st);
    }
  }
  switch (bn) {
    case 256: return launch_linear_bn<256, false>(P, a, st);
    case 128: return launch_linear_bn<128, false>(P, a, st);
    case 64: return launch_linear_bn<64, false>(P, a, st);
    default: return launch_linear_bn<32, false>(P, a, st);
  }
}

}  // namespace

namespace ltx {

// The row-parallel to_out's local steps (the collective between them is in comm.cpp).
int linear_partial_f32(const ltxattn_linear_args* a, float* partial, cudaStream_t st) {
  if (partial == nullptr || (reinterpret_cast<uintptr_t>(partial) & 15u))
    return fail_msg(LTXATTN_ERR_ALIGN, "the fp32 partial buffer must be 16-byte aligned");
  return run_linear(a, partial, st);
}

int linear_partial_f32_to_owners(const ltxattn_linear_args* a, float* const* planes, int world, int rank,
                                 int rows_per_owner, int64_t slot_stride, cudaStream_t st) {
  for (int d = 0; d < world; ++d)
    if (planes[d] == nullptr || (reinterpret_cast<uintptr_t>(planes[d]) & 15u))
      return fail_msg(LTXATTN_ERR_ALIGN, "rank %d's receive planes must be 16-byte aligned", d);
  OwnerPlanes o{world, rank, rows_per_owner, slot_stride, {}};
  for (int d = 0; d < world; ++d) o.planes[d] = planes[d];
  return run_linear(a, planes[rank], st, &o);
}

int bias_round(const float* sum, int splits, int64_t split_stride, const void* bias, void* out, int64_t out_stride,
               int m, int n, cudaStream_t st, int n_peer_out, void* const* peer_out) {
  const int64_t threads = (int64_t)m * (n / 8);
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7fffffff) return fail_msg(LTXATTN_ERR_UNSUPPORTED, "output too large");
  if (blocks == 0) return LTXATTN_OK;
  PeerRows pr{};
  for (int d = 0; d < n_peer_out && d < 7; ++d) pr.out[pr.n++] = static_cast<__nv_bfloat16*>(peer_out[d]);
  bias_round_kernel<<<(unsigned)blocks, 256, 0, st>>>(sum, n, splits, split_stride,
                                                      static_cast<const __nv_bfloat16*>(bias),
                                                      static_cast<__nv_bfloat16*>(out), out_stride, m, n, pr);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return launch_fail(e, "bias and rounding launch");
  return LTXATTN_OK;
}

}  // namespace ltx

extern "C" {

int ltxattn_linear(const ltxattn_linear_args* a, void* stream) {
  return run_linear(a, nullptr, static_cast<cudaStream_t>(stream));
}

size_t ltxattn_linear_workspace(const ltxattn_linear_args* a) {
  if (a == nullptr || a->m < 1 || a->n < 8 || a->k < 64 || a->n % 8 || a->k % 64) return 0;
  int splits = 1, kb_per = 0;
  plan_splits(a->m, a->n, a->k, &splits, &kb_per);
  return split_workspace(a->m, a->n, splits);
}

}  // extern "C"
