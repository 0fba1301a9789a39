// bwd_sm100.cu -- bf16 attention backward on tcgen05 (sm_100a).
//
// The reference trains LoRA adapters through MLX's autodiff VJP of the fused
// SDPA under per-block gradient checkpointing (LoRATrainingStep.swift:283-304,
// GradientCheckpoint.swift:48-67, DiTForward.swift:1012-1049).  This is that
// VJP in closed form, with P recomputed from the forward's saved per-row
// log-sum-exp, so no score matrix is ever stored:
//
//   P  = exp(scale*QK^T - lse)          dV = P^T dO
//   dP = dO V^T                         dS = P o (dP - Delta),  Delta = rowsum(dO o O)
//   dQ = scale * dS K                   dK = scale * dS^T Q
//
// Two launches, both deterministic (no atomics, so a recomputed step is
// bit-identical, as gradient checkpointing expects):
//   bwd_prep_kernel   Delta and lse*log2(e) per query row, padded to 128 rows
//   bwd_sm100_kernel  the two gradient passes as one grid, dK/dV CTAs first
//                     (the longer ones), then dQ CTAs: independent work, so
//                     the tail of one pass fills with CTAs of the other
//                     (config 2: 730 -> 675 us against two launches)
// The passes:
//   dQ pass           Q-stationary: per 128-row Q tile, loop over KV tiles;
//                     TMEM: S [0,128), dP [128,256), dQ [256,256+D),
//                     Q [384,384+D/2), dO [448,448+D/2) (bf16 pairs: the
//                     A operands of S = Q K^T and dP = dO V^T come from TMEM,
//                     so those MMAs read only K or V from shared memory).
//                     dS overwrites dP, so S_{i+1} runs while the softmax
//                     warps turn S_i / dP_i into dS_i.
//   dK/dV pass        KV-stationary: per 128-key tile, loop over Q tiles;
//                     TMEM: S^T [0,128), dP^T [128,256), dV [256,..), dK [384,..);
//                     P^T and dS^T overwrite dP^T, so S^T of the next Q tile
//                     runs while the softmax warps work on this one
// In both, the softmax warps turn S/dP into bf16 P or dS in place (TMEM) and
// the PV-style products read them straight from TMEM (tcgen05.mma A-from-TMEM).
// When rotary tables are given, dQ and dK leave through the transpose
// rotation: the gradient with respect to the un-rotated input.
#include <mutex>

#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

// warps 0-7: softmax (warp w reads TMEM lane quadrant w % 4; warps w and w + 4
// share a quadrant and take the two halves of its columns), warp 8: TMA
// producer, warp 9: TMEM owner and MMA issuer
constexpr int kThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kChunkBytes = 128u * 128u;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// column validity of 32 keys starting at key0 (mask bits in smem, tail by length)
__device__ __forceinline__ uint32_t key_bits(const uint32_t* mbits, bool use_mask, int key0, int Lk) {
  uint32_t bits = use_mask ? mbits[key0 / 32] : 0xffffffffu;
  const int lim = Lk - key0;
  if (lim < 32) bits &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
  return bits;
}

// Build mask bits for all KV tiles of batch b (zero-padded to whole tiles) and
// report whether any key is valid.  Every thread of the CTA calls this.
__device__ __forceinline__ int load_mask_bits(const BwdParams& p, int b, uint32_t* mbits) {
  int local_any = 0;
  if (p.mask != nullptr) {
    const uint8_t* mrow = p.mask + (int64_t)b * p.mask_sb;
    const int nwords = p.n_kv_tiles * (kTileN / 32);
    for (int w = threadIdx.x; w < nwords; w += kThreads) {
      uint32_t bits = 0;
      const int k0 = w * 32;
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int key = k0 + i;
        if (key < p.Lk && mrow[key] != 0) bits |= 1u << i;
      }
      mbits[w] = bits;
      local_any |= (bits != 0);
    }
  }
  return __syncthreads_or(local_any);
}

// ---------------------------------------------------------------------------
// Delta = rowsum(dO o O) and the row's lse (times log2(e) for the bf16
// kernels); padded rows get Delta 0 and lse +inf, so their recomputed P is
// exactly 0.  One warp per row.

template <int D, typename T>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const BwdPrepParams p) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.B * p.Hc * p.Lq_pad;
  if (gw >= rows) return;
  const int row = (int)(gw % p.Lq_pad);
  const int hl = (int)((gw / p.Lq_pad) % p.Hc);
  const int b = (int)(gw / ((int64_t)p.Lq_pad * p.Hc));
  float acc = 0.f;
  if (row < p.Lq) {
    const T* o = static_cast<const T*>(p.o) + (int64_t)b * p.o_sb + (int64_t)hl * p.o_sh + (int64_t)row * p.o_st;
    const T* g = static_cast<const T*>(p.dout) + (int64_t)b * p.do_sb + (int64_t)hl * p.do_sh + (int64_t)row * p.do_st;
#pragma unroll
    for (int e = 0; e < D / 32; ++e) acc += to_f32(o[lane + 32 * e]) * to_f32(g[lane + 32 * e]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    p.delta[gw] = acc;
    const float l = (row < p.Lq) ? p.lse[(int64_t)b * p.lse_sb + (int64_t)hl * p.lse_sh + row] : INFINITY;
    p.lse2[gw] = (p.log2_domain && row < p.Lq) ? l * 1.4426950408889634f : l;
  }
}

// One gradient row out of TMEM: g = scale * (TMEM columns), then, with a table
// (c, s non-null), the transpose rotation of RoPE (g1 c + g2 s, g2 c - g1 s for
// the pair (i, i + D/2), each product and sum rounded once in fp32), then bf16
// to dst.  It works on 32-column pieces of each half of the row, so at most 64
// values and one piece of the table are live in registers.  The table is read
// 16 bytes at a time when `vec` (rows 16-byte aligned), else entry by entry
// (each thread reads its own row, so scalar reads cost a cache line per lane
// per entry: at config 2 that was 117 us of the backward's 810).  `have`
// (warp-uniform: TMEM loads are warp-collective) false writes zeros; `live`
// false skips the store.
template <int D>
__device__ __forceinline__ void grad_row_out(uint32_t taddr, bool have, bool live, float scale,
                                             const __nv_bfloat16* c, const __nv_bfloat16* s, bool vec,
                                             __nv_bfloat16* dst) {
  constexpr int H = D / 2;
#pragma unroll
  for (int piece = 0; piece < H / 32; ++piece) {
    uint32_t r1[32], r2[32];
    if (have) {
      tmem_ld32(taddr + piece * 32, r1);
      tmem_ld32(taddr + H + piece * 32, r2);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) r1[e] = r2[e] = 0u;
    }
    if (!live) continue;
    float g1[32], g2[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      g1[e] = __uint_as_float(r1[e]) * scale;
      g2[e] = __uint_as_float(r2[e]) * scale;
    }
    if (c != nullptr) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // table entries piece*32 + 8u .. + 7
        float cc[8], ss[8];
        if (vec) {
          const uint4 cv = __ldg(reinterpret_cast<const uint4*>(c + piece * 32) + u);
          const uint4 sv = __ldg(reinterpret_cast<const uint4*>(s + piece * 32) + u);
          const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {  // bf16 -> fp32 is exact: the bits move to the top half
            cc[e] = __uint_as_float((e & 1) ? (cw[e >> 1] & 0xffff0000u) : (cw[e >> 1] << 16));
            ss[e] = __uint_as_float((e & 1) ? (sw[e >> 1] & 0xffff0000u) : (sw[e >> 1] << 16));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            cc[e] = __bfloat162float(c[piece * 32 + 8 * u + e]);
            ss[e] = __bfloat162float(s[piece * 32 + 8 * u + e]);
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = 8 * u + e;
          const float a1 = g1[i], a2 = g2[i];
          g1[i] = __fadd_rn(__fmul_rn(a1, cc[e]), __fmul_rn(a2, ss[e]));
          g2[i] = __fsub_rn(__fmul_rn(a2, cc[e]), __fmul_rn(a1, ss[e]));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      reinterpret_cast<uint4*>(dst + piece * 32)[u] =
          make_uint4(pack_bf16x2(g1[8 * u], g1[8 * u + 1]), pack_bf16x2(g1[8 * u + 2], g1[8 * u + 3]),
                     pack_bf16x2(g1[8 * u + 4], g1[8 * u + 5]), pack_bf16x2(g1[8 * u + 6], g1[8 * u + 7]));
      reinterpret_cast<uint4*>(dst + H + piece * 32)[u] =
          make_uint4(pack_bf16x2(g2[8 * u], g2[8 * u + 1]), pack_bf16x2(g2[8 * u + 2], g2[8 * u + 3]),
                     pack_bf16x2(g2[8 * u + 4], g2[8 * u + 5]), pack_bf16x2(g2[8 * u + 6], g2[8 * u + 7]));
    }
  }
}

// ---------------------------------------------------------------------------
// dQ: Q-stationary

template <int D>
struct DqSmem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr uint32_t kOffQ = 0, kOffDO = kTile, kOffK0 = 2 * kTile, kOffV0 = 3 * kTile,
                            kOffK1 = 4 * kTile, kOffV1 = 5 * kTile;
  // q_full, kv_full[2], kv_empty[2], s_full, p_full, o_full, qt_ready, p_half, s_read
  static constexpr uint32_t kOffBar = 6 * kTile;
  static constexpr uint32_t kOffCtl = kOffBar + 11 * 8;
  static constexpr uint32_t kOffTiles = kOffCtl + 16;
  static constexpr uint32_t kOffBits = kOffTiles + 2 * kMaxKvTiles;
};

template <int D>
__device__ __forceinline__ void bwd_dq_body(const BwdParams& p, int tile, int hl, int b, int Hc) {
  using S = DqSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm + S::kOffQ;
  uint8_t* sDO = sm + S::kOffDO;
  // stage st of K / V lives at sK0 / sV0 + st * 2 * kTile (K and V stages interleave)
  uint8_t* sK0 = sm + S::kOffK0;
  uint8_t* sV0 = sm + S::kOffV0;
  static_assert(S::kOffK1 == S::kOffK0 + 2 * S::kTile && S::kOffV1 == S::kOffV0 + 2 * S::kTile, "stage stride");
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kvf = bars + 1;  // [2]
  uint64_t* bar_kve = bars + 3;  // [2]
  uint64_t* bar_s = bars + 5;
  uint64_t* bar_p = bars + 6;
  uint64_t* bar_o = bars + 7;
  uint64_t* bar_qt = bars + 8;  // Q and dO rows copied into TMEM
  uint64_t* bar_ph = bars + 9;  // dS for keys 0-63 stored (warps 0-3); bar_p: keys 64-127 (warps 4-7)
  uint64_t* bar_sr = bars + 10; // every softmax thread has loaded its S columns: S may be overwritten
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  int* n_tiles_slot = reinterpret_cast<int*>(sm + S::kOffCtl + 8);
  uint16_t* tiles = reinterpret_cast<uint16_t*>(sm + S::kOffTiles);
  uint32_t* mbits = reinterpret_cast<uint32_t*>(sm + S::kOffBits);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = tile * kTileM;

  if (threadIdx.x == 0) {
    // p_full / p_half: the 128 threads of warps 4-7 / 0-3; qt_ready, s_read: all 256 softmax threads
    for (int i = 0; i < 11; ++i) mbar_init(bars + i, (i == 8 || i == 10) ? 256 : ((i == 6 || i == 9) ? 128 : 1));
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  const bool use_mask = p.mask != nullptr && load_mask_bits(p, b, mbits) != 0;
  if (warp == 0) {
    int count = 0;
    for (int j0 = 0; j0 < p.n_kv_tiles; j0 += 32) {
      const int j = j0 + lane;
      bool act = j < p.n_kv_tiles;
      if (act && use_mask) act = (mbits[4 * j] | mbits[4 * j + 1] | mbits[4 * j + 2] | mbits[4 * j + 3]) != 0u;
      const unsigned bal = __ballot_sync(0xffffffffu, act);
      if (act) tiles[count + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
      count += __popc(bal);
    }
    if (lane == 0) *n_tiles_slot = count;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n = *n_tiles_slot;

  if (warp == kProducerWarp) {
    if (lane == 0 && n > 0) {
      int issued = 0;
      mbar_arrive_expect_tx(bar_q, 2 * S::kTile);
#pragma unroll
      for (int c = 0; c < S::kChunks; ++c) {
        tma_load_4d(&p.tm_q, bar_q, sQ + c * kChunkBytes, c * 64, q0, hl, b);
        tma_load_4d(&p.tm_do, bar_q, sDO + c * kChunkBytes, c * 64, q0, hl, b);
      }
      for (int i = 0; i < n; ++i) {
        const int st = i & 1;
        if (i >= 2 && !mbar_wait(bar_kve + st, ((i >> 1) - 1) & 1, abort_flag, p.err, 21)) break;
        const int kv0 = (int)tiles[i] * kTileN;
        mbar_arrive_expect_tx(bar_kvf + st, 2 * S::kTile);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c) {
          tma_load_4d(&p.tm_k, bar_kvf + st, sK0 + st * 2 * S::kTile + c * kChunkBytes, c * 64, kv0, hl, b);
          tma_load_4d(&p.tm_v, bar_kvf + st, sV0 + st * 2 * S::kTile + c * kChunkBytes, c * 64, kv0, hl, b);
        }
        ++issued;
      }
      drain_wait(bar_q, 0);
      for (int i = issued - 2 < 0 ? 0 : issued - 2; i < issued; ++i) drain_wait(bar_kvf + (i & 1), (i >> 1) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0 && n > 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idesc_dq = idesc_bf16_f32(128, D, 0, 1);
      const uint32_t tS = tmem, tP = tmem + 128, tQ = tmem + 256, tQa = tmem + 384, tOa = tmem + 448;
      // S_i = Q K_i^T and dP_i = dO V_i^T (A operands from TMEM)
      auto issue_s = [&](int st) {
        const SDesc dKd = sdesc_split(smem_u32(sK0) + st * 2 * S::kTile, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_ts2(tS, tQa + kk * 8, dKd.lo + off, dKd.hi, idesc_s, kk > 0);
        }
      };
      auto issue_dp = [&](int st) {
        const SDesc dVd = sdesc_split(smem_u32(sV0) + st * 2 * S::kTile, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_ts2(tP, tOa + kk * 8, dVd.lo + off, dVd.hi, idesc_s, kk > 0);
        }
      };
      // Order per KV tile i: S_{i+1} as soon as softmax has loaded S_i (dS_i
      // goes to the dP columns, so the S columns are free early), then
      // dQ += dS_i K_i in two halves, then dP_{i+1} (after dQ has read dS_i).
      bool go = mbar_wait(bar_qt, 0, abort_flag, p.err, 22) && mbar_wait(bar_kvf, 0, abort_flag, p.err, 23);
      if (go) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
        umma_commit(bar_s);
      }
      for (int i = 0; i < n && go; ++i) {
        const int st = i & 1, st1 = (i + 1) & 1;
        const bool more = i + 1 < n;
        const SDesc dKmn = sdesc_split(smem_u32(sK0) + st * 2 * S::kTile, kChunkBytes, 1024);
        if (more) {
          if (!(go = mbar_wait(bar_sr, i & 1, abort_flag, p.err, 29))) break;
          if (!(go = mbar_wait(bar_kvf + st1, ((i + 1) >> 1) & 1, abort_flag, p.err, 23))) break;
          tc_fence_after();
          issue_s(st1);
        }
        // dQ += dS K in two halves of 64 keys: the first runs while softmax
        // finishes the second half of dS
        if (!(go = mbar_wait(bar_ph, i & 1, abort_flag, p.err, 28))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTileN / 32; ++kk)  // keys 0-63: dS at dP columns [0, 32)
          umma_ts2(tQ, tP + kk * 8, dKmn.lo + ((kk * 16 * 128) >> 4), dKmn.hi, idesc_dq, (i > 0 || kk > 0) ? 1u : 0u);
        if (!(go = mbar_wait(bar_p, i & 1, abort_flag, p.err, 24))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = kTileN / 32; kk < kTileN / 16; ++kk)  // keys 64-127: dS at dP columns [64, 96)
          umma_ts2(tQ, tP + 32 + kk * 8, dKmn.lo + ((kk * 16 * 128) >> 4), dKmn.hi, idesc_dq, 1u);
        umma_commit(bar_kve + st);
        if (more) {
          issue_dp(st1);
          umma_commit(bar_s);
        }
      }
      umma_commit(bar_o);
      drain_wait(bar_o, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off, tP = tmem + 128 + lane_off, tQ = tmem + 256 + lane_off;
    const int r = quad * 32 + lane;  // row of the tile = TMEM lane
    const int row = q0 + r;
    const int64_t rix = ((int64_t)b * Hc + hl) * p.Lq_pad + row;
    const float lse2 = p.lse2[rix];
    const float delta = p.delta[rix];
    const float sl2 = p.scale_log2;
    bool ok = true;
    if (n > 0) {
      // Q (warps 0-3) and dO (warps 4-7) rows into TMEM as bf16 pairs, the A
      // operands of S and dP: each thread copies its row out of the
      // 128-byte-swizzled tile
      ok = warp_wait(bar_q, 0, abort_flag, p.err, 27);
      if (ok) {
        const uint8_t* rowp = (half == 0 ? sQ : sDO) + r * 128;
        const uint32_t dst = tmem + (half == 0 ? 384u : 448u) + lane_off;
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c) {
          uint32_t v[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 x = *reinterpret_cast<const uint4*>(rowp + c * kChunkBytes + ((j ^ (r & 7)) << 4));
            v[4 * j] = x.x;
            v[4 * j + 1] = x.y;
            v[4 * j + 2] = x.z;
            v[4 * j + 3] = x.w;
          }
          tmem_st32(dst + c * 32, v);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(bar_qt);
    }
    // dS = P o (dP - Delta) for keys [64 * half, 64 * half + 64) of each tile;
    // the half published first feeds the first half of dQ += dS K
    for (int i = 0; i < n && ok; ++i) {
      if (!warp_wait(bar_s, i & 1, abort_flag, p.err, 25)) { ok = false; break; }
      tc_fence_after();
      const int kv0 = (int)tiles[i] * kTileN;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t rs[32], rp[32];
        tmem_ld32(tS + c * 32, rs);
        tmem_ld32(tP + c * 32, rp);
        tmem_wait_ld();
        if (cc == 1) {  // this thread's S columns are read: S_{i+1} may overwrite them
          tc_fence_before();
          mbar_arrive(bar_sr);
        }
        const uint32_t bits = key_bits(mbits, use_mask, kv0 + 32 * c, p.Lk);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ((bits >> (2 * e)) & 1u) ? fast_exp2(fmaf(__uint_as_float(rs[2 * e]), sl2, -lse2)) : 0.f;
          const float p1 = ((bits >> (2 * e + 1)) & 1u) ? fast_exp2(fmaf(__uint_as_float(rs[2 * e + 1]), sl2, -lse2)) : 0.f;
          pk[e] = pack_bf16x2(p0 * (__uint_as_float(rp[2 * e]) - delta), p1 * (__uint_as_float(rp[2 * e + 1]) - delta));
        }
        // bf16 dS of keys [64h, 64h+64) packs into dP columns [64h, 64h+32):
        // each half overwrites only columns it has already read
        tmem_st16(tP + half * 64 + cc * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(half == 0 ? bar_ph : bar_p);
    }
    if (half == 0) {
      const bool have = ok && n > 0 && warp_wait(bar_o, 0, abort_flag, p.err, 26);
      tc_fence_after();
      const int64_t toff = (int64_t)b * p.qt_sb + (int64_t)hl * p.qt_sh + (int64_t)row * p.qt_st;
      grad_row_out<D>(tQ, have, row < p.Lq, p.scale,
                      p.qcos ? static_cast<const __nv_bfloat16*>(p.qcos) + toff : nullptr,
                      p.qcos ? static_cast<const __nv_bfloat16*>(p.qsin) + toff : nullptr, p.rope_vec != 0,
                      static_cast<__nv_bfloat16*>(p.dq) + (int64_t)b * p.dq_sb + (int64_t)hl * p.dq_sh + (int64_t)row * p.dq_st);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dK, dV: KV-stationary

template <int D>
struct DkvSmem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr uint32_t kOffK = 0, kOffV = kTile, kOffQ0 = 2 * kTile, kOffDO0 = 3 * kTile,
                            kOffQ1 = 4 * kTile, kOffDO1 = 5 * kTile;
  static constexpr uint32_t kOffL = 6 * kTile;  // lse2[2][128], delta[2][128]
  static constexpr uint32_t kOffBar = kOffL + 4 * 128 * 4;  // kv_full, q_full[2], q_empty[2], s_full, p_full, o_full, p_half, s_read
  static constexpr uint32_t kOffCtl = kOffBar + 10 * 8;
  static constexpr uint32_t kOffBits = kOffCtl + 16;
};

template <int D>
__device__ __forceinline__ void bwd_dkdv_body(const BwdParams& p, int tile, int hl, int b, int Hc) {
  using S = DkvSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sK = sm + S::kOffK;
  uint8_t* sV = sm + S::kOffV;
  // stage st of Q / dO lives at sQ0 / sDO0 + st * 2 * kTile
  uint8_t* sQ0 = sm + S::kOffQ0;
  uint8_t* sDO0 = sm + S::kOffDO0;
  static_assert(S::kOffQ1 == S::kOffQ0 + 2 * S::kTile && S::kOffDO1 == S::kOffDO0 + 2 * S::kTile, "stage stride");
  float* sL = reinterpret_cast<float*>(sm + S::kOffL);  // lse2: sL[st*128 + q]; delta: sL[256 + st*128 + q]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_kv = bars + 0;
  uint64_t* bar_qf = bars + 1;  // [2]
  uint64_t* bar_qe = bars + 3;  // [2]
  uint64_t* bar_s = bars + 5;
  uint64_t* bar_p = bars + 6;
  uint64_t* bar_o = bars + 7;
  uint64_t* bar_ph = bars + 8;  // P^T, dS^T for queries 0-63 stored (warps 0-3); bar_p: 64-127 (warps 4-7)
  uint64_t* bar_sr = bars + 9;  // every softmax thread has loaded its S^T columns: S^T may be overwritten
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  uint32_t* mbits = reinterpret_cast<uint32_t*>(sm + S::kOffBits);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv0 = tile * kTileN;
  const int nq = p.n_q_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(bars + i, i == 9 ? 256 : ((i == 6 || i == 8) ? 128 : 1));
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  const bool use_mask = p.mask != nullptr && load_mask_bits(p, b, mbits) != 0;
  uint32_t tile_bits = 0;
  if (use_mask) {
    const uint32_t* w4 = mbits + (kv0 / 32);
    tile_bits = w4[0] | w4[1] | w4[2] | w4[3];
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // a KV tile whose keys are all masked gets zero gradients and no work
  const int n = (use_mask && tile_bits == 0) ? 0 : nq;
  const int64_t lrow = ((int64_t)b * Hc + hl) * p.Lq_pad;

  if (warp == kProducerWarp) {
    if (lane == 0 && n > 0) {
      int issued = 0;
      mbar_arrive_expect_tx(bar_kv, 2 * S::kTile);
#pragma unroll
      for (int c = 0; c < S::kChunks; ++c) {
        tma_load_4d(&p.tm_k, bar_kv, sK + c * kChunkBytes, c * 64, kv0, hl, b);
        tma_load_4d(&p.tm_v, bar_kv, sV + c * kChunkBytes, c * 64, kv0, hl, b);
      }
      for (int j = 0; j < n; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(bar_qe + st, ((j >> 1) - 1) & 1, abort_flag, p.err, 31)) break;
        const int q0 = j * kTileM;
        mbar_arrive_expect_tx(bar_qf + st, 2 * S::kTile + 2 * 128 * 4);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c) {
          tma_load_4d(&p.tm_q, bar_qf + st, sQ0 + st * 2 * S::kTile + c * kChunkBytes, c * 64, q0, hl, b);
          tma_load_4d(&p.tm_do, bar_qf + st, sDO0 + st * 2 * S::kTile + c * kChunkBytes, c * 64, q0, hl, b);
        }
        bulk_load(sL + st * 128, p.lse2 + lrow + q0, 128 * 4, bar_qf + st);
        bulk_load(sL + 256 + st * 128, p.delta + lrow + q0, 128 * 4, bar_qf + st);
        ++issued;
      }
      drain_wait(bar_kv, 0);
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) drain_wait(bar_qf + (j & 1), (j >> 1) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0 && n > 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idesc_g = idesc_bf16_f32(128, D, 0, 1);
      const uint32_t tS = tmem, tP = tmem + 128, tV = tmem + 256, tK = tmem + 384;
      const SDesc dKd = sdesc_split(smem_u32(sK), 16, 1024), dVd = sdesc_split(smem_u32(sV), 16, 1024);
      // S^T_j = K Q_j^T and dP^T_j = V dO_j^T (both operands from shared memory)
      auto issue_s = [&](int st) {
        const SDesc dQd = sdesc_split(smem_u32(sQ0) + st * 2 * S::kTile, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_ss2(tS, dKd.lo + off, dKd.hi, dQd.lo + off, dQd.hi, idesc_s, kk > 0);
        }
      };
      auto issue_dp = [&](int st) {
        const SDesc dOd = sdesc_split(smem_u32(sDO0) + st * 2 * S::kTile, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
          umma_ss2(tP, dVd.lo + off, dVd.hi, dOd.lo + off, dOd.hi, idesc_s, kk > 0);
        }
      };
      // Order per Q tile j: S^T_{j+1} as soon as softmax has loaded S^T_j (P^T
      // and dS^T go to the dP^T columns, so the S^T columns are free early),
      // then dV += P^T dO and dK += dS^T Q in two halves, then dP^T_{j+1}.
      bool go = mbar_wait(bar_kv, 0, abort_flag, p.err, 32) && mbar_wait(bar_qf, 0, abort_flag, p.err, 33);
      if (go) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
        umma_commit(bar_s);
      }
      for (int j = 0; j < n && go; ++j) {
        const int st = j & 1, st1 = (j + 1) & 1;
        const bool more = j + 1 < n;
        const uint32_t aQ = smem_u32(sQ0) + st * 2 * S::kTile, aDO = smem_u32(sDO0) + st * 2 * S::kTile;
        const SDesc dQmn = sdesc_split(aQ, kChunkBytes, 1024), dOmn = sdesc_split(aDO, kChunkBytes, 1024);
        if (more) {
          if (!(go = mbar_wait(bar_sr, j & 1, abort_flag, p.err, 38))) break;
          if (!(go = mbar_wait(bar_qf + st1, ((j + 1) >> 1) & 1, abort_flag, p.err, 33))) break;
          tc_fence_after();
          issue_s(st1);
        }
        // dV += P^T dO and dK += dS^T Q in two halves of 64 queries: the first
        // runs while softmax finishes the second half
#pragma unroll
        for (int h = 0; h < 2 && go; ++h) {
          if (!(go = mbar_wait(h == 0 ? bar_ph : bar_p, j & 1, abort_flag, p.err, 34))) break;
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < kTileM / 32; ++k4) {
            const int kk = h * (kTileM / 32) + k4;  // queries 16kk..; P^T of half h at dP^T columns 64h + 16 (k4/2) + 8 (k4%2)
            umma_ts2(tV, tP + h * 64 + (k4 >> 1) * 32 + (k4 & 1) * 8, dOmn.lo + ((kk * 16 * 128) >> 4), dOmn.hi, idesc_g,
                     (j > 0 || kk > 0) ? 1u : 0u);
          }
#pragma unroll
          for (int k4 = 0; k4 < kTileM / 32; ++k4) {
            const int kk = h * (kTileM / 32) + k4;  // dS^T of half h at dP^T columns 64h + 16 + 16 (k4/2) + 8 (k4%2)
            umma_ts2(tK, tP + h * 64 + 16 + (k4 >> 1) * 32 + (k4 & 1) * 8, dQmn.lo + ((kk * 16 * 128) >> 4), dQmn.hi,
                     idesc_g, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        if (!go) break;
        umma_commit(bar_qe + st);
        if (more) {
          issue_dp(st1);
          umma_commit(bar_s);
        }
      }
      umma_commit(bar_o);
      drain_wait(bar_o, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off, tP = tmem + 128 + lane_off;
    const uint32_t tV = tmem + 256 + lane_off, tK = tmem + 384 + lane_off;
    const int key = kv0 + quad * 32 + lane;  // key of the tile = TMEM lane
    bool kvalid = key < p.Lk;
    if (use_mask && kvalid) kvalid = (mbits[key / 32] >> (key % 32)) & 1u;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int st = j & 1;
      if (!warp_wait(bar_s, j & 1, abort_flag, p.err, 35)) { ok = false; break; }
      // the lse / delta rows arrived with the Q tile
      if (!warp_wait(bar_qf + st, (j >> 1) & 1, abort_flag, p.err, 36)) { ok = false; break; }
      tc_fence_after();
      const float* L2 = sL + st * 128;
      const float* DL = sL + 256 + st * 128;
      // this warp's queries [64 * half, 64 * half + 64): both dP^T chunks are
      // loaded first, because P^T and dS^T of the first 32 queries land in the
      // second chunk's columns (16-column groups: P^T c0, dS^T c0, P^T c1,
      // dS^T c1 from column 64 * half)
      uint32_t rp0[32], rp1[32];
      tmem_ld32(tP + (2 * half) * 32, rp0);
      tmem_ld32(tP + (2 * half + 1) * 32, rp1);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t rs[32];
        tmem_ld32(tS + c * 32, rs);
        tmem_wait_ld();
        if (cc == 1) {  // this thread's S^T columns are read: S^T_{j+1} may overwrite them
          tc_fence_before();
          mbar_arrive(bar_sr);
        }
        const uint32_t* rp = cc == 0 ? rp0 : rp1;
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int q = c * 32 + 2 * e;
          const float p0 = kvalid ? fast_exp2(fmaf(__uint_as_float(rs[2 * e]), sl2, -L2[q])) : 0.f;
          const float p1 = kvalid ? fast_exp2(fmaf(__uint_as_float(rs[2 * e + 1]), sl2, -L2[q + 1])) : 0.f;
          pp[e] = pack_bf16x2(p0, p1);
          pd[e] = pack_bf16x2(p0 * (__uint_as_float(rp[2 * e]) - DL[q]), p1 * (__uint_as_float(rp[2 * e + 1]) - DL[q + 1]));
        }
        tmem_st16(tP + half * 64 + cc * 32, pp);
        tmem_st16(tP + half * 64 + cc * 32 + 16, pd);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(half == 0 ? bar_ph : bar_p);  // queries 0-63 feed the first half of dV and dK
    }
    const bool have = ok && n > 0 && warp_wait(bar_o, 0, abort_flag, p.err, 37);
    tc_fence_after();
    if (half == 0) {
      grad_row_out<D>(tV, have, key < p.Lk, 1.f, nullptr, nullptr, false,
                      static_cast<__nv_bfloat16*>(p.dv) + (int64_t)b * p.dv_sb + (int64_t)hl * p.dv_sh + (int64_t)key * p.dv_st);
    } else {
      const int64_t toff = (int64_t)b * p.kt_sb + (int64_t)hl * p.kt_sh + (int64_t)key * p.kt_st;
      grad_row_out<D>(tK, have, key < p.Lk, p.scale,
                      p.kcos ? static_cast<const __nv_bfloat16*>(p.kcos) + toff : nullptr,
                      p.kcos ? static_cast<const __nv_bfloat16*>(p.ksin) + toff : nullptr, p.rope_vec != 0,
                      static_cast<__nv_bfloat16*>(p.dk) + (int64_t)b * p.dk_sb + (int64_t)hl * p.dk_sh + (int64_t)key * p.dk_st);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Both gradient passes in one launch: the dK/dV CTAs (the longer ones) first,
// then the dQ CTAs.  They are independent (each writes only its own
// gradient), and as one grid the tail of the first kind fills with CTAs of the
// second instead of leaving SMs idle at the end of each of two launches.
template <int D>
__global__ void __launch_bounds__(kThreads, 1) bwd_sm100_kernel(const __grid_constant__ BwdParams p, int Hc, int B) {
  const int n_kv = p.n_kv_tiles * Hc * B;
  int cta = blockIdx.x;
  if (cta < n_kv) {
    bwd_dkdv_body<D>(p, cta % p.n_kv_tiles, (cta / p.n_kv_tiles) % Hc, cta / (p.n_kv_tiles * Hc), Hc);
  } else {
    cta -= n_kv;
    bwd_dq_body<D>(p, cta % p.n_q_tiles, (cta / p.n_q_tiles) % Hc, cta / (p.n_q_tiles * Hc), Hc);
  }
}

template <typename K>
cudaError_t set_smem(K kernel, size_t smem) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

}  // namespace

size_t bwd_dq_smem_bytes(int D, int Lk, bool has_mask) {
  const int n_tiles = (Lk + kTileN - 1) / kTileN;
  const size_t fixed = D == 128 ? DqSmem<128>::kOffBits : DqSmem<64>::kOffBits;
  return 1024 + fixed + (has_mask ? (size_t)n_tiles * 16 : 0);
}

size_t bwd_dkdv_smem_bytes(int D, int Lk, bool has_mask) {
  const int n_tiles = (Lk + kTileN - 1) / kTileN;
  const size_t fixed = D == 128 ? DkvSmem<128>::kOffBits : DkvSmem<64>::kOffBits;
  return 1024 + fixed + (has_mask ? (size_t)n_tiles * 16 : 0);
}

cudaError_t launch_bwd_prep(const BwdPrepParams& p, cudaStream_t s) {
  const int64_t threads = (int64_t)p.B * p.Hc * p.Lq_pad * 32;
  const int blocks = (int)((threads + 255) / 256);
  if (p.f32) {
    if (p.D == 128)
      bwd_prep_kernel<128, float><<<blocks, 256, 0, s>>>(p);
    else
      bwd_prep_kernel<64, float><<<blocks, 256, 0, s>>>(p);
  } else {
    if (p.D == 128)
      bwd_prep_kernel<128, __nv_bfloat16><<<blocks, 256, 0, s>>>(p);
    else
      bwd_prep_kernel<64, __nv_bfloat16><<<blocks, 256, 0, s>>>(p);
  }
  return cudaGetLastError();
}

namespace {
constexpr int kMaxDev = 64;
std::mutex g_prep_mu;
size_t g_smem_set[kMaxDev][2] = {};  // [device][D == 128]
}  // namespace

// Shared-memory attribute of the backward kernel (the larger of the two
// passes' layouts), set once per device and size (cached), so the launches of
// a call queue back to back.
cudaError_t prepare_bwd_bf16(int D, size_t smem_dq, size_t smem_dkdv) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int di = D == 128 ? 1 : 0;
  const size_t smem = smem_dq > smem_dkdv ? smem_dq : smem_dkdv;
  std::lock_guard<std::mutex> lock(g_prep_mu);
  if (smem > g_smem_set[dev][di]) {
    e = D == 128 ? set_smem(bwd_sm100_kernel<128>, smem) : set_smem(bwd_sm100_kernel<64>, smem);
    if (e != cudaSuccess) return e;
    g_smem_set[dev][di] = smem;
  }
  return cudaSuccess;
}

cudaError_t launch_bwd_bf16(const BwdParams& p, int D, int Hc, int B, size_t smem_dq, size_t smem_dkdv,
                            cudaStream_t s) {
  const int64_t ctas = ((int64_t)p.n_kv_tiles + p.n_q_tiles) * Hc * B;
  if (ctas > INT32_MAX) return cudaErrorInvalidConfiguration;
  const size_t smem = smem_dq > smem_dkdv ? smem_dq : smem_dkdv;
  if (D == 128)
    bwd_sm100_kernel<128><<<(unsigned)ctas, kThreads, smem, s>>>(p, Hc, B);
  else
    bwd_sm100_kernel<64><<<(unsigned)ctas, kThreads, smem, s>>>(p, Hc, B);
  return cudaGetLastError();
}
}  // namespace ltx
