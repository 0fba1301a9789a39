// fwd_short_sm100.cu -- the bf16 forward for key/value sequences that fit in
// one 128-key tile (kv_len <= 128), run persistently.
//
// At the reference geometry this is the audio->video cross-attention (3120
// video queries against 126 audio keys, DiTAttention.swift:369-382 with
// DiT keys from the audio stream).  With one KV tile a 256-row query block
// costs a single S = Q K^T, one softmax and one P V: too little work to hide a
// CTA's launch, its Q load and its epilogue, and the one-CTA-per-SM forward
// kernel spends most of such a launch in those.  Here each CTA walks a
// contiguous range of units (256-row query block, head, batch; block fastest)
// and overlaps consecutive units:
//   - the producer loads Q of unit i+1 as soon as the S MMAs of unit i have
//     read Q, and K/V only when the (kv head, batch) changes;
//   - the MMA thread issues S of unit i+1 right after P V of unit i, while the
//     softmax warps run unit i's epilogue;
//   - each softmax warpgroup stages its O rows in its own shared-memory tile
//     and stores them with TMA, waiting for the previous unit's store to have
//     read the staging area only when it needs it again.
// The arithmetic per row is the forward kernel's with a single KV tile (the
// same exponentials, the same P rounding, the same row-sum order), so both
// kernels give the same bits.
//
// Warp roles as in the forward kernel: warps 0-3 softmax + epilogue of Q tile
// 0, warps 4-7 of Q tile 1, warp 8 TMA producer (lane 0), warp 9 TMEM owner
// and MMA issuer (lane 0).  TMEM: S0 [0,128), S1 [128,256), O0 [256,256+D),
// O1 [384,384+D); P_t overwrites the first 64 columns of S_t.  Both Q tiles
// of a unit are always computed; a tile past q_len reads zeros and is not
// stored.
//
// Every wait is bounded.  A softmax warpgroup decides to stop only at a
// reducing named barrier that all four of its warps reach each unit, so a
// timeout seen by one warp never leaves another parked at a barrier.
#include <mutex>

#include "fwd_common.cuh"

namespace ltx {

namespace {

template <int D>
struct ShortSmem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr uint32_t kOffQ = 0, kOffK = 2 * kTile, kOffV = 3 * kTile, kOffO = 4 * kTile;
  // q_full, q_free, kv_full, kv_free, s_full[2], p_half[2], p_full[2], o_full, o_free[2], mma_done
  static constexpr int kBars = 14;
  static constexpr uint32_t kOffBar = 6 * kTile;
  static constexpr uint32_t kOffCtl = kOffBar + kBars * 8;  // tmem slot, abort flag
  static constexpr uint32_t kBytes = kOffCtl + 16;
};

struct ShortUnit {
  int q0, hl, b, kv_key;
};

__device__ __forceinline__ ShortUnit short_unit(const FwdParams& p, int unit) {
  ShortUnit u;
  u.q0 = (unit % p.q_blocks) * kBlockM;
  u.hl = (unit / p.q_blocks) % p.Hc;
  u.b = unit / (p.q_blocks * p.Hc);
  u.kv_key = ((p.kv_head_off + u.hl) / p.group) + 65536 * u.b;  // the K/V a unit reads
  return u;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_short_sm100_kernel(const __grid_constant__ FwdParams p, int per_cta, int units) {
  using S = ShortSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm + S::kOffQ;  // Q tile t at sQ + t * kTile
  uint8_t* sK = sm + S::kOffK;
  uint8_t* sV = sm + S::kOffV;
  uint8_t* sO = sm + S::kOffO;  // epilogue staging of tile t at sO + t * kTile
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_qfull = bars + 0;
  uint64_t* bar_qfree = bars + 1;
  uint64_t* bar_kvfull = bars + 2;
  uint64_t* bar_kvfree = bars + 3;
  uint64_t* bar_s = bars + 4;      // [2]
  uint64_t* bar_ph = bars + 6;     // [2]
  uint64_t* bar_p = bars + 8;      // [2]
  uint64_t* bar_o = bars + 10;
  uint64_t* bar_ofree = bars + 11; // [2]
  uint64_t* bar_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u0 = blockIdx.x * per_cta;
  const int cnt = min(per_cta, units - u0);

  if (warp == 8 && lane == 0) {
    for (int i = 0; i < S::kBars; ++i) mbar_init(bars + i, (i >= 6 && i <= 9) || i == 11 || i == 12 ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_o);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    setmaxnreg_dec<kProducerRegs>();
    if (warp == 8) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        int q_issued = 0, kv_issued = 0, kv_prev = -1;
        for (int i = 0; i < cnt; ++i) {
          const ShortUnit u = short_unit(p, u0 + i);
          const int qh = p.q_head_off + u.hl;
          if (i > 0 && !mbar_wait(bar_qfree, (i - 1) & 1, abort_flag, p.err, 20)) break;
          mbar_arrive_expect_tx(bar_qfull, 2 * S::kTile);
#pragma unroll
          for (int c = 0; c < S::kChunks; ++c) {
            tma_load_4d(&p.tm_q, bar_qfull, sQ + c * kChunkBytes, c * 64, u.q0, qh, u.b);
            tma_load_4d(&p.tm_q, bar_qfull, sQ + S::kTile + c * kChunkBytes, c * 64, u.q0 + kTileM, qh, u.b);
          }
          ++q_issued;
          if (u.kv_key != kv_prev) {
            // the previous unit's P V must have read V (and its S MMAs K)
            if (i > 0 && !mbar_wait(bar_kvfree, (i - 1) & 1, abort_flag, p.err, 21)) break;
            const int kvh = (p.kv_head_off + u.hl) / p.group;
            mbar_arrive_expect_tx(bar_kvfull, 2 * S::kTile);
#pragma unroll
            for (int c = 0; c < S::kChunks; ++c) {
              tma_load_4d(&p.tm_k, bar_kvfull, sK + c * kChunkBytes, c * 64, 0, kvh, u.b);
              tma_load_4d(&p.tm_v, bar_kvfull, sV + c * kChunkBytes, c * 64, 0, kvh, u.b);
            }
            ++kv_issued;
            kv_prev = u.kv_key;
          }
        }
        // never leave the CTA with a bulk copy still writing its shared memory
        // (every earlier copy was consumed before the next one was issued)
        if (q_issued > 0) drain_wait(bar_qfull, (q_issued - 1) & 1);
        if (kv_issued > 0) drain_wait(bar_kvfull, (kv_issued - 1) & 1);
      }
      __syncwarp();
    } else if (warp == 9) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        const uint32_t tS0 = tmem, tO0 = tmem + 256;
        const SDesc dQ0 = sdesc_split(smem_u32(sQ), 16, 1024);
        const SDesc dQ1 = sdesc_split(smem_u32(sQ) + S::kTile, 16, 1024);
        const SDesc dK = sdesc_split(smem_u32(sK), 16, 1024);
        const SDesc dV = sdesc_split(smem_u32(sV), kChunkBytes, 1024);
        int kv_loads = 0, kv_prev = -1;
        bool go = true;
        for (int i = 0; i < cnt && go; ++i) {
          const ShortUnit u = short_unit(p, u0 + i);
          if (!mbar_wait(bar_qfull, i & 1, abort_flag, p.err, 22)) break;
          if (u.kv_key != kv_prev) {
            if (!mbar_wait(bar_kvfull, kv_loads & 1, abort_flag, p.err, 23)) break;
            ++kv_loads;
            kv_prev = u.kv_key;
          }
          tc_fence_after();
          issue_s<D>(tS0, dQ0, dK);
          umma_commit(bar_s + 0);
          issue_s<D>(tS0 + 128, dQ1, dK);
          umma_commit(bar_s + 1);
          umma_commit(bar_qfree);  // both S MMAs have read Q
#pragma unroll 1
          for (int t = 0; t < 2 && go; ++t) {
            const uint32_t tS = tS0 + t * 128, tO = tO0 + t * 128;
            go = mbar_wait(bar_ph + t, i & 1, abort_flag, p.err, 24);
            // O_t of the previous unit must have been read by its epilogue
            if (go && i > 0) go = mbar_wait(bar_ofree + t, (i - 1) & 1, abort_flag, p.err, 25);
            if (!go) break;
            tc_fence_after();
            issue_pv_half<D>(tO, tS, dV, false, 0);
            go = mbar_wait(bar_p + t, i & 1, abort_flag, p.err, 24);
            if (!go) break;
            tc_fence_after();
            issue_pv_half<D>(tO, tS, dV, true, 1);
          }
          if (!go) break;
          umma_commit(bar_o);
          umma_commit(bar_kvfree);
        }
        umma_commit(bar_done);
        drain_wait(bar_done, 0);  // every issued MMA has completed
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ---------------- softmax and epilogue of Q tile t ----------------
    const int t = warp >> 2;
    const int r = threadIdx.x & 127;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tO = tmem + 256 + t * 128 + lane_off;
    const float sl2 = p.scale_log2;
    const int Lk = p.Lk;
    uint8_t* stg = sO + t * S::kTile;
    uint8_t* srow = stg + r * 128;
    int mask_b = -1;
    bool mask_on = false;
    uint32_t mw[4] = {~0u, ~0u, ~0u, ~0u};
    bool ok = true;
    for (int i = 0; i < cnt; ++i) {
      const ShortUnit u = short_unit(p, u0 + i);
      const int row = u.q0 + t * kTileM + r;
      // key-mask words of batch row b (each warp its own copy); a row with no
      // valid key attends to every key (GemmaTextEncoder.swift:306-319)
      if (p.mask != nullptr && u.b != mask_b) {
        const uint8_t* mrow = p.mask + (int64_t)u.b * p.mask_sb;
        uint32_t any = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int key = 32 * w + lane;
          mw[w] = __ballot_sync(0xffffffffu, key < Lk && mrow[key] != 0);
          any |= mw[w];
        }
        mask_on = any != 0u;
        mask_b = u.b;
      }
      uint32_t g2 = 0x3f803f80u;  // bf16x2 (1, 1)
      if (p.gate != nullptr && row < p.Lq) {
        const float g = gate_bf16(__bfloat162float(
            p.gate[(int64_t)u.b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + u.hl) * p.g_sh]));
        g2 = pack_bf16x2(g, g);
      }

      // softmax of the unit's single KV tile
      ok = ok && warp_wait(bar_s + t, i & 1, abort_flag, p.err, 26);
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
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t bits = mask_on ? mw[w] : ~0u;
        const int lim = Lk - 32 * w;
        if (lim < 32) bits &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!((bits >> c) & 1u)) s[32 * w + c] = -INFINITY;
      }
      float mx;
      {
        float pm[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) pm[e] = fmaxf(s[e], s[8 + e]);
#pragma unroll
        for (int c = 16; c < 128; c += 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) pm[e] = max3(pm[e], s[c + e], s[c + 8 + e]);
        }
        mx = max3(max3(pm[0], pm[1], pm[2]), max3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
      }
      const float m = mx * sl2;
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      const float2 sl2x2 = make_float2(sl2, sl2), nmx2 = make_float2(neg_m, neg_m);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
        for (int c = 64 * h2; c < 64 * h2 + 64; c += 2) {
          const float2 x = fma2(make_float2(s[c], s[c + 1]), sl2x2, nmx2);
          const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          s[c] = e.x;
          s[c + 1] = e.y;
          acc[(c >> 1) & 3] = add2(acc[(c >> 1) & 3], e);
        }
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[64 * h2 + 2 * e], s[64 * h2 + 2 * e + 1]);
        tmem_st32(tS + 32 * h2, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(h2 == 0 ? bar_ph + t : bar_p + t);
      }
      float l;
      {
        const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const float2 tot = add2(a01, a23);
        l = 0.f;
        l += tot.x + tot.y;
      }

      // epilogue: O_t to registers, release it to the next unit's P V, then
      // stage (128-byte swizzle) and store with TMA
      ok = ok && warp_wait(bar_o, i & 1, abort_flag, p.err, 27);
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      if (r == 0) bulk_wait_read();  // the previous unit's store has read the staging tile
      named_barrier(1 + t, 128);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(o[8 * e + 0]) * inv_l, __uint_as_float(o[8 * e + 1]) * inv_l);
          v.y = pack_bf16x2(__uint_as_float(o[8 * e + 2]) * inv_l, __uint_as_float(o[8 * e + 3]) * inv_l);
          v.z = pack_bf16x2(__uint_as_float(o[8 * e + 4]) * inv_l, __uint_as_float(o[8 * e + 5]) * inv_l);
          v.w = pack_bf16x2(__uint_as_float(o[8 * e + 6]) * inv_l, __uint_as_float(o[8 * e + 7]) * inv_l);
          if (p.gate != nullptr) {
            v.x = bmul2(v.x, g2);
            v.y = bmul2(v.y, g2);
            v.z = bmul2(v.z, g2);
            v.w = bmul2(v.w, g2);
          }
          const int j = (c & 1) * 4 + e;
          *reinterpret_cast<uint4*>(srow + (c >> 1) * kChunkBytes + ((j ^ (r & 7)) << 4)) = v;
        }
      }
      tc_fence_before();
      mbar_arrive(bar_ofree + t);
      if (p.lse != nullptr && row < p.Lq) {
        p.lse[(int64_t)u.b * p.lse_sb + (int64_t)(p.head_begin + u.hl) * p.lse_sh + row] =
            (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
      }
      fence_proxy_async_smem();  // the bulk copy reads these rows through the async proxy
      const bool all_ok = named_barrier_and(1 + t, 128, ok);
      if (r == 0 && all_ok && u.q0 + t * kTileM < p.Lq) {
#pragma unroll
        for (int ch = 0; ch < S::kChunks; ++ch)
          tma_store_4d(&p.tm_o, stg + ch * kChunkBytes, ch * 64, u.q0 + t * kTileM, p.head_begin + u.hl, u.b);
        bulk_commit();
      }
      if (!all_ok) break;
    }
    if (r == 0) bulk_wait_read();  // the CTA's shared memory must outlive the copies' reads
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

constexpr int kMaxDev = 64;
std::mutex g_short_mu;
bool g_short_ready[kMaxDev][2] = {};

}  // namespace

size_t fwd_short_smem_bytes(int D) {
  return 1024 /* alignment slack */ + (D == 128 ? ShortSmem<128>::kBytes : ShortSmem<64>::kBytes);
}

// Once per device and head dim: the register count the warpgroup split
// assumes, and the dynamic shared-memory limit.
cudaError_t prepare_fwd_short(int D) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int di = D == 128 ? 1 : 0;
  std::lock_guard<std::mutex> lock(g_short_mu);
  if (g_short_ready[dev][di]) return cudaSuccess;
  const void* k = D == 128 ? (const void*)fwd_short_sm100_kernel<128> : (const void*)fwd_short_sm100_kernel<64>;
  cudaFuncAttributes fa;
  if ((e = cudaFuncGetAttributes(&fa, k)) != cudaSuccess) return e;
  if (fa.numRegs != (int)kLaunchRegs) return cudaErrorInvalidConfiguration;
  if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_short_smem_bytes(D))) !=
      cudaSuccess)
    return e;
  g_short_ready[dev][di] = true;
  return cudaSuccess;
}

cudaError_t launch_fwd_short(const FwdParams& p, int D, int units, int sms, cudaStream_t s) {
  const int per = (units + sms - 1) / sms;
  const int grid = (units + per - 1) / per;
  const size_t smem = fwd_short_smem_bytes(D);
  if (D == 128)
    fwd_short_sm100_kernel<128><<<grid, kThreads, smem, s>>>(p, per, units);
  else
    fwd_short_sm100_kernel<64><<<grid, kThreads, smem, s>>>(p, per, units);
  return cudaGetLastError();
}

}  // namespace ltx
