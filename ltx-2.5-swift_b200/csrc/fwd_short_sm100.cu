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
//   - the MMA thread issues S of unit i+1 right behind P V of unit i, per Q
//     tile (PV0_i, S0_{i+1}, PV1_i, S1_{i+1}), so the two tiles' softmaxes
//     alternate on the exponential unit instead of competing for it;
//   - a dedicated epilogue warpgroup normalises, gates and stores unit i's O
//     (staged in shared memory, stored with TMA) while the softmax warpgroups
//     already work on unit i+1.
// The arithmetic per row is the forward kernel's with a single KV tile (the
// same exponentials, the same P rounding, the same row-sum order), so both
// kernels give the same bits.
//
// 512 threads: warps 0-3 softmax of Q tile 0, warps 4-7 of Q tile 1, warp 8
// TMA producer (lane 0), warp 9 TMEM owner and MMA issuer (lane 0), warps
// 12-15 the epilogue of both tiles (thread r owns row r of each; warps 10-11
// idle).  Registers: launched at 128 per thread, the softmax warpgroups take
// 184 and the other two 72 (2*128*184 + 2*128*72 = 512*128).  TMEM: S0
// [0,128), S1 [128,256), O0 [256,256+D), O1 [384,384+D).  The softmax hands
// each row's max and sum to the epilogue through shared memory,
// double-buffered by unit.  Both Q tiles of a unit are always computed; a
// tile past q_len reads zeros and is not stored.
//
// Where P_t lives.  With D = 64, O_t takes 64 columns and P_t (bf16, two per
// column) gets the other 64 of its 128-column block: P0 [320,384), P1
// [448,512).  The softmax then frees the S_t columns as soon as it has loaded
// S_t into registers (s_read), and the MMA thread issues S_t of the next unit
// right away, before P V_t of this one: while the softmax exponentiates unit
// i, the tensor pipe already computes unit i + 1's scores, so the softmax
// warps go from one unit to the next without waiting for P V and S.  Before
// writing P_t of unit i + 1 the softmax waits for P V_t of unit i (pv_done).
// With D = 128 the O tiles fill TMEM and P_t overwrites the first 64 columns
// of S_t: S_t of the next unit then follows P V_t of this one.
//
// Every wait is bounded.  A warpgroup decides to stop only at a reducing named
// barrier that all four of its warps reach each unit, so a timeout seen by one
// warp never leaves another parked at a barrier.
#include <mutex>

#include "fwd_common.cuh"

namespace ltx {

namespace {

constexpr int kShortThreads = 512;
constexpr uint32_t kShortLaunchRegs = 128;  // 65536 / 512
constexpr uint32_t kShortSoftmaxRegs = 184;
constexpr uint32_t kShortOtherRegs = 72;
static_assert(2 * 128 * kShortSoftmaxRegs + 2 * 128 * kShortOtherRegs <= kShortThreads * kShortLaunchRegs,
              "register re-split exceeds the launch allocation");

// Q is double-buffered where shared memory allows (D = 64: the next unit's Q
// loads a whole unit ahead); with D = 128 one buffer fits beside K, V and the
// staging tiles.
template <int D>
struct ShortSmem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr int kQBuf = D == 64 ? 2 : 1;
  static constexpr uint32_t kOffQ = 0, kOffK = 2 * kQBuf * kTile, kOffV = kOffK + kTile, kOffO = kOffV + kTile;
  // q_full[2], q_free[2], kv_full, kv_free, s_full[2], p_half[2], p_full[2], o_full, o_free[2],
  // mma_done, stat[2 unit parities][2 tiles], s_read[2], pv_done[2]
  static constexpr int kBars = 24;
  static constexpr bool kSplitP = D == 64;  // P_t in its own TMEM columns (see above)
  static constexpr uint32_t kOffBar = kOffO + 2 * kTile;
  static constexpr uint32_t kOffCtl = kOffBar + kBars * 8;  // tmem slot, abort flag
  static constexpr uint32_t kOffRow = kOffCtl + 16;         // float2 (max, sum) [2 units][2 tiles][128 rows]
  static constexpr uint32_t kBytes = kOffRow + 2 * 2 * 128 * 8;
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
__global__ void __launch_bounds__(kShortThreads, 1)
    fwd_short_sm100_kernel(const __grid_constant__ FwdParams p, int per_cta, int units) {
  using S = ShortSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm + S::kOffQ;  // Q tile t of buffer qb at sQ + (2 * qb + t) * kTile
  uint8_t* sK = sm + S::kOffK;
  uint8_t* sV = sm + S::kOffV;
  uint8_t* sO = sm + S::kOffO;  // epilogue staging of tile t at sO + t * kTile
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_qfull = bars + 0;  // [Q buffer]
  uint64_t* bar_qfree = bars + 2;  // [Q buffer]
  uint64_t* bar_kvfull = bars + 4;
  uint64_t* bar_kvfree = bars + 5;
  uint64_t* bar_s = bars + 6;      // [2]
  uint64_t* bar_ph = bars + 8;     // [2]
  uint64_t* bar_p = bars + 10;     // [2]
  uint64_t* bar_o = bars + 12;
  uint64_t* bar_ofree = bars + 13; // [2]
  uint64_t* bar_done = bars + 15;
  // (max, sum) of unit i's rows of tile t written: stat[(i & 1) * 2 + t], one
  // phase every second unit, so the epilogue (which must release O of unit i
  // before the softmax can reach unit i + 2) never sees it two phases ahead
  uint64_t* bar_stat = bars + 16;
  uint64_t* bar_sread = bars + 20;  // [2] S_t of a unit loaded by its softmax (128 arrivals; kSplitP)
  uint64_t* bar_pvd = bars + 22;    // [2] P V_t of a unit complete (kSplitP)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  float2* rowstat = reinterpret_cast<float2*>(sm + S::kOffRow);  // [(i & 1) * 2 + t][row]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u0 = blockIdx.x * per_cta;
  const int cnt = min(per_cta, units - u0);

  if (warp == 8 && lane == 0) {
    for (int i = 0; i < S::kBars; ++i)
      mbar_init(bars + i, (i >= 8 && i <= 11) || i == 13 || i == 14 || (i >= 16 && i <= 21) ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    // the first unit's Q and K/V loads start here, overlapping TMEM allocation
    // and the rest of the prologue (the producer loop skips them)
    if (cnt > 0) {
      grid_dep_wait();  // the kernel that wrote q / k (the RoPE pre-pass) has completed
      const ShortUnit u = short_unit(p, u0);
      const int qh = p.q_head_off + u.hl, kvh = (p.kv_head_off + u.hl) / p.group;
      mbar_arrive_expect_tx(bar_qfull, 2 * S::kTile);
#pragma unroll
      for (int c = 0; c < S::kChunks; ++c) {
        tma_load_4d(&p.tm_q, bar_qfull, sQ + c * kChunkBytes, c * 64, u.q0, qh, u.b);
        tma_load_4d(&p.tm_q, bar_qfull, sQ + S::kTile + c * kChunkBytes, c * 64, u.q0 + kTileM, qh, u.b);
      }
      mbar_arrive_expect_tx(bar_kvfull, 2 * S::kTile);
#pragma unroll
      for (int c = 0; c < S::kChunks; ++c) {
        tma_load_4d(&p.tm_k, bar_kvfull, sK + c * kChunkBytes, c * 64, 0, kvh, u.b);
        tma_load_4d(&p.tm_v, bar_kvfull, sV + c * kChunkBytes, c * 64, 0, kvh, u.b);
      }
    }
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
  grid_dep_wait();  // the kernel that wrote q / k (the RoPE pre-pass) has completed

  if (warp >= 12) {
    setmaxnreg_dec<kShortOtherRegs>();
    // ---------------- epilogue of both Q tiles ----------------
    const int r = threadIdx.x & 127;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    for (int i = 0; i < cnt; ++i) {
      const ShortUnit u = short_unit(p, u0 + i);
      ok = ok && warp_wait(bar_o, i & 1, abort_flag, p.err, 27);
      tc_fence_after();
      if (r == 0) bulk_wait_read();  // the previous unit's store has read the staging tiles
      named_barrier(3, 128);
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        const int row = u.q0 + t * kTileM + r;
        ok = ok && warp_wait(bar_stat + (i & 1) * 2 + t, (i >> 1) & 1, abort_flag, p.err, 28);
        const float2 ms = rowstat[((i & 1) * 2 + t) * 128 + r];
        const float l = ms.y;
        const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
        uint32_t g2 = 0x3f803f80u;  // bf16x2 (1, 1)
        if (p.gate != nullptr && row < p.Lq) {
          const float g = gate_bf16(__bfloat162float(
              p.gate[(int64_t)u.b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + u.hl) * p.g_sh]));
          g2 = pack_bf16x2(g, g);
        }
        const uint32_t tO = tmem + 256 + t * 128 + lane_off;
        uint8_t* srow = sO + t * S::kTile + r * 128;
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
        // O_t is in registers and shared memory: the next unit's P V may overwrite it
        tc_fence_before();
        mbar_arrive(bar_ofree + t);
        if (p.lse != nullptr && row < p.Lq) {
          p.lse[(int64_t)u.b * p.lse_sb + (int64_t)(p.head_begin + u.hl) * p.lse_sh + row] =
              (l > 0.f) ? (ms.x + log2f(l)) * kLn2 : -INFINITY;
        }
      }
      fence_proxy_async_smem();  // the bulk copy reads these rows through the async proxy
      const bool all_ok = named_barrier_and(3, 128, ok);
      if (r == 0 && all_ok) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (u.q0 + t * kTileM >= p.Lq) continue;
#pragma unroll
          for (int ch = 0; ch < S::kChunks; ++ch)
            tma_store_4d(&p.tm_o, sO + t * S::kTile + ch * kChunkBytes, ch * 64, u.q0 + t * kTileM,
                         p.head_begin + u.hl, u.b);
        }
        bulk_commit();
      }
      if (!all_ok) break;
    }
    if (r == 0) bulk_wait_read();  // the CTA's shared memory must outlive the copies' reads
  } else if (warp >= 8) {
    setmaxnreg_dec<kShortOtherRegs>();
    if (warp == 8) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        // the first unit's Q and K/V were issued in the prologue
        int q_issued = cnt > 0 ? 1 : 0, kv_issued = cnt > 0 ? 1 : 0;
        int kv_prev = cnt > 0 ? short_unit(p, u0).kv_key : -1;
        for (int i = 1; i < cnt; ++i) {
          const ShortUnit u = short_unit(p, u0 + i);
          const int qh = p.q_head_off + u.hl;
          const int qb = i % S::kQBuf, qn = i / S::kQBuf;  // buffer, and its use count
          // the S MMAs of the unit that last used this buffer must have read it
          if (i >= S::kQBuf && !mbar_wait(bar_qfree + qb, (qn - 1) & 1, abort_flag, p.err, 20)) break;
          uint8_t* dst = sQ + 2 * qb * S::kTile;
          mbar_arrive_expect_tx(bar_qfull + qb, 2 * S::kTile);
#pragma unroll
          for (int c = 0; c < S::kChunks; ++c) {
            tma_load_4d(&p.tm_q, bar_qfull + qb, dst + c * kChunkBytes, c * 64, u.q0, qh, u.b);
            tma_load_4d(&p.tm_q, bar_qfull + qb, dst + S::kTile + c * kChunkBytes, c * 64, u.q0 + kTileM, qh, u.b);
          }
          ++q_issued;
          if (u.kv_key != kv_prev) {
            // the units of the previous K/V must be done with it: kv_free
            // completes one phase per reload (the MMA thread commits it only
            // after the last unit before a reload), so a phase-parity wait is
            // never more than one phase away from the barrier
            if (kv_issued > 0 && !mbar_wait(bar_kvfree, (kv_issued - 1) & 1, abort_flag, p.err, 21)) break;
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
        // (only the last copy into each buffer can still be in flight)
        for (int j = q_issued > S::kQBuf ? q_issued - S::kQBuf : 0; j < q_issued; ++j)
          drain_wait(bar_qfull + j % S::kQBuf, (j / S::kQBuf) & 1);
        if (kv_issued > 0) drain_wait(bar_kvfull, (kv_issued - 1) & 1);
      }
      __syncwarp();
    } else if (warp == 9) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
        const SDesc dQ = sdesc_split(smem_u32(sQ), 16, 1024);
        const SDesc dK = sdesc_split(smem_u32(sK), 16, 1024);
        const SDesc dV = sdesc_split(smem_u32(sV), kChunkBytes, 1024);
        auto qdesc = [&](int i, int t) {
          return SDesc{dQ.lo + (uint32_t)((i % S::kQBuf) * 2 + t) * (S::kTile >> 4), dQ.hi};
        };
        int kv_loads = 0, kv_prev = -1;
        // Q (and K/V when they change) of unit i in shared memory
        auto inputs_ready = [&](int i, const ShortUnit& u) {
          if (!mbar_wait(bar_qfull + i % S::kQBuf, (i / S::kQBuf) & 1, abort_flag, p.err, 22)) return false;
          if (u.kv_key != kv_prev) {
            if (!mbar_wait(bar_kvfull, kv_loads & 1, abort_flag, p.err, 23)) return false;
            ++kv_loads;
            kv_prev = u.kv_key;
          }
          tc_fence_after();
          return true;
        };
        // P V of tile t of unit i (after its P halves, and after the epilogue
        // has read O_t of unit i - 1); P_t from its own columns (kSplitP) or
        // from the first 64 columns of S_t
        auto pv = [&](int i, int t) {
          const uint32_t tO = t ? tO1 : tO0;
          const uint32_t tP = S::kSplitP ? tO + 64 : (t ? tS1 : tS0);
          if (!mbar_wait(bar_ph + t, i & 1, abort_flag, p.err, 24)) return false;
          if (i > 0 && !mbar_wait(bar_ofree + t, (i - 1) & 1, abort_flag, p.err, 25)) return false;
          tc_fence_after();
          issue_pv_half<D>(tO, tP, dV, false, 0);
          if (!mbar_wait(bar_p + t, i & 1, abort_flag, p.err, 24)) return false;
          tc_fence_after();
          issue_pv_half<D>(tO, tP, dV, true, 1);
          if (S::kSplitP) umma_commit(bar_pvd + t);
          return true;
        };
        // kSplitP: S_t of unit i + 1 once the softmax has loaded S_t of unit i
        auto s_next = [&](int i, int t) {
          if (!mbar_wait(bar_sread + t, i & 1, abort_flag, p.err, 29)) return false;
          tc_fence_after();
          issue_s<D>(t ? tS1 : tS0, qdesc(i + 1, t), dK);
          umma_commit(bar_s + t);
          return true;
        };
        ShortUnit cur = short_unit(p, u0);
        bool go = inputs_ready(0, cur);
        if (go) {
          issue_s<D>(tS0, qdesc(0, 0), dK);
          umma_commit(bar_s + 0);
          issue_s<D>(tS1, qdesc(0, 1), dK);
          umma_commit(bar_s + 1);
          umma_commit(bar_qfree + 0);
        }
        // Issue order PV0_i, S0_{i+1}, PV1_i, S1_{i+1} when unit i+1 reuses
        // K/V and its Q has its own buffer, so the two tiles' softmaxes
        // alternate; otherwise both P V first (a K/V reload needs P V of
        // unit i done, and a single Q buffer fills only after S_i).
        for (int i = 0; i < cnt && go && S::kSplitP; ++i) {
          // S of unit i + 1 first when it reuses K/V (its Q has its own
          // buffer), then both P V of unit i; a K/V reload waits for P V of
          // unit i and so comes after it
          const bool more = i + 1 < cnt;
          const ShortUnit nxt = more ? short_unit(p, u0 + i + 1) : cur;
          const bool same_kv = more && nxt.kv_key == cur.kv_key;
          if (same_kv) {
            if (!(go = inputs_ready(i + 1, nxt) && s_next(i, 0) && s_next(i, 1))) break;
            umma_commit(bar_qfree + (i + 1) % S::kQBuf);
          }
          if (!(go = pv(i, 0) && pv(i, 1))) break;
          umma_commit(bar_o);
          if (more && !same_kv) {
            umma_commit(bar_kvfree);  // the next unit reloads K/V
            if (!(go = inputs_ready(i + 1, nxt) && s_next(i, 0) && s_next(i, 1))) break;
            umma_commit(bar_qfree + (i + 1) % S::kQBuf);
          }
          cur = nxt;
        }
        for (int i = 0; i < cnt && go && !S::kSplitP; ++i) {
          const bool more = i + 1 < cnt;
          const ShortUnit nxt = more ? short_unit(p, u0 + i + 1) : cur;
          const bool pingpong = S::kQBuf == 2 && more && nxt.kv_key == cur.kv_key;
          if (!(go = pv(i, 0))) break;
          if (pingpong) {
            if (!(go = inputs_ready(i + 1, nxt))) break;
            issue_s<D>(tS0, qdesc(i + 1, 0), dK);
            umma_commit(bar_s + 0);
          }
          if (!(go = pv(i, 1))) break;
          umma_commit(bar_o);
          if (more && nxt.kv_key != cur.kv_key) umma_commit(bar_kvfree);  // the next unit reloads K/V
          if (more) {
            if (!pingpong) {
              if (!(go = inputs_ready(i + 1, nxt))) break;
              issue_s<D>(tS0, qdesc(i + 1, 0), dK);
              umma_commit(bar_s + 0);
            }
            issue_s<D>(tS1, qdesc(i + 1, 1), dK);
            umma_commit(bar_s + 1);
            umma_commit(bar_qfree + (i + 1) % S::kQBuf);
          }
          cur = nxt;
        }
        umma_commit(bar_done);
        drain_wait(bar_done, 0);  // every issued MMA has completed
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kShortSoftmaxRegs>();
    // ---------------- softmax of Q tile t ----------------
    const int t = warp >> 2;
    const int r = threadIdx.x & 127;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tP = S::kSplitP ? tmem + 256 + t * 128 + 64 + lane_off : tS;  // where P_t goes
    const float sl2 = p.scale_log2;
    const int Lk = p.Lk;
    int mask_b = -1;
    bool mask_on = false;
    uint32_t mw[4] = {~0u, ~0u, ~0u, ~0u};
    bool ok = true;
    for (int i = 0; i < cnt; ++i) {
      const ShortUnit u = short_unit(p, u0 + i);
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
      if (S::kSplitP) {  // S_t is in registers: the next unit's S_t may overwrite its columns
        tc_fence_before();
        mbar_arrive(bar_sread + t);
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
        if (h2 == 1) {  // the row's (max, sum) for the epilogue, before the hand-off
          const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
          const float2 tot = add2(a01, a23);
          float l = 0.f;
          l += tot.x + tot.y;
          rowstat[((i & 1) * 2 + t) * 128 + r] = make_float2(m, l);
          mbar_arrive(bar_stat + (i & 1) * 2 + t);
        }
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_bf16x2(s[64 * h2 + 2 * e], s[64 * h2 + 2 * e + 1]);
        if (S::kSplitP && h2 == 0 && i > 0) {  // P V_t of the previous unit has read the P_t columns
          ok = ok && warp_wait(bar_pvd + t, (i - 1) & 1, abort_flag, p.err, 30);
          tc_fence_after();
        }
        tmem_st32(tP + 32 * h2, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(h2 == 0 ? bar_ph + t : bar_p + t);
      }
      if (!named_barrier_and(1 + t, 128, ok)) break;
    }
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
  if (fa.numRegs != (int)kShortLaunchRegs) return cudaErrorInvalidConfiguration;
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
  if (D == 128) return launch_pdl(fwd_short_sm100_kernel<128>, dim3(grid), dim3(kShortThreads), smem, s, p, per, units);
  return launch_pdl(fwd_short_sm100_kernel<64>, dim3(grid), dim3(kShortThreads), smem, s, p, per, units);
}

}  // namespace ltx
