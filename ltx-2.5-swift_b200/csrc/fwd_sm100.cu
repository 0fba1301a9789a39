// fwd_sm100.cu -- bf16 fused attention forward on tcgen05 (sm_100a).
//
// Computes, per (batch, head, 256-row query block):
//     O = softmax(scale * Q K^T + mask) V,   lse = log sum exp(scale * Q K^T + mask)
// the function of DiTAttention.swift:369-382 (fused arm: MLXFast SDPA;
// explicit arm: fp32 logits -> softmax -> PV), online-softmax style with O(N)
// memory: no score matrix leaves the SM.
//
// CTA layout (384 threads = 3 warpgroups, one CTA per SM, two 128-row Q
// tiles sharing K/V):
//   warps 0-3  softmax of Q tile 0 (thread i owns row i = TMEM lane i;
//              warp w reads lane quadrant w % 4); also the lazy O rescale and
//              the epilogue of tile 0
//   warps 4-7  the same for Q tile 1
//   warp 8     TMA producer (lane 0): Q0/Q1 once, K_j and V_j through two stages
//   warp 9     TMEM owner; lane 0 issues every tcgen05.mma
//   warps 10-11 idle (they complete the third warpgroup)
// Registers: launched at kLaunchRegs per thread; the producer warpgroup gives
// its share to the softmax warpgroups (setmaxnreg), which hold a 128-wide
// score row each: 2*128*kSoftmaxRegs + 128*kProducerRegs = 384*kLaunchRegs.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+D), O1 [384,384+D).
// P_t (bf16, two per column) overwrites the first 64 columns of S_t and feeds
// the PV MMA straight from TMEM.  Softmax publishes P_t in two halves (keys
// 0-63, then 64-127; barriers p_half and p_full), so the first four k-steps
// of PV_t run while the second half is still being exponentiated.
//
// MMA issue order in steady state:  PV0_j, S0_{j+1}, PV1_j, S1_{j+1}.
// tcgen05 ops of one thread execute in order, so S_t{j+1} never overwrites
// P_t{j} before PV_t{j} has read it, and the commit that publishes S_t{j+1}
// also proves PV_t{j} finished, so softmax t may rescale O_t.  While softmax 0
// works on tile j+1 the tensor pipe runs PV1_j and S1_{j+1}, and vice versa.
//
// Online softmax in the log2 domain with a lazy max: the running max m only
// moves when a tile's max exceeds it by more than 8 (a factor of 256), so O is
// rescaled rarely; exp2(s - m) then stays <= 256, which fp32 and bf16 carry
// exactly as well as values <= 1.  The final O / l is the same function.
// Every exponential runs on the MUFU (ex2.approx.f32).  Measured alternatives
// that were slower at config 2: an FMA-pipe polynomial for an eighth or a
// quarter of them (exp2_poly2; kPolyCols keeps the option, at 0) and paired
// f16 exponentials (ex2.approx.f16x2; the widening conversions share the MUFU pipe).
//
// Keys: a tile whose keys are all masked is skipped outright (its weight is
// exactly zero); partial tiles and the ragged tail get -inf logits per
// column.  A batch row whose mask has no valid key attends to all keys
// (GemmaTextEncoder.swift:306-319).
//
// Work units are (256-row query block, head, batch), q_block fastest, on a
// 1-D grid.  The first n_full units run whole, one CTA each, and store O
// directly.  Each later ("tail") unit runs as num_splits CTAs, each over a
// contiguous share of the unit's active KV tiles, writing an fp32 partial O
// (normalised by its own l) and its log2-domain lse; the combine kernel merges
// them.  CTAs start roughly in index order, so the split CTAs fill what would
// otherwise be a thin last wave; short query sequences split every unit.
#include <mutex>

#include "fwd_common.cuh"

namespace ltx {

namespace {

// Exponentials per 128-column row evaluated on the FMA pipe (exp2_poly2)
// instead of the MUFU; pair p of a row uses the polynomial when p % 8 < kPolyCols / 16.
#ifndef LTX_FWD_POLY_COLS
#define LTX_FWD_POLY_COLS 0
#endif
constexpr int kPolyCols = LTX_FWD_POLY_COLS;
static_assert(kPolyCols % 16 == 0 && kPolyCols <= 128, "polynomial share is whole 16-column groups");

template <int D>
struct Smem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr uint32_t kOffQ0 = 0, kOffQ1 = kTile, kOffK0 = 2 * kTile, kOffK1 = 3 * kTile,
                            kOffV0 = 4 * kTile, kOffV1 = 5 * kTile;
  // q0_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full[2], o_full, p_half[2], q1_full
  static constexpr uint32_t kOffBar = 6 * kTile;
  static constexpr uint32_t kOffCtl = kOffBar + 17 * 8;  // tmem slot, abort, n_tiles
  static constexpr uint32_t kOffTiles = kOffCtl + 16;    // uint16 [kMaxKvTiles]
  static constexpr uint32_t kOffBits = kOffTiles + 2 * kMaxKvTiles;  // uint32 mask bits
};

// The work unit and KV share of CTA `cta` (see the grid layout above).
struct Unit {
  int q_block, hl, b;  // 256-row query block, local head, batch
  int split, ns;       // KV share split of ns (ns == 1: the whole unit)
  int tail;            // index among the split units (ns > 1)
};

__device__ __forceinline__ Unit decode_unit(const FwdParams& p, int cta) {
  Unit u;
  int unit = cta;
  u.split = 0;
  u.ns = 1;
  if (unit >= p.n_full) {
    const int c = unit - p.n_full;
    u.ns = p.num_splits;
    unit = p.n_full + c / u.ns;
    u.split = c - (c / u.ns) * u.ns;
  }
  u.tail = unit - p.n_full;
  u.q_block = unit % p.q_blocks;
  u.hl = (unit / p.q_blocks) % p.Hc;
  u.b = unit / (p.q_blocks * p.Hc);
  return u;
}

// %ctaid.x read that the compiler cannot merge with an earlier read: the
// epilogue decodes its unit again instead of keeping it live through the loop.
__device__ __forceinline__ int ctaid_x_fresh() {
  int x;
  asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(x));
  return x;
}

// kBanded: causal / sliding-window rows and the free-row rule (the Gemma
// encoder's self-attention); the DiT's attention runs the kBanded = false
// instance, which carries none of that per-row state.
template <int D, bool kBanded>
__global__ void __launch_bounds__(kThreads, 1) fwd_bf16_sm100_kernel(const __grid_constant__ FwdParams p) {
  using S = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  // stage st of K lives at sK + st * kTile, of V at sV + st * kTile; Q tile t at sQ + t * kTile
  uint8_t* sQ = sm + S::kOffQ0;
  uint8_t* sK = sm + S::kOffK0;
  uint8_t* sV = sm + S::kOffV0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_q = bars + 0;   // Q tile 0 loaded
  uint64_t* bar_q1 = bars + 16; // Q tile 1 loaded
  uint64_t* bar_kf = bars + 1;   // [2]
  uint64_t* bar_ke = bars + 3;   // [2]
  uint64_t* bar_vf = bars + 5;   // [2]
  uint64_t* bar_ve = bars + 7;   // [2]
  uint64_t* bar_s = bars + 9;    // [2] per Q tile
  uint64_t* bar_p = bars + 11;   // [2] per Q tile
  uint64_t* bar_o = bars + 13;
  uint64_t* bar_ph = bars + 14;  // [2] first half of P_t (keys 0-63) stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);
  int* n_tiles_slot = reinterpret_cast<int*>(sm + S::kOffCtl + 8);
  uint16_t* tiles = reinterpret_cast<uint16_t*>(sm + S::kOffTiles);
  uint32_t* mbits = reinterpret_cast<uint32_t*>(sm + S::kOffBits);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Unit un = decode_unit(p, blockIdx.x);
  const int hl = un.hl, b = un.b;
  const int q0 = un.q_block * kBlockM;
  const bool two = q0 + kTileM < p.Lq;  // is Q tile 1 inside the sequence?
  const int Lk = p.Lk;

  // ---------------- prologue ----------------
  // The producer thread initialises the barriers and starts the Q0 load at
  // once: Q does not depend on the key mask or the tile list, so its latency
  // overlaps the rest of the prologue.  (Every other thread first touches a
  // barrier after the __syncthreads below.)
  const int qh = p.q_head_off + hl;
  if (warp == 8 && lane == 0) {
    for (int i = 0; i < 17; ++i) mbar_init(bars + i, (i == 11 || i == 12 || i == 14 || i == 15) ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q);
    grid_dep_wait();  // the kernel that wrote q (the RoPE pre-pass) has completed
    mbar_arrive_expect_tx(bar_q, S::kTile);
#pragma unroll
    for (int c = 0; c < S::kChunks; ++c) tma_load_4d(&p.tm_q, bar_q, sQ + c * kChunkBytes, c * 64, q0, qh, b);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_o);
    if (un.ns > 1) tma_prefetch_desc(&p.tm_part);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }

  grid_dep_wait();  // every thread, before its first global access
  // key-mask bits (padded with zero words to a whole tile), one 32-key word
  // per thread: two 16-byte loads when the rows are aligned, else byte loads: word w is one
  // warp's ballot over keys 32w .. 32w + 31, each lane reading one mask byte;
  // a warp loads up to four words before it ballots
  bool use_mask = p.mask != nullptr;
  int local_any = 0;
  if (use_mask) {
    const uint8_t* mrow = p.mask + (int64_t)b * p.mask_sb;
    const int nwords = p.n_kv_tiles * (kTileN / 32);
    for (int w = threadIdx.x; w < nwords; w += kThreads) {
      uint32_t bits = 0;
      const int k0 = w * 32;
      if (p.mask_vec && k0 + 32 <= Lk) {
        // two 16-byte loads, then per byte "nonzero" as one bit
        const uint4 lo = *reinterpret_cast<const uint4*>(mrow + k0);
        const uint4 hi = *reinterpret_cast<const uint4*>(mrow + k0 + 16);
        const uint32_t wd[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t m = __vcmpne4(wd[i], 0u);  // 0xff in each nonzero byte
          bits |= (((m >> 7) & 1u) | ((m >> 14) & 2u) | ((m >> 21) & 4u) | ((m >> 28) & 8u)) << (4 * i);
        }
      } else {
        for (int i = 0; i < 32; ++i) {
          const int key = k0 + i;
          if (key < Lk && mrow[key] != 0) bits |= 1u << i;
        }
      }
      mbits[w] = bits;
      local_any |= (bits != 0);
    }
  }
  const int any_valid = __syncthreads_or(local_any);
  use_mask = use_mask && (any_valid != 0);

  // Causal / sliding rows (GemmaTextEncoder.swift:292-323): row i attends key j
  // when j <= i and i - j < window, and j is valid.  A row left with no such key
  // attends every key instead ("free" row) -- so does every row of a batch whose
  // mask has no valid key.  Softmax thread x (x < 256) owns row q0 + x.
  constexpr bool banded = kBanded;
  const bool batch_empty = p.mask != nullptr && any_valid == 0;
  bool free_row = batch_empty;
  if (banded && !batch_empty && use_mask && threadIdx.x < kBlockM) {
    const int row = q0 + threadIdx.x;
    if (row < p.Lq) {
      const int lo = p.window > 0 ? max(0, row - p.window + 1) : 0;
      const int hi = p.causal ? min(row, Lk - 1) : Lk - 1;
      bool any = false;
      for (int w = hi >> 5; w >= (lo >> 5) && !any; --w) {  // from the diagonal down
        uint32_t bits = mbits[w];
        if (w == (hi >> 5) && (hi & 31) != 31) bits &= (1u << ((hi & 31) + 1)) - 1u;
        if (w == (lo >> 5)) bits &= ~0u << (lo & 31);
        any = bits != 0u;
      }
      free_row = !any;
    }
  }
  bool cta_free = batch_empty;
  if constexpr (banded) cta_free = __syncthreads_or(free_row ? 1 : 0) != 0;

  // the list of KV tiles this CTA needs: every tile when one of its rows is free,
  // else the tiles inside its rows' band that hold a valid key
  if (warp == 0) {
    const int q_last = min(q0 + (two ? kBlockM : kTileM) - 1, p.Lq - 1);
    int count = 0;
    for (int j0 = 0; j0 < p.n_kv_tiles; j0 += 32) {
      const int j = j0 + lane;
      bool act = j < p.n_kv_tiles;
      if (banded && act && !cta_free) {
        if (p.causal) act = j * kTileN <= q_last;
        if (p.window > 0) act = act && j * kTileN + kTileN - 1 >= q0 - p.window + 1;
      }
      if (act && use_mask && !(banded && cta_free)) {
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
  const int t_begin = (int)(((int64_t)un.split * n_all) / un.ns);
  const int t_end = (int)(((int64_t)(un.split + 1) * n_all) / un.ns);
  const int n = t_end - t_begin;
  const int kvh = (p.kv_head_off + hl) / p.group;  // grouped query heads share a kv head

  if (warp >= 8) {
    setmaxnreg_dec<kProducerRegs>();
    if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int k_issued = 0, v_issued = 0;
      bool q1_issued = false;
      // issue order Q0 (already in flight), K0, Q1, V0, ...: S0 needs only the
      // first two, so it can start while the CTA's other first loads arrive
      for (int j = 0; j < n; ++j) {
        const int st = j & 1, u = j >> 1;
        const int kv0 = (int)tiles[t_begin + j] * kTileN;
        if (j >= 2 && !mbar_wait(bar_ke + st, (u - 1) & 1, abort_flag, p.err, 1)) break;
        mbar_arrive_expect_tx(bar_kf + st, S::kTile);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c)
          tma_load_4d(&p.tm_k, bar_kf + st, sK + st * S::kTile + c * kChunkBytes, c * 64, kv0, kvh, b);
        ++k_issued;
        if (j == 0 && two) {
          q1_issued = true;
          mbar_arrive_expect_tx(bar_q1, S::kTile);
#pragma unroll
          for (int c = 0; c < S::kChunks; ++c)
            tma_load_4d(&p.tm_q, bar_q1, sQ + S::kTile + c * kChunkBytes, c * 64, q0 + kTileM, qh, b);
        }
        if (j >= 2 && !mbar_wait(bar_ve + st, (u - 1) & 1, abort_flag, p.err, 2)) break;
        mbar_arrive_expect_tx(bar_vf + st, S::kTile);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c)
          tma_load_4d(&p.tm_v, bar_vf + st, sV + st * S::kTile + c * kChunkBytes, c * 64, kv0, kvh, b);
        ++v_issued;
      }
      // never leave the CTA with a bulk copy still writing its shared memory
      drain_wait(bar_q, 0);
      if (q1_issued) drain_wait(bar_q1, 0);
      for (int i = k_issued < 2 ? 0 : k_issued - 2; i < k_issued; ++i) drain_wait(bar_kf + (i & 1), (i >> 1) & 1);
      for (int i = v_issued < 2 ? 0 : v_issued - 2; i < v_issued; ++i) drain_wait(bar_vf + (i & 1), (i >> 1) & 1);
    }
    __syncwarp();
    } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n > 0) {
      const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
      // base descriptors, built once; stage st adds st * kTile >> 4 to the low word
      const SDesc dQ0 = sdesc_split(smem_u32(sQ), 16, 1024);
      const SDesc dQ1 = sdesc_split(smem_u32(sQ) + S::kTile, 16, 1024);
      const SDesc dK = sdesc_split(smem_u32(sK), 16, 1024);
      const SDesc dV = sdesc_split(smem_u32(sV), kChunkBytes, 1024);
      const uint32_t stage_step = S::kTile >> 4;
      auto kdesc = [&](int st) { return SDesc{dK.lo + st * stage_step, dK.hi}; };
      auto vdesc = [&](int st) { return SDesc{dV.lo + st * stage_step, dV.hi}; };
      bool go = mbar_wait(bar_q, 0, abort_flag, p.err, 3) && mbar_wait(bar_kf, 0, abort_flag, p.err, 4);
      if (go) {
        tc_fence_after();
        issue_s<D>(tS0, dQ0, kdesc(0));
        umma_commit(bar_s + 0);
      }
      if (go && two) {
        go = mbar_wait(bar_q1, 0, abort_flag, p.err, 3);
        if (go) {
          tc_fence_after();
          issue_s<D>(tS1, dQ1, kdesc(0));
          umma_commit(bar_s + 1);
        }
      }
      if (go) {
        umma_commit(bar_ke + 0);
        for (int j = 0; j < n; ++j) {
          const int st = j & 1, u = j >> 1;
          const bool more = j + 1 < n;
          const int st1 = (j + 1) & 1, u1 = (j + 1) >> 1;
          if (!mbar_wait(bar_ph + 0, j & 1, abort_flag, p.err, 5)) break;
          if (!mbar_wait(bar_vf + st, u & 1, abort_flag, p.err, 6)) break;
          tc_fence_after();
          issue_pv_half<D>(tO0, tS0, vdesc(st), j > 0, 0);
          if (!mbar_wait(bar_p + 0, j & 1, abort_flag, p.err, 5)) break;
          tc_fence_after();
          issue_pv_half<D>(tO0, tS0, vdesc(st), true, 1);
          if (more) {
            if (!mbar_wait(bar_kf + st1, u1 & 1, abort_flag, p.err, 7)) break;
            tc_fence_after();
            issue_s<D>(tS0, dQ0, kdesc(st1));
            umma_commit(bar_s + 0);
          }
          if (two) {
            if (!mbar_wait(bar_ph + 1, j & 1, abort_flag, p.err, 8)) break;
            tc_fence_after();
            issue_pv_half<D>(tO1, tS1, vdesc(st), j > 0, 0);
            if (!mbar_wait(bar_p + 1, j & 1, abort_flag, p.err, 8)) break;
            tc_fence_after();
            issue_pv_half<D>(tO1, tS1, vdesc(st), true, 1);
          }
          umma_commit(bar_ve + st);
          if (more) {
            if (two) {
              issue_s<D>(tS1, dQ1, kdesc(st1));
              umma_commit(bar_s + 1);
            }
            umma_commit(bar_ke + st1);
          }
        }
      }
      umma_commit(bar_o);
      drain_wait(bar_o, 0);
    }
    __syncwarp();
    }
  } else {
    setmaxnreg_inc<kSoftmaxRegs>();
    if (warp < 4 || two) {
    // ---------------- softmax / correction / epilogue of Q tile t ----------------
    const int t = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tO = tmem + 256 + t * 128 + lane_off;
    const float sl2 = p.scale_log2;
    const int row = q0 + t * kTileM + (threadIdx.x & 127);
    uint64_t* my_s = bar_s + t;
    uint64_t* my_p = bar_p + t;
    float m = -INFINITY;  // running max, log2 domain (lazy)
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      if (!warp_wait(my_s, i & 1, abort_flag, p.err, 9)) { ok = false; break; }
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
      const bool masked_tile = use_mask || kv0 + kTileN > Lk || banded;
      if (masked_tile) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint32_t bits = 0xffffffffu;
          if (use_mask && !(banded && free_row)) bits = mbits[kv0 / 32 + w];
          const int lim = Lk - (kv0 + 32 * w);
          if (lim < 32) bits &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
          if (banded && !free_row) {  // compiled only into the kBanded instance
            const int kw0 = kv0 + 32 * w;
            if (p.causal) {
              const int cnt = row - kw0 + 1;  // keys kw0 .. row
              bits &= cnt >= 32 ? ~0u : (cnt <= 0 ? 0u : ((1u << cnt) - 1u));
            }
            if (p.window > 0) {
              const int skip = row - p.window + 1 - kw0;  // keys below row - window + 1
              bits &= skip <= 0 ? ~0u : (skip >= 32 ? 0u : (~0u << skip));
            }
          }
          if (bits != 0xffffffffu) {  // a word whose keys are all valid needs no per-column select
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (!((bits >> c) & 1u)) s[32 * w + c] = -INFINITY;
          }
        }
      }
      // row max: eight independent 3-input-max chains, then a short tree
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
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      const float2 sl2x2 = make_float2(sl2, sl2), nmx2 = make_float2(neg_m, neg_m);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
        for (int c = 64 * h2; c < 64 * h2 + 64; c += 2) {
          const float2 x = fma2(make_float2(s[c], s[c + 1]), sl2x2, nmx2);
          float2 e;
          if (((c >> 1) & 7) < kPolyCols / 16) {
            e = exp2_poly2(x);
            if (masked_tile) {  // the polynomial leaves <= 2^-126 for -inf; masked weights are exactly 0
              e.x = (s[c] == -INFINITY) ? 0.f : e.x;
              e.y = (s[c + 1] == -INFINITY) ? 0.f : e.y;
            }
          } else {
            e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          }
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
        mbar_arrive(h2 == 0 ? bar_ph + t : my_p);
      }
      {
        const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const float2 tot = add2(a01, a23);
        l += tot.x + tot.y;
      }
    }

    // epilogue
    const Unit ue = decode_unit(p, ctaid_x_fresh());
    // the output gate of this row and head (its load overlaps the wait for O)
    uint32_t g2 = 0x3f803f80u;  // bf16x2 (1, 1)
    if (p.gate != nullptr && ue.ns == 1 && row < p.Lq) {
      const float g = gate_bf16(__bfloat162float(
          p.gate[(int64_t)ue.b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + ue.hl) * p.g_sh]));
      g2 = pack_bf16x2(g, g);
    }
    const bool have_o = ok && n > 0 && warp_wait(bar_o, 0, abort_flag, p.err, 10);
    tc_fence_after();
    const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
    if (ue.ns == 1) {
      // Stage the normalised bf16 row in K stage t (idle once O is complete: every
      // MMA has finished and no load is outstanding), 128-byte swizzled like the
      // loads, then one thread per tile stores it with TMA (coalesced; rows past
      // Lq are clipped by the tensor map).
      uint8_t* stg = sK + t * S::kTile;
      const int r = threadIdx.x & 127;
      uint8_t* srow = stg + r * 128;
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
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(o[8 * e + 0]) * inv_l, __uint_as_float(o[8 * e + 1]) * inv_l);
          v.y = pack_bf16x2(__uint_as_float(o[8 * e + 2]) * inv_l, __uint_as_float(o[8 * e + 3]) * inv_l);
          v.z = pack_bf16x2(__uint_as_float(o[8 * e + 4]) * inv_l, __uint_as_float(o[8 * e + 5]) * inv_l);
          v.w = pack_bf16x2(__uint_as_float(o[8 * e + 6]) * inv_l, __uint_as_float(o[8 * e + 7]) * inv_l);
          if (p.gate != nullptr) {  // T(T(O) * g): one bf16x2 multiply (the product is exact in fp32)
            v.x = bmul2(v.x, g2);
            v.y = bmul2(v.y, g2);
            v.z = bmul2(v.z, g2);
            v.w = bmul2(v.w, g2);
          }
          const int j = (c & 1) * 4 + e;  // 16-byte unit within the 64-column chunk c / 2
          *reinterpret_cast<uint4*>(srow + (c >> 1) * kChunkBytes + ((j ^ (r & 7)) << 4)) = v;
        }
      }
      if (p.lse != nullptr && row < p.Lq) {
        p.lse[(int64_t)ue.b * p.lse_sb + (int64_t)(p.head_begin + ue.hl) * p.lse_sh + row] =
            (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
      }
      fence_proxy_async_smem();  // the bulk copy reads these rows through the async proxy
      named_barrier(1 + t, 128);
      if (r == 0) {
#pragma unroll
        for (int ch = 0; ch < S::kChunks; ++ch)
          tma_store_4d(&p.tm_o, stg + ch * kChunkBytes, ch * 64, ue.q_block * kBlockM + t * kTileM,
                       p.head_begin + ue.hl, ue.b);
        // fused all-gather: the same tile into every other rank's output (the
        // copies read shared memory and leave; the transfer over NVLink overlaps
        // whatever runs next on this SM)
        for (int i = 0; i < p.peer_n; ++i)
#pragma unroll
          for (int ch = 0; ch < S::kChunks; ++ch)
            tma_store_4d(&p.tm_peer[i], stg + ch * kChunkBytes, ch * 64, ue.q_block * kBlockM + t * kTileM,
                         p.head_begin + ue.hl, ue.b);
        bulk_commit();
      }
      if (r == 0) bulk_wait_read();  // the CTA's shared memory must outlive the copy's reads
    } else {
      // fp32 partial of this split: staged like the bf16 output (128 rows x D fp32
      // = two K/V tiles' worth, so tile t uses 2 * kTile bytes from sK + 2t * kTile),
      // in 32-column chunks of 128-byte rows, and stored with TMA by one thread
      // into the [split][tail unit][256 rows] partial layout
      const int64_t prow = ((int64_t)ue.split * p.n_tail + ue.tail) * kBlockM + t * kTileM + (threadIdx.x & 127);
      uint8_t* stg = sK + t * 2 * S::kTile;
      const int r = threadIdx.x & 127;
      uint8_t* srow = stg + r * 128;
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
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(srow + c * (128 * 128) + ((j ^ (r & 7)) << 4)) =
              make_float4(__uint_as_float(o[4 * j]) * inv_l, __uint_as_float(o[4 * j + 1]) * inv_l,
                          __uint_as_float(o[4 * j + 2]) * inv_l, __uint_as_float(o[4 * j + 3]) * inv_l);
      }
      if (row < p.Lq) p.part_lse[prow] = (have_o && l > 0.f) ? m + log2f(l) : -INFINITY;
      fence_proxy_async_smem();
      named_barrier(1 + t, 128);
      if (r == 0) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tma_store_4d(&p.tm_part, stg + c * (128 * 128), c * 32, t * kTileM, ue.tail, ue.split);
        bulk_commit();
        bulk_wait_read();
      }
    }
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

// Entry handshake of the fused all-gather: tell every peer that this rank has
// entered call `epoch` (its earlier work on its own output is complete: this
// kernel follows it in stream order), then wait until every peer has entered
// it too, so no peer store lands in an output that its rank still reads.
// Bounded: on timeout the error word records site 60 and the kernel returns.
__global__ void gather_enter_kernel(const GatherSync g) {
  const int d = threadIdx.x;
  const bool peer = d < g.n && d != g.rank;
  if (peer) {
    __threadfence_system();
    atomicMax_system(g.sig[d] + 8 + g.rank, g.epoch);
  }
  if (peer) {
    volatile unsigned int* f = g.sig[g.rank] + 8 + d;
    const uint64_t t0 = globaltimer_ns();
    while (*f < g.epoch) {
      if (globaltimer_ns() - t0 > LTX_WAIT_LIMIT_NS) {
        atomicCAS(g.err, 0, (60 << 8) | kErrTimeout);
        break;
      }
    }
  }
  __threadfence_system();
}

// Completion of the fused all-gather, after the attention kernel: every store of
// that kernel (its tiles in the other ranks' outputs included) has been performed
// when this kernel starts, so tell every peer that this rank's tiles of `epoch`
// have landed, then wait until every peer has said the same here.  Bounded
// (site 61).
__global__ void gather_done_kernel(const GatherSync g) {
  const int d = threadIdx.x;
  const bool peer = d < g.n && d != g.rank;
  if (peer) {
    __threadfence_system();
    atomicMax_system(g.sig[d] + g.word + g.rank, g.epoch);
  }
  if (peer) {
    volatile unsigned int* f = g.sig[g.rank] + g.word + d;
    const uint64_t t0 = globaltimer_ns();
    while (*f < g.epoch) {
      if (globaltimer_ns() - t0 > LTX_WAIT_LIMIT_NS) {
        atomicCAS(g.err, 0, (61 << 8) | kErrTimeout);
        break;
      }
    }
  }
  __threadfence_system();
}

// Merge split partials: lse = log2-sum-exp2 of the splits' lse, O = sum_s w_s O_s.
// One warp per row of the split units (partial row gw = tail unit * 256 + r).
template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.n_tail * kBlockM;
  if (gw >= rows) return;
  const int unit = p.n_full + (int)(gw / kBlockM);
  const int row = (unit % p.q_blocks) * kBlockM + (int)(gw % kBlockM);
  const int hl = (unit / p.q_blocks) % p.Hc;
  const int b = unit / (p.q_blocks * p.Hc);
  if (row >= p.Lq) return;
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
  const int64_t ooff = (int64_t)b * p.o_sb + (int64_t)(p.head_begin + hl) * p.o_sh + (int64_t)row * p.o_st;
  __nv_bfloat16 ov[kPer];
  if (p.gate != nullptr) {  // T(T(O) * g)
    const float g = gate_bf16(
        __bfloat162float(p.gate[(int64_t)b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + hl) * p.g_sh]));
#pragma unroll
    for (int e = 0; e < kPer; ++e) ov[e] = __float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(acc[e] * inv)) * g);
  } else {
#pragma unroll
    for (int e = 0; e < kPer; ++e) ov[e] = __float2bfloat16_rn(acc[e] * inv);
  }
#pragma unroll
  for (int e = 0; e < kPer; ++e) p.out[ooff + lane + 32 * e] = ov[e];
  for (int i = 0; i < p.peer_n; ++i)  // fused all-gather: the row in every other rank's output
#pragma unroll
    for (int e = 0; e < kPer; ++e) p.peer_out[i][ooff + lane + 32 * e] = ov[e];
  if (p.lse != nullptr && lane == 0)
    p.lse[(int64_t)b * p.lse_sb + (int64_t)(p.head_begin + hl) * p.lse_sh + row] =
        (wsum > 0.f) ? (mx + log2f(wsum)) * kLn2 : -INFINITY;
}

}  // namespace

size_t fwd_bf16_smem_bytes(int D, int Lk, bool has_mask) {
  const int n_tiles = (Lk + kTileN - 1) / kTileN;
  const size_t fixed = (D == 128) ? Smem<128>::kOffBits : Smem<64>::kOffBits;
  return 1024 /* alignment slack */ + fixed + (has_mask ? (size_t)n_tiles * 16 : 0);
}

// The warpgroup register split is sized for kLaunchRegs per thread; refuse to
// launch a build whose kernel was allotted a different count (a setmaxnreg.inc
// beyond the launch allocation would never return).
template <typename K>
cudaError_t check_launch_regs(K kernel) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return e;
  return fa.numRegs == (int)kLaunchRegs ? cudaSuccess : cudaErrorInvalidConfiguration;
}

// Per-device, per-head-dim launch preparation, done once (the register check)
// or when a larger shared-memory size is first needed; calls on the hot path
// then cost a cached comparison.
namespace {
constexpr int kMaxDev = 64;
std::mutex g_prep_mu;
size_t g_smem_set[kMaxDev][2] = {};
bool g_regs_ok[kMaxDev][2] = {};
}  // namespace

cudaError_t prepare_fwd_bf16(int D, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int di = D == 128 ? 1 : 0;
  std::lock_guard<std::mutex> lock(g_prep_mu);
  if (!g_regs_ok[dev][di]) {
    e = D == 128 ? check_launch_regs(fwd_bf16_sm100_kernel<128, false>)
                 : check_launch_regs(fwd_bf16_sm100_kernel<64, false>);
    if (e == cudaSuccess)
      e = D == 128 ? check_launch_regs(fwd_bf16_sm100_kernel<128, true>)
                   : check_launch_regs(fwd_bf16_sm100_kernel<64, true>);
    if (e != cudaSuccess) return e;
    g_regs_ok[dev][di] = true;
  }
  if (smem > g_smem_set[dev][di]) {
    for (int banded = 0; banded < 2 && e == cudaSuccess; ++banded) {
      const void* k = D == 128 ? (banded ? (const void*)fwd_bf16_sm100_kernel<128, true> : (const void*)fwd_bf16_sm100_kernel<128, false>)
                               : (banded ? (const void*)fwd_bf16_sm100_kernel<64, true> : (const void*)fwd_bf16_sm100_kernel<64, false>);
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    if (e != cudaSuccess) return e;
    g_smem_set[dev][di] = smem;
  }
  return cudaSuccess;
}

// Launch only (prepare_fwd_bf16 must have succeeded for D and at least smem).
cudaError_t launch_fwd_bf16(const FwdParams& p, int D, size_t smem, cudaStream_t s) {
  const dim3 grid(p.n_full + p.n_tail * p.num_splits);
  const bool banded = p.causal || p.window > 0;
  // programmatic launch: CTAs set up barriers and TMEM while the kernel
  // before (the RoPE pre-pass, a q/k preparation) finishes
  if (D == 128 && banded) return launch_pdl(fwd_bf16_sm100_kernel<128, true>, grid, dim3(kThreads), smem, s, p);
  if (D == 128) return launch_pdl(fwd_bf16_sm100_kernel<128, false>, grid, dim3(kThreads), smem, s, p);
  if (banded) return launch_pdl(fwd_bf16_sm100_kernel<64, true>, grid, dim3(kThreads), smem, s, p);
  return launch_pdl(fwd_bf16_sm100_kernel<64, false>, grid, dim3(kThreads), smem, s, p);
}

cudaError_t launch_gather_enter(const GatherSync& g, cudaStream_t s) {
  gather_enter_kernel<<<1, 32, 0, s>>>(g);
  return cudaGetLastError();
}

cudaError_t launch_gather_done(const GatherSync& g, cudaStream_t s) {
  gather_done_kernel<<<1, 32, 0, s>>>(g);
  return cudaGetLastError();
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t s) {
  const int64_t rows = (int64_t)p.n_tail * kFwdBlockM;
  const int64_t threads = rows * 32;
  const int blocks = (int)((threads + 255) / 256);
  if (p.D == 128)
    combine_kernel<128><<<blocks, 256, 0, s>>>(p);
  else
    combine_kernel<64><<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ltx
