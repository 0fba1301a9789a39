// fwd_persist_sm100.cu -- the bf16 forward run persistently: one CTA per SM
// walks several work units (256-row query block, head, batch) and overlaps
// the end of one unit with the start of the next.
//
// The one-CTA-per-unit forward (fwd_sm100.cu) pays, per unit, a CTA launch,
// barrier and TMEM setup, the first Q/K/V loads with nothing to overlap
// them, and an epilogue during which the tensor pipe idles: about 8 us per
// unit at the 3,120-token video shape, whose 416 units also run as three
// waves of 148 for 2.81 waves of work.  Here CTA c runs units c, c + G,
// c + 2G, ... (G = the grid, at most one CTA per SM) and the roles never
// drain between units:
//   - the producer loads the next unit's Q tile t as soon as the last
//     S_t = Q_t K^T of the current unit has completed (q_free), and the K/V
//     ring runs on across unit boundaries;
//   - the MMA thread issues across the boundary in the steady-state order,
//     PV0 of the last tile, S0 of the next unit's first tile, PV1, S1, so
//     each softmax warpgroup finds its next S ready after its epilogue;
//   - the softmax warpgroup of tile t reads O_t from TMEM into registers and
//     releases the O_t columns (o_free), which is all the next unit's first
//     P V waits for; it then stores the normalised rows with TMA through a
//     16 KB staging tile of its own, one 64-column chunk at a time (the rest
//     of shared memory holds the next unit's Q/K/V).  Full-line TMA stores
//     matter here: per-row 16-byte stores write partial sectors, and at the
//     3,120-token shape they made the kernel 6% slower than the one-CTA-per-
//     unit kernel, whose epilogue stages in an idle K stage.
// Calls with a causal or window band do not come here: a unit's KV tiles depend
// only on its batch row.  With a key mask the prologue reads every batch row's
// mask once into shared memory (one bit per key) and lists the tiles holding a
// valid key; a unit then walks its batch row's list (the text cross-attention's
// 1024 slots with 94 valid keys: one tile), masking keys per column, and a row
// with no valid key attends every key (GemmaTextEncoder.swift:306-319).  The
// arithmetic of a unit is the one-CTA-per-unit kernel's (the same tiles, masks,
// exponentials, lazy rescale, P rounding, row-sum order and normalisation), so
// both give the same bits.
//
// Thread layout, register split and TMEM map are the forward kernel's:
// warps 0-3 softmax of Q tile 0, warps 4-7 of Q tile 1, warp 8 TMA producer
// (lane 0), warp 9 TMEM owner and MMA issuer (lane 0), warps 10-11 idle;
// TMEM S0 [0,128), S1 [128,256), O0 [256,256+D), O1 [384,384+D).  A unit of
// the ragged last query block with no rows in Q tile 1 runs tile 0 alone.
//
// Barrier phases are counted per role: the producer and MMA thread count K/V
// tiles (ring stage g & 1, use g >> 1) and per-tile Q loads; the softmax
// warpgroup of tile t counts the S_t tiles and the units it has processed.
// Every wait is bounded (2 s) and a timeout stops every role.
#include <mutex>
#include <type_traits>

#include "fwd_common.cuh"

namespace ltx {

namespace {

template <int D>
struct PSmem {
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunkBytes;
  static constexpr uint32_t kOffQ = 0, kOffK = 2 * kTile, kOffV = 4 * kTile;
  static constexpr uint32_t kOffStg = 6 * kTile;  // [2] epilogue staging, one 64-column chunk per tile
  // q_full[2], q_free[2], k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2],
  // p_half[2], p_full[2], o_full[2], o_free[2], done
  static constexpr int kBars = 23;
  static constexpr uint32_t kOffBar = kOffStg + 2 * kChunkBytes;
  static constexpr uint32_t kOffCtl = kOffBar + kBars * 8;  // tmem slot, abort flag
  static constexpr uint32_t kOffMeta = kOffCtl + 16;        // key-mask tables (masked calls only)
  static constexpr uint32_t kBytes = kOffMeta;
};

// Key-mask tables after kOffMeta, for B batch rows of nt KV tiles: the live tile
// count and the "mask applies" flag per row (int [B] each), the live tiles
// (uint16 [B][nt]) and the mask bits (uint32 [B][4 nt], bit i of word w = key
// 32 w + i valid).
__host__ __device__ constexpr uint32_t align16u(uint32_t x) { return (x + 15u) & ~15u; }
__host__ __device__ constexpr uint32_t meta_off_tiles(int B) { return align16u(8u * (uint32_t)B); }
__host__ __device__ constexpr uint32_t meta_off_bits(int B, int nt) {
  return meta_off_tiles(B) + align16u(2u * (uint32_t)B * (uint32_t)nt);
}
__host__ __device__ constexpr uint32_t meta_bytes(int B, int nt) { return meta_off_bits(B, nt) + 16u * B * nt; }

struct PUnit {
  int q0, hl, b;
  bool two;   // Q tile 1 holds rows of the sequence
  int n;      // KV tiles the unit walks
  bool mask;  // per-key mask bits apply
};

// The key-mask tables of the prologue (meta == null when the call has no mask).
struct MaskTables {
  const uint8_t* meta;
  int B, nt;
  __device__ __forceinline__ int tile(int b, int j) const {
    return meta == nullptr ? j : reinterpret_cast<const uint16_t*>(meta + meta_off_tiles(B))[b * nt + j];
  }
  __device__ __forceinline__ uint32_t word(int b, int w) const {
    return reinterpret_cast<const uint32_t*>(meta + meta_off_bits(B, nt))[b * 4 * nt + w];
  }
};

// A copy of x the compiler cannot see through, so values derived from it are
// recomputed instead of kept live in registers.
__device__ __forceinline__ int fresh_int(int x) {
  int y;
  asm volatile("mov.b32 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ PUnit persist_unit(const FwdParams& p, const MaskTables& mt, int unit) {
  PUnit u;
  u.q0 = (unit % p.q_blocks) * kBlockM;
  u.hl = (unit / p.q_blocks) % p.Hc;
  u.b = unit / (p.q_blocks * p.Hc);
  u.two = u.q0 + kTileM < p.Lq;
  u.n = mt.meta == nullptr ? p.n_kv_tiles : reinterpret_cast<const int*>(mt.meta)[u.b];
  u.mask = mt.meta != nullptr && reinterpret_cast<const int*>(mt.meta)[mt.B + u.b] != 0;
  return u;
}

// kMasked: the call has a key mask (the prologue builds the per-row tables); the
// unmasked instance carries none of that state through its loops.
template <int D, bool kMasked>
__global__ void __launch_bounds__(kThreads, 1) fwd_persist_sm100_kernel(const __grid_constant__ FwdParams p) {
  using S = PSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm + S::kOffQ;  // Q tile t at sQ + t * kTile
  uint8_t* sK = sm + S::kOffK;  // K stage st at sK + st * kTile
  uint8_t* sV = sm + S::kOffV;
  uint8_t* sStg = sm + S::kOffStg;  // staging tile t at sStg + t * kChunkBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* bar_qf = bars + 0;   // [2] Q tile t loaded
  uint64_t* bar_qe = bars + 2;   // [2] the unit's last S_t has read Q tile t
  uint64_t* bar_kf = bars + 4;   // [2]
  uint64_t* bar_ke = bars + 6;   // [2]
  uint64_t* bar_vf = bars + 8;   // [2]
  uint64_t* bar_ve = bars + 10;  // [2]
  uint64_t* bar_s = bars + 12;   // [2] S_t in TMEM
  uint64_t* bar_ph = bars + 14;  // [2] first half of P_t stored (128 arrivals)
  uint64_t* bar_p = bars + 16;   // [2] all of P_t stored (128 arrivals)
  uint64_t* bar_of = bars + 18;  // [2] O_t of a unit complete
  uint64_t* bar_oe = bars + 20;  // [2] O_t read by the epilogue (128 arrivals)
  uint64_t* bar_done = bars + 22;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kOffCtl + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int units = p.n_full;
  const int nt = p.n_kv_tiles;
  const MaskTables mt{kMasked ? sm + S::kOffMeta : nullptr, units / (p.q_blocks * p.Hc), nt};

  if (warp == 8 && lane == 0) {
    for (int i = 0; i < S::kBars; ++i) mbar_init(bars + i, (i >= 14 && i < 18) || i == 20 || i == 21 ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q);
    // the first unit's Q does not depend on the key mask: its load overlaps
    // the rest of the prologue (TMEM allocation, the mask tables)
    if ((int)blockIdx.x < units) {
      grid_dep_wait();  // the kernel that wrote q (the RoPE pre-pass) has completed
      const PUnit u0 = persist_unit(p, MaskTables{nullptr, 0, nt}, blockIdx.x);
      for (int t = 0; t < (u0.two ? 2 : 1); ++t) {
        mbar_arrive_expect_tx(bar_qf + t, S::kTile);
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c)
          tma_load_4d(&p.tm_q, bar_qf + t, sQ + t * S::kTile + c * kChunkBytes, c * 64, u0.q0 + t * kTileM,
                      p.q_head_off + u0.hl, u0.b);
      }
    }
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
  grid_dep_wait();  // the kernel that wrote q / k (the RoPE pre-pass) has completed

  if (kMasked) {
    // every batch row's mask bits (one 32-key word per thread per pass: two
    // 16-byte loads when the rows are aligned, else byte loads; keys past Lk
    // read as masked), then one warp per row lists the tiles holding a valid key
    const int B = units / (p.q_blocks * p.Hc);
    uint8_t* meta = sm + S::kOffMeta;
    int* count = reinterpret_cast<int*>(meta);
    int* on = count + B;
    uint16_t* tiles = reinterpret_cast<uint16_t*>(meta + meta_off_tiles(B));
    uint32_t* bits = reinterpret_cast<uint32_t*>(meta + meta_off_bits(B, nt));
    const int nwords = 4 * nt;
    const int Lk = p.Lk;
    for (int idx = threadIdx.x; idx < B * nwords; idx += kThreads) {
      const int b = idx / nwords, k0 = (idx - b * nwords) * 32;
      const uint8_t* mrow = p.mask + (int64_t)b * p.mask_sb;
      uint32_t w = 0;
      if (p.mask_vec && k0 + 32 <= Lk) {
        const uint4 lo = *reinterpret_cast<const uint4*>(mrow + k0);
        const uint4 hi = *reinterpret_cast<const uint4*>(mrow + k0 + 16);
        const uint32_t wd[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t m = __vcmpne4(wd[i], 0u);  // 0xff in each nonzero byte
          w |= (((m >> 7) & 1u) | ((m >> 14) & 2u) | ((m >> 21) & 4u) | ((m >> 28) & 8u)) << (4 * i);
        }
      } else {
        for (int i = 0; i < 32; ++i)
          if (k0 + i < Lk && mrow[k0 + i] != 0) w |= 1u << i;
      }
      bits[idx] = w;
    }
    __syncthreads();
    for (int b = warp; b < B; b += kThreads / 32) {
      const uint32_t* wb = bits + b * nwords;
      int cnt = 0;
      for (int j0 = 0; j0 < nt; j0 += 32) {
        const int j = j0 + lane;
        const bool act = j < nt && (wb[4 * j] | wb[4 * j + 1] | wb[4 * j + 2] | wb[4 * j + 3]) != 0u;
        const unsigned bal = __ballot_sync(0xffffffffu, act);
        if (act) tiles[b * nt + cnt + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
        cnt += __popc(bal);
      }
      const bool free_row = cnt == 0;  // no valid key: every key, unmasked
      if (free_row) {
        for (int j = lane; j < nt; j += 32) tiles[b * nt + j] = static_cast<uint16_t>(j);
        cnt = nt;
      }
      if (lane == 0) {
        count[b] = cnt;
        on[b] = free_row ? 0 : 1;
      }
    }
    __syncthreads();
  }

  if (warp >= 8) {
    setmaxnreg_dec<kProducerRegs>();
    if (warp == 8) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        int nq0 = 0, nq1 = 0;  // loads issued into Q tile 0 / 1
        int gk = 0, gv = 0;    // K and V tiles issued (ring stage i & 1, use i >> 1)
        bool ok = true;
        // Q tile t of a unit; the previous unit's last S_t must have read the buffer
        auto load_q = [&](auto tc, const PUnit& u, int qh) -> bool {
          constexpr int t = decltype(tc)::value;
          int& nq = t == 0 ? nq0 : nq1;
          if (nq > 0 && !mbar_wait(bar_qe + t, (nq - 1) & 1, abort_flag, p.err, 40)) return false;
          mbar_arrive_expect_tx(bar_qf + t, S::kTile);
#pragma unroll
          for (int c = 0; c < S::kChunks; ++c)
            tma_load_4d(&p.tm_q, bar_qf + t, sQ + t * S::kTile + c * kChunkBytes, c * 64, u.q0 + t * kTileM, qh, u.b);
          ++nq;
          return true;
        };
        for (int unit = blockIdx.x; unit < units && ok; unit += G) {
          const PUnit u = persist_unit(p, mt, unit);
          const int qh = p.q_head_off + u.hl;
          const int kvh = (p.kv_head_off + u.hl) / p.group;
          if (unit == (int)blockIdx.x) {  // loaded in the prologue
            nq0 = 1;
            nq1 = u.two ? 1 : 0;
          } else {
            ok = load_q(std::integral_constant<int, 0>{}, u, qh) &&
                 (!u.two || load_q(std::integral_constant<int, 1>{}, u, qh));
          }
          for (int j = 0; j < u.n && ok; ++j) {
            const int kv0 = mt.tile(u.b, j) * kTileN;
            int st = gk & 1;
            if (gk >= 2 && !(ok = mbar_wait(bar_ke + st, ((gk >> 1) - 1) & 1, abort_flag, p.err, 41))) break;
            mbar_arrive_expect_tx(bar_kf + st, S::kTile);
#pragma unroll
            for (int c = 0; c < S::kChunks; ++c)
              tma_load_4d(&p.tm_k, bar_kf + st, sK + st * S::kTile + c * kChunkBytes, c * 64, kv0, kvh, u.b);
            ++gk;
            st = gv & 1;
            if (gv >= 2 && !(ok = mbar_wait(bar_ve + st, ((gv >> 1) - 1) & 1, abort_flag, p.err, 42))) break;
            mbar_arrive_expect_tx(bar_vf + st, S::kTile);
#pragma unroll
            for (int c = 0; c < S::kChunks; ++c)
              tma_load_4d(&p.tm_v, bar_vf + st, sV + st * S::kTile + c * kChunkBytes, c * 64, kv0, kvh, u.b);
            ++gv;
          }
        }
        // never leave the CTA with a bulk copy still writing its shared memory:
        // a load into a buffer is issued only after the one before it into that
        // buffer was consumed, so only the last load per Q tile and the last
        // two per ring can still be in flight
        if (nq0 > 0) drain_wait(bar_qf + 0, (nq0 - 1) & 1);
        if (nq1 > 0) drain_wait(bar_qf + 1, (nq1 - 1) & 1);
        for (int i = gk < 2 ? 0 : gk - 2; i < gk; ++i) drain_wait(bar_kf + (i & 1), (i >> 1) & 1);
        for (int i = gv < 2 ? 0 : gv - 2; i < gv; ++i) drain_wait(bar_vf + (i & 1), (i >> 1) & 1);
      }
      __syncwarp();
    } else if (warp == 9) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        // per-tile work as generic lambdas over a compile-time tile index, so
        // no per-tile state lives in an indexed (local-memory) array
        using T0 = std::integral_constant<int, 0>;
        using T1 = std::integral_constant<int, 1>;
        const SDesc dQ0 = sdesc_split(smem_u32(sQ), 16, 1024);
        const SDesc dQ1 = sdesc_split(smem_u32(sQ) + S::kTile, 16, 1024);
        const SDesc dK = sdesc_split(smem_u32(sK), 16, 1024);
        const SDesc dV = sdesc_split(smem_u32(sV), kChunkBytes, 1024);
        const uint32_t stage_step = S::kTile >> 4;
        int nq0 = 0, nq1 = 0;  // units begun on Q tile t (q_full phase count)
        int np0 = 0, np1 = 0;  // P_t tiles consumed (p_half / p_full phase count)
        // S_t of (unit, tile j) whose K sits in ring slot g; j == 0 first waits
        // for the unit's Q tile t, j == n - 1 (n: the unit's tile count) then
        // releases Q tile t
        auto issue_s_step = [&](auto tc, int j, int n, int g) -> bool {
          constexpr int t = decltype(tc)::value;
          int& nq = t == 0 ? nq0 : nq1;
          if (j == 0) {
            if (!mbar_wait(bar_qf + t, nq & 1, abort_flag, p.err, 43)) return false;
            ++nq;
          }
          tc_fence_after();
          issue_s<D>(tmem + 128 * t, t == 0 ? dQ0 : dQ1, SDesc{dK.lo + (g & 1) * stage_step, dK.hi});
          umma_commit(bar_s + t);
          if (j == n - 1) umma_commit(bar_qe + t);
          return true;
        };
        // P V_t of (unit, tile j) with V in ring stage st; the first P V of a
        // unit overwrites O_t, so it waits for the previous unit's epilogue on
        // this tile to have read O_t
        auto pv_step = [&](auto tc, int j, int n, int st) -> bool {
          constexpr int t = decltype(tc)::value;
          int& np = t == 0 ? np0 : np1;
          const int nq = t == 0 ? nq0 : nq1;
          const SDesc vd{dV.lo + st * stage_step, dV.hi};
          if (!mbar_wait(bar_ph + t, np & 1, abort_flag, p.err, 45)) return false;
          if (j == 0 && nq > 1 && !mbar_wait(bar_oe + t, (nq - 2) & 1, abort_flag, p.err, 47)) return false;
          tc_fence_after();
          issue_pv_half<D>(tmem + 256 + 128 * t, tmem + 128 * t, vd, j > 0, 0);
          if (!mbar_wait(bar_p + t, np & 1, abort_flag, p.err, 45)) return false;
          tc_fence_after();
          issue_pv_half<D>(tmem + 256 + 128 * t, tmem + 128 * t, vd, true, 1);
          ++np;
          if (j == n - 1) umma_commit(bar_of + t);
          return true;
        };
        bool go = true;
        int unit = blockIdx.x;
        PUnit u = persist_unit(p, mt, unit);
        int g = 0;  // ring slot of the current tile
        if (unit < units) {
          go = mbar_wait(bar_kf, 0, abort_flag, p.err, 44) && issue_s_step(T0{}, 0, u.n, 0);
          if (go && u.two) go = issue_s_step(T1{}, 0, u.n, 0);
          if (go) umma_commit(bar_ke + 0);
        }
        for (; unit < units && go; unit += G) {
          const int nxt_unit = unit + G;
          const bool has_next = nxt_unit < units;
          const PUnit v = has_next ? persist_unit(p, mt, nxt_unit) : u;
          const int n = u.n;
          for (int j = 0; j < n; ++j, ++g) {
            const int st = g & 1;
            // the step after this one: (unit, j + 1) or (next unit, 0); S_t of
            // it right behind P V_t of this one (a unit with no rows in Q tile
            // 1 issues neither P V1 nor S1)
            const bool more = j + 1 < n || has_next;
            const bool nx_two = j + 1 < n ? u.two : v.two;
            const int nj = j + 1 < n ? j + 1 : 0;
            const int nn = j + 1 < n ? n : v.n;
            const int g1 = g + 1, st1 = g1 & 1;
            go = mbar_wait(bar_vf + st, (g >> 1) & 1, abort_flag, p.err, 46) && pv_step(T0{}, j, n, st);
            if (go && more)
              go = mbar_wait(bar_kf + st1, (g1 >> 1) & 1, abort_flag, p.err, 48) && issue_s_step(T0{}, nj, nn, g1);
            if (go && u.two) go = pv_step(T1{}, j, n, st);
            if (go && more && nx_two) go = issue_s_step(T1{}, nj, nn, g1);
            if (!go) break;
            umma_commit(bar_ve + st);
            if (more) umma_commit(bar_ke + st1);
          }
          u = v;
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
    int ns = 0;     // S_t tiles consumed
    int nunit = 0;  // units processed on this tile
    bool ok = true;
    for (int unit = blockIdx.x; unit < units && ok; unit += G) {
      // only the tile count, the mask flag and the batch row stay live through
      // the tile loop; the epilogue decodes the unit again
      int n, ub;
      bool umask;
      {
        const PUnit u = persist_unit(p, mt, unit);
        if (t == 1 && !u.two) continue;
        n = u.n;
        ub = u.b;
        umask = kMasked && u.mask;
      }
      float m = -INFINITY;  // running max, log2 domain (lazy)
      float l = 0.f;
      for (int i = 0; i < n; ++i, ++ns) {
        if (!(ok = warp_wait(bar_s + t, ns & 1, abort_flag, p.err, 49))) break;
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
        // masked keys and keys past Lk get -inf logits
        const int kv0 = (kMasked ? mt.tile(ub, i) : i) * kTileN;
        const bool masked_tile = umask || kv0 + kTileN > Lk;
        if (masked_tile) {
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t bits = umask ? mt.word(ub, kv0 / 32 + w) : 0xffffffffu;
            const int lim = Lk - (kv0 + 32 * w);
            if (lim < 32) bits &= (lim <= 0) ? 0u : ((1u << lim) - 1u);
            if (bits != 0xffffffffu) {  // a word whose keys are all valid needs no per-column select
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (!((bits >> c) & 1u)) s[32 * w + c] = -INFINITY;
            }
          }
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
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
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
        {
          const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
          const float2 tot = add2(a01, a23);
          l += tot.x + tot.y;
        }
      }
      if (!ok) break;

      // ---- epilogue: O_t / l, gated, stored with TMA ----
      const PUnit u = persist_unit(p, mt, fresh_int(unit));
      const int row = u.q0 + t * kTileM + r;
      uint32_t g2 = 0x3f803f80u;  // bf16x2 (1, 1)
      if (p.gate != nullptr && row < p.Lq) {
        const float gv = gate_bf16(__bfloat162float(
            p.gate[(int64_t)u.b * p.g_sb + (int64_t)row * p.g_st + (int64_t)(p.head_begin + u.hl) * p.g_sh]));
        g2 = pack_bf16x2(gv, gv);
      }
      if (!(ok = warp_wait(bar_of + t, nunit & 1, abort_flag, p.err, 50))) break;
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      uint4 packed[D / 8];
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
          if (p.gate != nullptr) {  // T(T(O) * g): one bf16x2 multiply (the product is exact in fp32)
            v.x = bmul2(v.x, g2);
            v.y = bmul2(v.y, g2);
            v.z = bmul2(v.z, g2);
            v.w = bmul2(v.w, g2);
          }
          packed[c * 4 + e] = v;
        }
      }
      // O_t is in registers: the next unit's first P V may overwrite it
      tc_fence_before();
      mbar_arrive(bar_oe + t);
      ++nunit;
      // one 64-column chunk at a time through this tile's staging tile (128-byte
      // swizzled like the loads), stored by one thread with TMA; rows past Lq
      // are clipped by the tensor map
      uint8_t* srow = sStg + t * kChunkBytes + r * 128;
#pragma unroll
      for (int ch = 0; ch < S::kChunks; ++ch) {
        if (r == 0) bulk_wait_read();  // the previous store has read the staging tile
        named_barrier(1 + t, 128);
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(srow + ((j ^ (r & 7)) << 4)) = packed[ch * 8 + j];
        fence_proxy_async_smem();  // the bulk copy reads these rows through the async proxy
        named_barrier(1 + t, 128);
        if (r == 0) {
          tma_store_4d(&p.tm_o, sStg + t * kChunkBytes, ch * 64, u.q0 + t * kTileM, p.head_begin + u.hl, u.b);
          bulk_commit();
        }
      }
      if (p.lse != nullptr && row < p.Lq)
        p.lse[(int64_t)u.b * p.lse_sb + (int64_t)(p.head_begin + u.hl) * p.lse_sh + row] =
            (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
    }
    if (r == 0) bulk_wait_read();  // the CTA's shared memory must outlive the stores' reads
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
std::mutex g_persist_mu;
bool g_persist_regs_ok[kMaxDev][2] = {};
size_t g_persist_smem_set[kMaxDev][2] = {};

}  // namespace

size_t fwd_persist_smem_bytes(int D, int batch, int kv_tiles, bool has_mask) {
  return 1024 /* alignment slack */ + (D == 128 ? PSmem<128>::kBytes : PSmem<64>::kBytes) +
         (has_mask ? meta_bytes(batch, kv_tiles) : 0);
}

// Once per device and head dim: the register count the warpgroup split
// assumes; and the dynamic shared-memory limit whenever a larger size is needed.
cudaError_t prepare_fwd_persist(int D, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int di = D == 128 ? 1 : 0;
  std::lock_guard<std::mutex> lock(g_persist_mu);
  const void* ks[2] = {
      D == 128 ? (const void*)fwd_persist_sm100_kernel<128, false> : (const void*)fwd_persist_sm100_kernel<64, false>,
      D == 128 ? (const void*)fwd_persist_sm100_kernel<128, true> : (const void*)fwd_persist_sm100_kernel<64, true>};
  if (!g_persist_regs_ok[dev][di]) {
    for (const void* k : ks) {
      cudaFuncAttributes fa;
      if ((e = cudaFuncGetAttributes(&fa, k)) != cudaSuccess) return e;
      if (fa.numRegs != (int)kLaunchRegs) return cudaErrorInvalidConfiguration;
    }
    g_persist_regs_ok[dev][di] = true;
  }
  if (smem > g_persist_smem_set[dev][di]) {
    for (const void* k : ks)
      if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
        return e;
    g_persist_smem_set[dev][di] = smem;
  }
  return cudaSuccess;
}

// p.n_full is the unit count; `ctas` <= units CTAs walk them round-robin
// (prepare_fwd_persist must have succeeded for D and at least smem).
cudaError_t launch_fwd_persist(const FwdParams& p, int D, int ctas, size_t smem, cudaStream_t s) {
  const bool m = p.mask != nullptr;
  if (D == 128 && m) return launch_pdl(fwd_persist_sm100_kernel<128, true>, dim3(ctas), dim3(kThreads), smem, s, p);
  if (D == 128) return launch_pdl(fwd_persist_sm100_kernel<128, false>, dim3(ctas), dim3(kThreads), smem, s, p);
  if (m) return launch_pdl(fwd_persist_sm100_kernel<64, true>, dim3(ctas), dim3(kThreads), smem, s, p);
  return launch_pdl(fwd_persist_sm100_kernel<64, false>, dim3(ctas), dim3(kThreads), smem, s, p);
}

}  // namespace ltx
