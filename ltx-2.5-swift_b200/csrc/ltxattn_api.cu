// ltxattn_api.cu -- the C ABI of libltxattn_cuda (include/ltxattn.h).
//
// Validation mirrors the reference's up-front refusals
// (DiTAttention.Failure, DiTAttention.swift:107-122): a wrong shape, dtype or
// alignment is an error code with a message, never a silent fallback.
#include <dlfcn.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ltxattn.h"
#include "ltxattn_internal.h"

namespace ltx {

__device__ int g_error_word;

namespace {

thread_local std::string t_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

// A runtime call of the library failed: report it, and take the failure out of
// the runtime's per-thread last-error slot so that it is not read again as the
// result of a later, unrelated kernel launch (ours or the caller's).  Sticky
// errors stay: the runtime reports those on every call anyway.
int cuda_fail(cudaError_t e, const char* what) {
  (void)cudaGetLastError();
  return fail(LTXATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency).

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [D, T, H, B] bf16 view, box {64, 128, 1, 1}, 128-byte swizzle.  Strides of
// size-1 dims are irrelevant to addressing; they are replaced by a packed
// value so the encoder's alignment checks see a valid number.
int make_tmap(CUtensorMap* map, const void* ptr, int D, int T, int H, int B, int64_t st, int64_t sh,
              int64_t sb, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(LTXATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  int64_t s1 = st, s2 = sh, s3 = sb;
  if (T == 1) s1 = D;
  if (H == 1) s2 = s1 * T;
  if (B == 1) s3 = s2 * H;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)s1 * 2, (cuuint64_t)s2 * 2, (cuuint64_t)s3 * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LTXATTN_ERR_ALIGN, "%s: cuTensorMapEncodeTiled rejected the view (CUresult %d)", name, (int)r);
  return LTXATTN_OK;
}

// fp32 [D, T, H, B] contiguous buffer, box {32, 128, 1, 1} (128-byte rows), 128-byte swizzle
int make_tmap_f32(CUtensorMap* map, void* ptr, int D, int T, int H, int B, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(LTXATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 4, (cuuint64_t)D * T * 4, (cuuint64_t)D * T * H * 4};
  cuuint32_t box[4] = {32, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LTXATTN_ERR_ALIGN, "%s: cuTensorMapEncodeTiled rejected the view (CUresult %d)", name, (int)r);
  return LTXATTN_OK;
}

int current_sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// shared validation of the forward / backward shape block

struct Shape {
  int dtype, B, H, Lq, Lk, D, h0, Hc;
  size_t esize;
};

int check_tensor(const ltxattn_tensor& t, const char* name, const Shape& s, bool need_tma) {
  if (t.data == nullptr) return fail(LTXATTN_ERR_ARG, "%s is NULL", name);
  if (t.stride_b < 0 || t.stride_h < 0 || t.stride_t < 0)
    return fail(LTXATTN_ERR_SHAPE, "%s has a negative stride", name);
  if (need_tma) {
    if (!aligned16(t.data)) return fail(LTXATTN_ERR_ALIGN, "%s is not 16-byte aligned", name);
    const int64_t q = 16 / (int64_t)s.esize;
    if ((s.B > 1 && t.stride_b % q) || (s.H > 1 && t.stride_h % q) || t.stride_t % q)
      return fail(LTXATTN_ERR_ALIGN, "%s strides must be multiples of %lld elements (16 bytes)", name,
                  (long long)q);
  }
  return LTXATTN_OK;
}

int check_shape(int dtype, int B, int H, int Lq, int Lk, int D, int head_begin, int head_count, Shape* s) {
  if (dtype != LTXATTN_F32 && dtype != LTXATTN_BF16)
    return fail(LTXATTN_ERR_DTYPE, "dtype %d is neither LTXATTN_F32 nor LTXATTN_BF16", dtype);
  if (B < 1 || H < 1 || Lq < 1 || Lk < 1)
    return fail(LTXATTN_ERR_SHAPE, "batch %d, heads %d, q_len %d, kv_len %d: all must be >= 1", B, H, Lq, Lk);
  if (D != 64 && D != 128)
    return fail(LTXATTN_ERR_UNSUPPORTED, "head_dim %d is not supported (64 and 128 are: the DiT's audio and video heads)",
                D);
  if (Lk > kMaxKvLen) return fail(LTXATTN_ERR_UNSUPPORTED, "kv_len %d exceeds %d", Lk, kMaxKvLen);
  const int hc = head_count == 0 ? H - head_begin : head_count;
  if (head_begin < 0 || hc < 1 || head_begin + hc > H)
    return fail(LTXATTN_ERR_ARG, "head range [%d, %d) is outside [0, %d)", head_begin, head_begin + hc, H);
  if ((int64_t)B * hc > 65535 * 65535LL) return fail(LTXATTN_ERR_SHAPE, "too many heads");
  if (B > 65535 || hc > 65535) return fail(LTXATTN_ERR_UNSUPPORTED, "batch and head count must be <= 65535");
  s->dtype = dtype;
  s->B = B;
  s->H = H;
  s->Lq = Lq;
  s->Lk = Lk;
  s->D = D;
  s->h0 = head_begin;
  s->Hc = hc;
  s->esize = dtype == LTXATTN_BF16 ? 2 : 4;
  return LTXATTN_OK;
}

int check_rotary(const ltxattn_rotary& r, const char* name, int tokens_needed) {
  if (r.cos == nullptr) return LTXATTN_OK;
  if (r.sin == nullptr) return fail(LTXATTN_ERR_ARG, "%s has cos but no sin", name);
  if (r.tokens < tokens_needed)
    return fail(LTXATTN_ERR_SHAPE, "%s covers %d tokens, expected at least %d", name, r.tokens, tokens_needed);
  if (r.stride_b < 0 || r.stride_h < 0 || r.stride_t < 0)
    return fail(LTXATTN_ERR_SHAPE, "%s has a negative stride", name);
  return LTXATTN_OK;
}

// ---------------------------------------------------------------------------
// KV splitting for a launch of at least one wave.  One CTA per SM: the units
// (256-row query block, head, batch) run in waves of sm_count, and a thin last
// wave leaves most SMs idle for a whole unit's time.  Splitting the KV range
// of the last n_tail units s ways (n_tail = the last partial wave plus k whole
// waves) replaces that wave by ceil(n_tail * s / sms) waves of 1/s-size CTAs:
//   time = (waves - k) * t(1) + ceil(n_tail * s / sms) * t(s) + combine
//   t(s) = t_cta + ceil(kv_tiles / s) * t_tile
// with t_tile ~ 1.8 us per 128-key step of a two-tile CTA, t_cta ~ 8 us of
// per-CTA prologue and epilogue, and the combine moving s fp32 partials of the
// tail units' O (written and read back) at ~5 TB/s plus ~3 us for its launch.
// The cheapest choice must beat no split by 1.5%.  (29,760 tokens and 4 heads
// per GPU: 468 units = 3 waves + 24, split 6 ways; 32 heads at 3,120 tokens:
// 416 units, no split; 126 queries against 3,120 keys, 32 heads: all 32 units
// split 4 ways, one wave.)
struct SplitChoice {
  int64_t n_tail;
  int splits;
  double us;  // the model's time for the choice
};

SplitChoice tail_splits(int64_t units, int sms, int kv_tiles, int D) {
  constexpr double kTileUs = 1.83, kCtaUs = 9.0, kBytesPerUs = 5.0e6, kLaunchUs = 3.0;
  auto unit_us = [&](int sp) { return kCtaUs + (double)((kv_tiles + sp - 1) / sp) * kTileUs; };
  const int64_t waves = units / sms, rem = units % sms;
  const double whole = (double)((units + sms - 1) / sms) * unit_us(1);
  SplitChoice best{0, 1, whole};
  double best_us = whole;
  for (int64_t k = 0; k <= waves; ++k) {
    const int64_t n_tail = rem + k * sms;
    if (n_tail == 0) continue;
    for (int sp = 2; sp <= kMaxSplits && kv_tiles / sp >= 2; ++sp) {
      const double combine = kLaunchUs + 2.0 * sp * (double)n_tail * kFwdBlockM * D * 4.0 / kBytesPerUs;
      const double us = (double)(waves - k) * unit_us(1) + (double)((n_tail * sp + sms - 1) / sms) * unit_us(sp) +
                        combine;
      if (us < best_us) {
        best_us = us;
        best = {n_tail, sp, us};
      }
    }
  }
  return best_us < 0.985 * whole ? best : SplitChoice{0, 1, whole};
}

// The persistent forward (fwd_persist_sm100.cu) against one CTA per unit, with
// constants fitted to CUDA-event timings on a B200 (32 heads x 3,120 queries,
// D = 128, 2 to 25 KV tiles per unit, L2 flushed):
//   one CTA per unit:  ceil(units / sms) * (1.83 us * kv_tiles + 9.0 us)
//   persistent:        4.6 us + ceil(units / sms) * (2.07 us * kv_tiles + 4.6 us)
// A unit boundary costs the persistent kernel less than a CTA does the other
// (4.6 against 9.0 us), but its KV step is ~13% slower, so it wins for short
// KV ranges (below ~12 tiles at three rounds: 30.8 against 37.8 us at 2 tiles)
// and loses at the 3,120-token self-attention (173.5 against 163.8 us).
double tiled_us(int64_t units, int sms, int kv_tiles) {
  return (double)((units + sms - 1) / sms) * (1.83 * kv_tiles + 9.0);
}
double persist_us(int64_t units, int sms, int kv_tiles) {
  return 4.6 + (double)((units + sms - 1) / sms) * (2.07 * kv_tiles + 4.6);
}

// Uniform split count (every unit split) for masked or banded calls, whose
// per-unit work the planner cannot see: the same cost terms over all units,
// at most 4 splits of >= 8 KV tiles each, and 3% better than no split.
int uniform_splits(int64_t units, int sms, int kv_tiles, double out_elems) {
  constexpr double kTileUs = 1.8, kCtaUs = 8.0, kBytesPerUs = 5.0e6;
  auto cost = [&](int sp) {
    const double waves = (double)((units * sp + sms - 1) / sms);
    const double combine = sp > 1 ? 2.0 * sp * out_elems * 4.0 / kBytesPerUs : 0.0;
    return waves * ((double)kv_tiles / sp * kTileUs + kCtaUs) + combine;
  };
  int best = 1;
  double best_cost = cost(1);
  for (int sp = 2; sp <= 4 && kv_tiles / sp >= 8; ++sp) {
    const double c = cost(sp);
    if (c < best_cost) {
      best = sp;
      best_cost = c;
    }
  }
  return best_cost < 0.97 * cost(1) ? best : 1;
}

// ---------------------------------------------------------------------------
// forward plan: workspace layout and split count (identical for the
// workspace query and the call)

struct FwdPlan {
  Shape s;
  bool rope_q, rope_k;
  const ltxattn_rotary* kr;  // table used for k
  int kv_heads, group;        // grouped KV heads: query head h reads kv head h / group
  int causal, window;
  int q_tiles, kv_tiles, splits;
  int64_t units, n_full, n_tail;  // bf16: n_tail units split `splits` ways after n_full whole ones
  bool short_kv;                  // bf16, one KV tile, more units than SMs: the persistent kernel
  bool persist;                   // bf16, no band, at least a wave: the persistent multi-tile kernel
  int sms;
  size_t off_q, off_k, off_po, off_pl, total;
};

int plan_fwd(const ltxattn_fwd_args* a, FwdPlan* P) {
  if (a == nullptr) return fail(LTXATTN_ERR_ARG, "args is NULL");
  int rc = check_shape(a->dtype, a->batch, a->heads, a->q_len, a->kv_len, a->head_dim, a->head_begin,
                       a->head_count, &P->s);
  if (rc) return rc;
  const Shape& s = P->s;
  P->kv_heads = a->kv_heads == 0 ? s.H : a->kv_heads;
  if (P->kv_heads < 1 || s.H % P->kv_heads)
    return fail(LTXATTN_ERR_SHAPE, "kv_heads %d does not divide heads %d", a->kv_heads, s.H);
  P->group = s.H / P->kv_heads;
  P->causal = a->causal != 0;
  P->window = a->window;
  if (a->window < 0) return fail(LTXATTN_ERR_ARG, "window %d is negative", a->window);
  if (P->causal && s.Lq != s.Lk)
    return fail(LTXATTN_ERR_SHAPE, "causal attention needs q_len == kv_len (got %d and %d)", s.Lq, s.Lk);
  P->rope_q = a->q_rotary.cos != nullptr;
  if (P->rope_q && P->group > 1)
    return fail(LTXATTN_ERR_UNSUPPORTED, "grouped KV heads take no rotary tables: rotate q and k before the call");
  P->kr = (a->k_rotary.cos != nullptr) ? &a->k_rotary : &a->q_rotary;
  P->rope_k = P->rope_q;  // k_rotary without q_rotary is ignored (DiTAttention.swift:364)
  if (P->rope_q) {
    if ((rc = check_rotary(a->q_rotary, "q_rotary", s.Lq))) return rc;
    if ((rc = check_rotary(*P->kr, a->k_rotary.cos ? "k_rotary" : "q_rotary (used for k)", s.Lk))) return rc;
  }
  P->q_tiles = s.dtype == LTXATTN_BF16 ? (s.Lq + kFwdBlockM - 1) / kFwdBlockM : (s.Lq + kTileM - 1) / kTileM;
  P->kv_tiles = (s.Lk + kTileN - 1) / kTileN;
  P->splits = 1;
  P->units = (int64_t)P->q_tiles * s.Hc * s.B;
  P->n_tail = 0;
  P->short_kv = false;
  P->persist = false;
  P->sms = 0;
  if (s.dtype == LTXATTN_BF16) {
    const int64_t units = P->units;
    if (a->num_splits > 0) {
      P->splits = std::min({a->num_splits, P->kv_tiles, kMaxSplits});
      P->n_tail = units;
    } else if (a->num_splits == 0) {
      const int sms = current_sm_count();
      P->sms = sms;
      // one KV tile and more units than SMs: a persistent CTA per SM overlaps
      // its units (fwd_short_sm100.cu); no split
      P->short_kv = P->kv_tiles == 1 && !P->causal && P->window == 0 && units > sms;
      const bool opaque = a->key_mask != nullptr || P->causal || P->window > 0;  // per-unit work unknown
      const bool banded = P->causal || P->window > 0;
      // a key mask but no band: units of one batch row walk the same live tiles,
      // which the persistent kernel lists once per row (shared memory permitting);
      // the live count is unknown here, so the model is evaluated at kv_tiles
      const bool persist_masked = a->key_mask != nullptr && !banded && units >= sms && P->kv_tiles > 1 &&
                                  fwd_persist_smem_bytes(s.D, s.B, P->kv_tiles, true) <= kMaxDynamicSmem &&
                                  persist_us(units, sms, P->kv_tiles) < tiled_us(units, sms, P->kv_tiles);
      if (units < sms && P->kv_tiles > 1 && opaque) {
        // fewer units than SMs: as many splits as keep one wave
        P->splits = std::max(1, std::min({(int)(sms / units), P->kv_tiles, kMaxSplits}));
        P->n_tail = units;
      } else if (P->short_kv) {
        P->splits = 1;
      } else if (units < sms && P->kv_tiles > 1) {
        const SplitChoice c = tail_splits(units, sms, P->kv_tiles, s.D);
        P->splits = c.splits;
        P->n_tail = c.n_tail;
      } else if (persist_masked) {
        P->persist = true;
      } else if (units >= sms && opaque) {
        P->splits = uniform_splits(units, sms, P->kv_tiles, (double)s.B * s.Hc * s.Lq * s.D);
        P->n_tail = units;
      } else if (units >= sms) {
        // whole units back to back on persistent CTAs, or one CTA per unit with
        // the last units' KV ranges split: whichever the model times shorter
        const SplitChoice c = tail_splits(units, sms, P->kv_tiles, s.D);
        if (P->kv_tiles > 1 && persist_us(units, sms, P->kv_tiles) < c.us) {
          P->persist = true;
        } else {
          P->splits = c.splits;
          P->n_tail = c.n_tail;
        }
      }
    } else {
      return fail(LTXATTN_ERR_ARG, "num_splits %d is negative", a->num_splits);
    }
    if (P->splits == 1) P->n_tail = 0;
  }
  P->n_full = P->units - P->n_tail;
  if (P->n_full + P->n_tail * P->splits > (int64_t)INT32_MAX)
    return fail(LTXATTN_ERR_UNSUPPORTED, "%lld query blocks exceed one launch", (long long)P->units);
  size_t off = 0;
  P->off_q = off;
  if (P->rope_q) off += align256((size_t)s.B * s.Hc * s.Lq * s.D * s.esize);
  P->off_k = off;
  if (P->rope_k) off += align256((size_t)s.B * s.Hc * s.Lk * s.D * s.esize);
  P->off_po = off;
  if (P->splits > 1) off += align256((size_t)P->splits * P->n_tail * kFwdBlockM * s.D * sizeof(float));
  P->off_pl = off;
  if (P->splits > 1) off += align256((size_t)P->splits * P->n_tail * kFwdBlockM * sizeof(float));
  P->total = off;
  return LTXATTN_OK;
}

struct BwdPlan {
  Shape s;
  bool rope;
  const ltxattn_rotary* kr;
  int Lq_pad;
  size_t off_q, off_k, off_l, off_d, total;
};

int plan_bwd(const ltxattn_bwd_args* a, BwdPlan* P) {
  if (a == nullptr) return fail(LTXATTN_ERR_ARG, "args is NULL");
  int rc = check_shape(a->dtype, a->batch, a->heads, a->q_len, a->kv_len, a->head_dim, a->head_begin,
                       a->head_count, &P->s);
  if (rc) return rc;
  const Shape& s = P->s;
  P->rope = a->q_rotary.cos != nullptr;
  P->kr = (a->k_rotary.cos != nullptr) ? &a->k_rotary : &a->q_rotary;
  if (P->rope) {
    if ((rc = check_rotary(a->q_rotary, "q_rotary", s.Lq))) return rc;
    if ((rc = check_rotary(*P->kr, a->k_rotary.cos ? "k_rotary" : "q_rotary (used for k)", s.Lk))) return rc;
  }
  P->Lq_pad = (s.Lq + kTileM - 1) / kTileM * kTileM;
  size_t off = 0;
  P->off_q = off;
  if (P->rope) off += align256((size_t)s.B * s.Hc * s.Lq * s.D * s.esize);
  P->off_k = off;
  if (P->rope) off += align256((size_t)s.B * s.Hc * s.Lk * s.D * s.esize);
  P->off_l = off;
  off += align256((size_t)s.B * s.Hc * P->Lq_pad * sizeof(float));
  P->off_d = off;
  off += align256((size_t)s.B * s.Hc * P->Lq_pad * sizeof(float));
  P->total = off;
  return LTXATTN_OK;
}

RopeParams rope_params(const ltxattn_tensor& x, const ltxattn_rotary& r, const Shape& s, int T, void* y) {
  RopeParams p{};
  p.x = x.data;
  p.x_sb = x.stride_b;
  p.x_sh = x.stride_h;
  p.x_st = x.stride_t;
  p.cos = r.cos;
  p.sin = r.sin;
  p.t_sb = r.stride_b;
  p.t_sh = r.stride_h;
  p.t_st = r.stride_t;
  p.y = y;  // contiguous [B][Hc][T][D]
  p.y_st = s.D;
  p.y_sh = (int64_t)T * s.D;
  p.y_sb = (int64_t)s.Hc * T * s.D;
  p.B = s.B;
  p.Hc = s.Hc;
  p.T = T;
  p.D = s.D;
  p.head_begin = s.h0;
  return p;
}

}  // namespace

int set_error_message(int status, const char* msg) {
  t_last_error = msg;
  return status;
}

// The device error word's address, looked up once per device (a call then
// makes no runtime query that could disturb a stream capture).  The address
// belongs to the context of that first call; after a cudaDeviceReset in the
// same process it is stale, so the library is not used across one.
int* device_error_word() {
  constexpr int kDevs = 64;
  static std::mutex mu;
  static int* cache[kDevs] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevs) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_error_word) != cudaSuccess) return nullptr;
    cache[dev] = p;
  }
  return cache[dev];
}

}  // namespace ltx

using namespace ltx;

extern "C" {

int ltxattn_abi_version(void) { return LTXATTN_ABI_VERSION; }

const char* ltxattn_last_error(void) { return t_last_error.c_str(); }

size_t ltxattn_fwd_workspace(const ltxattn_fwd_args* a) {
  FwdPlan P;
  if (plan_fwd(a, &P) != LTXATTN_OK) return 0;
  return P.total;
}

int ltxattn_fwd_plan(const ltxattn_fwd_args* a, ltxattn_fwd_plan_info* info) {
  if (info == nullptr) return fail(LTXATTN_ERR_ARG, "info is NULL");
  FwdPlan P;
  const int rc = plan_fwd(a, &P);
  if (rc) return rc;
  const bool bf16 = P.s.dtype == LTXATTN_BF16;
  info->kernel = !bf16 ? 0 : (P.short_kv ? 2 : (P.persist ? 3 : 1));
  info->splits = P.splits;
  info->units = P.units;
  info->split_units = P.n_tail;
  info->launches = 1 + ((P.rope_q || P.rope_k) ? 1 : 0) + (P.splits > 1 ? 1 : 0);
  return LTXATTN_OK;
}

}  // extern "C"

// ltxattn_fwd, and ltxattn_fwd_gather when g is set (validated by the caller):
// the same call with KV ranges unsplit and the epilogue's peer stores.
static int fwd_impl(const ltxattn_fwd_args* a_in, void* stream, const ltxattn_gather_peers* g) {
  ltxattn_fwd_args a_unsplit;
  const ltxattn_fwd_args* a = a_in;
  FwdPlan P;
  int rc = plan_fwd(a, &P);
  if (rc) return rc;
  if (g != nullptr && (P.persist || P.short_kv)) {
    // the fused all-gather lives in the tiled kernel and the combine: a call the
    // planner gives to a persistent kernel runs tiled with unsplit KV ranges
    a_unsplit = *a_in;
    a_unsplit.num_splits = 1;
    a = &a_unsplit;
    if ((rc = plan_fwd(a, &P))) return rc;
  }
  const Shape& s = P.s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = s.dtype == LTXATTN_BF16;
  if ((rc = check_tensor(a->q, "q", s, bf16 && !P.rope_q))) return rc;
  if ((rc = check_tensor(a->k, "k", s, bf16 && !P.rope_k))) return rc;
  if ((rc = check_tensor(a->v, "v", s, bf16))) return rc;
  if ((rc = check_tensor(a->out, "out", s, bf16))) return rc;
  if (a->gate != nullptr && (a->gate_stride_b < 0 || a->gate_stride_t < 0 || a->gate_stride_h < 0))
    return fail(LTXATTN_ERR_SHAPE, "gate has a negative stride");
  if (P.total > 0) {
    if (a->workspace == nullptr || a->workspace_bytes < P.total)
      return fail(LTXATTN_ERR_WORKSPACE, "workspace of %zu bytes is needed, %zu given", P.total,
                  a->workspace == nullptr ? (size_t)0 : a->workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
      return fail(LTXATTN_ERR_ALIGN, "workspace must be 256-byte aligned");
  }
  int* err = device_error_word();
  if (!err) return fail(LTXATTN_ERR_CUDA, "no device error word (is a CUDA device current?)");
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);

  // inputs as the attention kernel sees them: rotated copies in the workspace
  // (contiguous, local heads) or the caller's views
  ltxattn_tensor q = a->q, k = a->k;
  int q_head_off = s.h0, kv_head_off = s.h0;
  cudaError_t e;
  // The rotation pre-pass is launched only after every piece of host work of
  // this call is done, so it and the attention kernel queue back to back with
  // no host gap between them.
  RopeParams rope_k{}, rope_q{};
  if (P.rope_q) {
    // k is always rotated with q (with its own table or q's); one launch
    // rotates both into the workspace
    rope_k = rope_params(a->k, *P.kr, s, s.Lk, ws + P.off_k);
    rope_q = rope_params(a->q, a->q_rotary, s, s.Lq, ws + P.off_q);
    q.data = ws + P.off_q;
    q.stride_t = s.D;
    q.stride_h = (int64_t)s.Lq * s.D;
    q.stride_b = (int64_t)s.Hc * s.Lq * s.D;
    q_head_off = 0;
  }
  ltxattn_tensor v = a->v;
  if (P.rope_k) {
    k.data = ws + P.off_k;
    k.stride_t = s.D;
    k.stride_h = (int64_t)s.Lk * s.D;
    k.stride_b = (int64_t)s.Hc * s.Lk * s.D;
  }
  const int k_head_off = P.rope_k ? 0 : s.h0;
  const int v_head_off = s.h0;

  auto launch_pre_pass = [&]() -> int {
    if (!P.rope_q) return LTXATTN_OK;
    const cudaError_t er = launch_rope(&rope_q, &rope_k, bf16, st);
    return er == cudaSuccess ? LTXATTN_OK : cuda_fail(er, "rope launch");
  };
  if (!bf16) {
    if ((rc = launch_pre_pass())) return rc;
    F32Params p{};
    p.q = static_cast<const float*>(q.data);
    p.k = static_cast<const float*>(k.data);
    p.v = static_cast<const float*>(v.data);
    p.q_sb = q.stride_b; p.q_sh = q.stride_h; p.q_st = q.stride_t;
    p.k_sb = k.stride_b; p.k_sh = k.stride_h; p.k_st = k.stride_t;
    p.v_sb = v.stride_b; p.v_sh = v.stride_h; p.v_st = v.stride_t;
    p.q_head_off = q_head_off;
    p.kv_head_off = 0;
    // k and v may sit at different head offsets (k rotated into the workspace)
    if (k_head_off != v_head_off) {
      p.k = static_cast<const float*>(k.data);  // local heads
      p.v = static_cast<const float*>(v.data) + (int64_t)v_head_off * v.stride_h;
    } else {
      p.kv_head_off = k_head_off;
    }
    p.out = static_cast<float*>(a->out.data);
    p.o_sb = a->out.stride_b; p.o_sh = a->out.stride_h; p.o_st = a->out.stride_t;
    p.lse = a->lse;
    p.lse_sb = a->lse_stride_b; p.lse_sh = a->lse_stride_h;
    p.mask = a->key_mask;
    p.mask_sb = a->key_mask_stride_b;
    p.Lq = s.Lq; p.Lk = s.Lk; p.head_begin = s.h0;
    p.scale = a->scale;
    p.group = P.group;
    p.causal = P.causal;
    p.window = P.window;
    p.gate = static_cast<const float*>(a->gate);
    p.g_sb = a->gate_stride_b; p.g_st = a->gate_stride_t; p.g_sh = a->gate_stride_h;
    e = launch_fwd_f32(p, s.D, s.Hc, s.B, st);
    if (e != cudaSuccess) return cuda_fail(e, "fwd_f32 launch");
    return LTXATTN_OK;
  }

  FwdParams p{};
  if ((rc = make_tmap(&p.tm_q, q.data, s.D, s.Lq, P.rope_q ? s.Hc : s.H, s.B, q.stride_t,
                      q.stride_h, q.stride_b, "q")))
    return rc;
  if ((rc = make_tmap(&p.tm_k, k.data, s.D, s.Lk, P.rope_k ? s.Hc : P.kv_heads, s.B, k.stride_t, k.stride_h,
                      k.stride_b, "k")))
    return rc;
  // v keeps the caller's head indexing; k may be local.  One kv_head_off
  // serves both only when they agree, so v is re-based to local heads when
  // k is a local copy.
  const void* vptr = v.data;
  int vH = P.kv_heads;
  if (P.rope_k) {
    vptr = static_cast<const __nv_bfloat16*>(v.data) + (int64_t)s.h0 * v.stride_h;
    vH = s.Hc;
    if (!aligned16(vptr)) return fail(LTXATTN_ERR_ALIGN, "v head block is not 16-byte aligned");
  }
  if ((rc = make_tmap(&p.tm_v, vptr, s.D, s.Lk, vH, s.B, v.stride_t, v.stride_h, v.stride_b, "v"))) return rc;
  if ((rc = make_tmap(&p.tm_o, a->out.data, s.D, s.Lq, s.H, s.B, a->out.stride_t, a->out.stride_h,
                      a->out.stride_b, "out")))
    return rc;
  p.out = static_cast<__nv_bfloat16*>(a->out.data);
  p.o_sb = a->out.stride_b;
  p.o_sh = a->out.stride_h;
  p.o_st = a->out.stride_t;
  p.lse = a->lse;
  p.lse_sb = a->lse_stride_b;
  p.lse_sh = a->lse_stride_h;
  p.mask = a->key_mask;
  p.mask_sb = a->key_mask_stride_b;
  p.mask_vec = a->key_mask != nullptr && aligned16(a->key_mask) && (s.B == 1 || a->key_mask_stride_b % 16 == 0);
  p.Lq = s.Lq;
  p.Lk = s.Lk;
  p.head_begin = s.h0;
  p.q_head_off = q_head_off;
  p.kv_head_off = P.rope_k ? 0 : s.h0;
  p.n_kv_tiles = P.kv_tiles;
  p.q_blocks = P.q_tiles;
  p.Hc = s.Hc;
  p.n_full = (int)P.n_full;
  p.n_tail = (int)P.n_tail;
  p.num_splits = P.splits;
  p.group = P.group;
  p.causal = P.causal;
  p.window = P.window;
  p.gate = static_cast<const __nv_bfloat16*>(a->gate);
  p.g_sb = a->gate_stride_b;
  p.g_st = a->gate_stride_t;
  p.g_sh = a->gate_stride_h;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  if (P.splits > 1 && (rc = make_tmap_f32(&p.tm_part, ws + P.off_po, s.D, kFwdBlockM, (int)P.n_tail, P.splits,
                                          "split partials")))
    return rc;
  p.part_lse = P.splits > 1 ? reinterpret_cast<float*>(ws + P.off_pl) : nullptr;
  p.err = err;
  GatherSync gs{};
  if (g != nullptr) {
    gs.n = g->world;
    gs.rank = g->rank;
    gs.epoch = g->epoch;
    gs.err = err;
    for (int d = 0; d < g->world; ++d) {
      gs.sig[d] = g->signals[d];
      if (d == g->rank) continue;
      // rank d's output, same geometry as this rank's (every rank passes the same shape)
      if ((rc = make_tmap(&p.tm_peer[p.peer_n], g->out[d], s.D, s.Lq, s.H, s.B, a->out.stride_t, a->out.stride_h,
                          a->out.stride_b, "peer out")))
        return rc;
      ++p.peer_n;
    }
  }
  const size_t smem = fwd_bf16_smem_bytes(s.D, s.Lk, a->key_mask != nullptr);
  e = prepare_fwd_bf16(s.D, smem);
  if (e == cudaErrorInvalidConfiguration)
    return fail(LTXATTN_ERR_CUDA, "fwd_bf16: the loaded kernel's register count differs from its warpgroup split");
  if (e != cudaSuccess) return cuda_fail(e, "fwd_bf16 setup");
  if ((rc = launch_pre_pass())) return rc;
  if (P.short_kv) {
    e = prepare_fwd_short(s.D);
    if (e == cudaErrorInvalidConfiguration)
      return fail(LTXATTN_ERR_CUDA, "fwd_short: the loaded kernel's register count differs from its warpgroup split");
    if (e != cudaSuccess) return cuda_fail(e, "fwd_short setup");
    e = launch_fwd_short(p, s.D, (int)P.units, P.sms, st);
    if (e != cudaSuccess) return cuda_fail(e, "fwd_short launch");
    return LTXATTN_OK;
  }
  if (P.persist) {
    const size_t psmem = fwd_persist_smem_bytes(s.D, s.B, P.kv_tiles, a->key_mask != nullptr);
    e = prepare_fwd_persist(s.D, psmem);
    if (e == cudaErrorInvalidConfiguration)
      return fail(LTXATTN_ERR_CUDA, "fwd_persist: the loaded kernel's register count differs from its warpgroup split");
    if (e != cudaSuccess) return cuda_fail(e, "fwd_persist setup");
    e = launch_fwd_persist(p, s.D, (int)std::min<int64_t>(P.units, P.sms), psmem, st);
    if (e != cudaSuccess) return cuda_fail(e, "fwd_persist launch");
    return LTXATTN_OK;
  }
  if (g != nullptr && (e = launch_gather_enter(gs, st)) != cudaSuccess) return cuda_fail(e, "gather entry launch");
  e = launch_fwd_bf16(p, s.D, smem, st);
  if (e != cudaSuccess) return cuda_fail(e, "fwd_bf16 launch");
  if (P.splits > 1) {
    CombineParams c{};
    c.part_o = reinterpret_cast<const float*>(ws + P.off_po);
    c.part_lse = p.part_lse;
    c.out = p.out;
    c.o_sb = p.o_sb;
    c.o_sh = p.o_sh;
    c.o_st = p.o_st;
    c.lse = a->lse;
    c.lse_sb = a->lse_stride_b;
    c.lse_sh = a->lse_stride_h;
    c.Hc = s.Hc;
    c.Lq = s.Lq;
    c.D = s.D;
    c.num_splits = P.splits;
    c.head_begin = s.h0;
    c.q_blocks = P.q_tiles;
    c.n_full = (int)P.n_full;
    c.n_tail = (int)P.n_tail;
    c.gate = p.gate;
    c.g_sb = p.g_sb;
    c.g_st = p.g_st;
    c.g_sh = p.g_sh;
    if (g != nullptr)
      for (int d = 0; d < g->world; ++d)
        if (d != g->rank) c.peer_out[c.peer_n++] = static_cast<__nv_bfloat16*>(g->out[d]);
    e = launch_combine(c, st);
    if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  }
  if (g != nullptr && (e = launch_gather_done(gs, st)) != cudaSuccess) return cuda_fail(e, "gather completion launch");
  return LTXATTN_OK;
}

extern "C" {

int ltxattn_fwd(const ltxattn_fwd_args* a, void* stream) { return fwd_impl(a, stream, nullptr); }

int ltxattn_fwd_gather(const ltxattn_fwd_args* a, const ltxattn_gather_peers* g, void* stream) {
  if (a == nullptr || g == nullptr) return fail(LTXATTN_ERR_ARG, "args or peers is NULL");
  if (a->dtype != LTXATTN_BF16) return fail(LTXATTN_ERR_DTYPE, "ltxattn_fwd_gather: bf16 only");
  if (g->world < 2 || g->world > 8 || g->rank < 0 || g->rank >= g->world)
    return fail(LTXATTN_ERR_ARG, "ltxattn_fwd_gather: rank %d of world %d (2 to 8 ranks)", g->rank, g->world);
  if (g->epoch == 0) return fail(LTXATTN_ERR_ARG, "ltxattn_fwd_gather: epochs start at 1");
  if (g->out[g->rank] != a->out.data)
    return fail(LTXATTN_ERR_ARG, "ltxattn_fwd_gather: peers->out[rank] must be args->out.data");
  for (int d = 0; d < g->world; ++d) {
    if (g->out[d] == nullptr || g->signals[d] == nullptr)
      return fail(LTXATTN_ERR_ARG, "ltxattn_fwd_gather: rank %d's output or signal words are NULL", d);
    if ((reinterpret_cast<uintptr_t>(g->out[d]) & 15u) || (reinterpret_cast<uintptr_t>(g->signals[d]) & 3u))
      return fail(LTXATTN_ERR_ALIGN, "ltxattn_fwd_gather: rank %d's output must be 16-byte aligned", d);
  }
  if ((a->out.stride_b % 8) || (a->out.stride_h % 8) || (a->out.stride_t % 8))
    return fail(LTXATTN_ERR_ALIGN, "ltxattn_fwd_gather: output strides must be multiples of 8 elements");
  return fwd_impl(a, stream, g);
}

}  // extern "C"

// Validation and parameter block of one q / k preparation.
static int qk_prep_params(const ltxattn_qk_prep_args* a, QkPrepParams* out, bool* is_bf16) {
  if (a == nullptr) return fail(LTXATTN_ERR_ARG, "args is NULL");
  Shape s;
  int rc = check_shape(a->dtype, a->batch, a->heads, a->tokens, a->tokens, a->head_dim, 0, 0, &s);
  if (rc) return rc;
  const int inner = s.H * s.D;
  if (inner % 512 != 0 || inner > 8192)
    return fail(LTXATTN_ERR_UNSUPPORTED, "heads * head_dim = %d is not a multiple of 512 up to 8192", inner);
  if (a->x == nullptr || a->weight == nullptr) return fail(LTXATTN_ERR_ARG, "x and weight must be device pointers");
  if (a->x_stride_b < 0 || a->x_stride_t < 0) return fail(LTXATTN_ERR_SHAPE, "x has a negative stride");
  if (!(a->eps >= 0.0f)) return fail(LTXATTN_ERR_ARG, "eps must be non-negative");
  if ((rc = check_rotary(a->rotary, "rotary", s.Lq))) return rc;
  if ((rc = check_tensor(a->out, "out", s, false))) return rc;
  const bool bf16 = s.dtype == LTXATTN_BF16;
  QkPrepParams p{};
  p.x = a->x;
  p.x_sb = a->x_stride_b;
  p.x_st = a->x_stride_t;
  p.w = a->weight;
  p.eps = a->eps;
  p.cos = a->rotary.cos;
  p.sin = a->rotary.sin;
  p.t_sb = a->rotary.stride_b;
  p.t_sh = a->rotary.stride_h;
  p.t_st = a->rotary.stride_t;
  p.out = a->out.data;
  p.o_sb = a->out.stride_b;
  p.o_sh = a->out.stride_h;
  p.o_st = a->out.stride_t;
  p.B = s.B;
  p.tokens = s.Lq;
  p.inner = inner;
  p.D = s.D;
  const int64_t per16 = bf16 ? 8 : 4;  // elements per 16 bytes
  auto m8 = [per16](int64_t v) { return v % per16 == 0; };
  p.vec = aligned16(a->x) && m8(a->x_stride_b) && m8(a->x_stride_t) && aligned16(a->weight) &&
          aligned16(a->out.data) && m8(a->out.stride_b) && m8(a->out.stride_h) && m8(a->out.stride_t) &&
          (a->rotary.cos == nullptr || (aligned16(a->rotary.cos) && aligned16(a->rotary.sin) &&
                                        m8(a->rotary.stride_b) && m8(a->rotary.stride_h) && m8(a->rotary.stride_t)));
  p.err = device_error_word();
  *out = p;
  *is_bf16 = bf16;
  return LTXATTN_OK;
}

extern "C" {

int ltxattn_qk_prep(const ltxattn_qk_prep_args* a, void* stream) {
  QkPrepParams p;
  bool bf16 = false;
  const int rc = qk_prep_params(a, &p, &bf16);
  if (rc) return rc;
  const cudaError_t e = launch_qk_prep(p, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LTXATTN_OK : cuda_fail(e, "qk_prep launch");
}

int ltxattn_qk_prep_pair(const ltxattn_qk_prep_args* q, const ltxattn_qk_prep_args* k, void* stream) {
  QkPrepParams pq, pk;
  bool bq = false, bk = false;
  int rc = qk_prep_params(q, &pq, &bq);
  if (rc) return rc;
  if ((rc = qk_prep_params(k, &pk, &bk))) return rc;
  if (bq != bk) return fail(LTXATTN_ERR_DTYPE, "q and k preparations must share one dtype");
  if (pq.inner != pk.inner) return fail(LTXATTN_ERR_SHAPE, "q and k inner widths differ (%d, %d)", pq.inner, pk.inner);
  const cudaError_t e = launch_qk_prep_pair(pq, pk, bq, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LTXATTN_OK : cuda_fail(e, "qk_prep_pair launch");
}

int ltxattn_rotary_tables(const ltxattn_rotary_table_args* a, void* stream) {
  if (a == nullptr) return fail(LTXATTN_ERR_ARG, "args is NULL");
  if (a->dtype != LTXATTN_F32 && a->dtype != LTXATTN_BF16)
    return fail(LTXATTN_ERR_DTYPE, "dtype %d is neither LTXATTN_F32 nor LTXATTN_BF16", a->dtype);
  if (a->n_pos < 1 || a->n_pos > 4) return fail(LTXATTN_ERR_SHAPE, "n_pos %d is outside 1..4", a->n_pos);
  if (a->tokens < 0 || a->heads <= 0 || a->inner <= 0 || a->inner % (2 * a->heads))
    return fail(LTXATTN_ERR_SHAPE, "inner %d does not split into %d heads of rotary pairs", a->inner, a->heads);
  const int count = a->inner / (2 * a->n_pos);
  if (count < 2) return fail(LTXATTN_ERR_SHAPE, "inner %d gives fewer than 2 frequencies per dimension", a->inner);
  if (!(a->theta > 0.0)) return fail(LTXATTN_ERR_ARG, "theta must be positive");
  for (int d = 0; d < a->n_pos; ++d)
    if (!(a->max_pos[d] != 0.0f)) return fail(LTXATTN_ERR_ARG, "max_pos[%d] is zero", d);
  if (a->tokens > 0 && (a->positions == nullptr || a->cos == nullptr || a->sin == nullptr))
    return fail(LTXATTN_ERR_ARG, "positions, cos and sin must be device pointers");
  RotaryTableParams p{};
  p.positions = a->positions;
  p.cos = a->cos;
  p.sin = a->sin;
  p.theta = a->theta;
  for (int d = 0; d < 4; ++d) p.max_pos[d] = d < a->n_pos ? a->max_pos[d] : 1.0f;
  p.n_pos = a->n_pos;
  p.tokens = a->tokens;
  p.inner = a->inner;
  p.heads = a->heads;
  p.count = count;
  p.pad = a->inner / 2 - count * a->n_pos;
  const cudaError_t e = launch_rotary_tables(p, a->dtype == LTXATTN_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LTXATTN_OK : cuda_fail(e, "rotary tables launch");
}

int ltxattn_rope(const ltxattn_rope_args* a, void* stream) {
  if (a == nullptr) return fail(LTXATTN_ERR_ARG, "args is NULL");
  Shape s;
  int rc = check_shape(a->dtype, a->batch, a->heads, a->tokens, a->tokens, a->head_dim, 0, 0, &s);
  if (rc) return rc;
  if (a->rotary.cos == nullptr) return fail(LTXATTN_ERR_ARG, "rotary.cos is NULL");
  if ((rc = check_rotary(a->rotary, "rotary", s.Lq))) return rc;
  if ((rc = check_tensor(a->x, "x", s, false))) return rc;
  if ((rc = check_tensor(a->out, "out", s, false))) return rc;
  RopeParams p = rope_params(a->x, a->rotary, s, s.Lq, a->out.data);
  p.y_sb = a->out.stride_b;
  p.y_sh = a->out.stride_h;
  p.y_st = a->out.stride_t;
  const cudaError_t e = launch_rope(&p, nullptr, s.dtype == LTXATTN_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LTXATTN_OK : cuda_fail(e, "rope launch");
}

size_t ltxattn_bwd_workspace(const ltxattn_bwd_args* a) {
  BwdPlan P;
  if (plan_bwd(a, &P) != LTXATTN_OK) return 0;
  return P.total;
}

int ltxattn_bwd(const ltxattn_bwd_args* a, void* stream) {
  BwdPlan P;
  int rc = plan_bwd(a, &P);
  if (rc) return rc;
  const Shape& s = P.s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = s.dtype == LTXATTN_BF16;
  if ((rc = check_tensor(a->q, "q", s, bf16 && !P.rope))) return rc;
  if ((rc = check_tensor(a->k, "k", s, bf16 && !P.rope))) return rc;
  if ((rc = check_tensor(a->v, "v", s, bf16))) return rc;
  if ((rc = check_tensor(a->out, "out", s, false))) return rc;
  if ((rc = check_tensor(a->dout, "dout", s, bf16))) return rc;
  if ((rc = check_tensor(a->dq, "dq", s, bf16))) return rc;
  if ((rc = check_tensor(a->dk, "dk", s, bf16))) return rc;
  if ((rc = check_tensor(a->dv, "dv", s, bf16))) return rc;
  if (a->lse == nullptr) return fail(LTXATTN_ERR_ARG, "lse is NULL (the backward recomputes P from it)");
  if (a->workspace == nullptr || a->workspace_bytes < P.total)
    return fail(LTXATTN_ERR_WORKSPACE, "workspace of %zu bytes is needed, %zu given", P.total,
                a->workspace == nullptr ? (size_t)0 : a->workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
    return fail(LTXATTN_ERR_ALIGN, "workspace must be 256-byte aligned");
  int* err = device_error_word();
  if (!err) return fail(LTXATTN_ERR_CUDA, "no device error word (is a CUDA device current?)");
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  const size_t es = s.esize;
  const int64_t h0 = s.h0;
  // every view below is based at local head 0
  auto at = [&](const ltxattn_tensor& t) {
    return static_cast<const void*>(static_cast<const uint8_t*>(t.data) + h0 * t.stride_h * (int64_t)es);
  };
  ltxattn_tensor q = a->q, k = a->k;
  q.data = const_cast<void*>(at(a->q));
  k.data = const_cast<void*>(at(a->k));
  cudaError_t e;
  // every launch of this call is queued after all host work (no host gaps)
  RopeParams rope_q{}, rope_k{};
  if (P.rope) {
    rope_q = rope_params(a->q, a->q_rotary, s, s.Lq, ws + P.off_q);
    rope_k = rope_params(a->k, *P.kr, s, s.Lk, ws + P.off_k);
    q.data = ws + P.off_q;
    q.stride_t = s.D;
    q.stride_h = (int64_t)s.Lq * s.D;
    q.stride_b = (int64_t)s.Hc * s.Lq * s.D;
    k.data = ws + P.off_k;
    k.stride_t = s.D;
    k.stride_h = (int64_t)s.Lk * s.D;
    k.stride_b = (int64_t)s.Hc * s.Lk * s.D;
  }
  float* lse2 = reinterpret_cast<float*>(ws + P.off_l);
  float* delta = reinterpret_cast<float*>(ws + P.off_d);
  BwdPrepParams pp{};
  pp.o = at(a->out);
  pp.o_sb = a->out.stride_b; pp.o_sh = a->out.stride_h; pp.o_st = a->out.stride_t;
  pp.dout = at(a->dout);
  pp.do_sb = a->dout.stride_b; pp.do_sh = a->dout.stride_h; pp.do_st = a->dout.stride_t;
  pp.lse = a->lse + h0 * a->lse_stride_h;
  pp.lse_sb = a->lse_stride_b; pp.lse_sh = a->lse_stride_h;
  pp.lse2 = lse2;
  pp.delta = delta;
  pp.B = s.B; pp.Hc = s.Hc; pp.Lq = s.Lq; pp.Lq_pad = P.Lq_pad; pp.D = s.D;
  pp.log2_domain = bf16 ? 1 : 0;
  pp.f32 = bf16 ? 0 : 1;
  auto launch_pre = [&]() -> int {
    if (P.rope) {
      e = launch_rope(&rope_q, &rope_k, bf16, st);
      if (e != cudaSuccess) return cuda_fail(e, "rope launch");
    }
    e = launch_bwd_prep(pp, st);
    return e == cudaSuccess ? LTXATTN_OK : cuda_fail(e, "bwd prep launch");
  };

  BwdParams p{};
  p.lse2 = lse2;
  p.delta = delta;
  p.Lq_pad = P.Lq_pad;
  p.dq = const_cast<void*>(at(a->dq));
  p.dq_sb = a->dq.stride_b; p.dq_sh = a->dq.stride_h; p.dq_st = a->dq.stride_t;
  p.dk = const_cast<void*>(at(a->dk));
  p.dk_sb = a->dk.stride_b; p.dk_sh = a->dk.stride_h; p.dk_st = a->dk.stride_t;
  p.dv = const_cast<void*>(at(a->dv));
  p.dv_sb = a->dv.stride_b; p.dv_sh = a->dv.stride_h; p.dv_st = a->dv.stride_t;
  p.mask = a->key_mask;
  p.mask_sb = a->key_mask_stride_b;
  if (P.rope) {
    const ltxattn_rotary& qr = a->q_rotary;
    const ltxattn_rotary& kr = *P.kr;
    p.qcos = static_cast<const uint8_t*>(qr.cos) + h0 * qr.stride_h * (int64_t)es;
    p.qsin = static_cast<const uint8_t*>(qr.sin) + h0 * qr.stride_h * (int64_t)es;
    p.qt_sb = qr.stride_b; p.qt_sh = qr.stride_h; p.qt_st = qr.stride_t;
    p.kcos = static_cast<const uint8_t*>(kr.cos) + h0 * kr.stride_h * (int64_t)es;
    p.ksin = static_cast<const uint8_t*>(kr.sin) + h0 * kr.stride_h * (int64_t)es;
    p.kt_sb = kr.stride_b; p.kt_sh = kr.stride_h; p.kt_st = kr.stride_t;
    const int64_t per16 = 16 / (int64_t)es;  // elements per 16 bytes
    auto al = [&](const void* ptr) { return aligned16(ptr); };
    auto m = [&](int64_t st) { return st % per16 == 0; };
    p.rope_vec = al(p.qcos) && al(p.qsin) && al(p.kcos) && al(p.ksin) && m(qr.stride_b) && m(qr.stride_h) &&
                 m(qr.stride_t) && m(kr.stride_b) && m(kr.stride_h) && m(kr.stride_t);
  }
  p.Lq = s.Lq;
  p.Lk = s.Lk;
  p.n_q_tiles = P.Lq_pad / kTileM;
  p.n_kv_tiles = (s.Lk + kTileN - 1) / kTileN;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.err = err;
  if (!bf16) {
    p.q = static_cast<const float*>(q.data);
    p.q_sb = q.stride_b; p.q_sh = q.stride_h; p.q_st = q.stride_t;
    p.k = static_cast<const float*>(k.data);
    p.k_sb = k.stride_b; p.k_sh = k.stride_h; p.k_st = k.stride_t;
    p.v = static_cast<const float*>(at(a->v));
    p.v_sb = a->v.stride_b; p.v_sh = a->v.stride_h; p.v_st = a->v.stride_t;
    p.dout = static_cast<const float*>(at(a->dout));
    p.do_sb = a->dout.stride_b; p.do_sh = a->dout.stride_h; p.do_st = a->dout.stride_t;
    if ((rc = launch_pre())) return rc;
    e = launch_bwd_f32(p, s.D, s.Hc, s.B, st);
    if (e != cudaSuccess) return cuda_fail(e, "bwd_f32 launch");
    return LTXATTN_OK;
  }
  if ((rc = make_tmap(&p.tm_q, q.data, s.D, s.Lq, s.Hc, s.B, q.stride_t, q.stride_h, q.stride_b, "q"))) return rc;
  if ((rc = make_tmap(&p.tm_k, k.data, s.D, s.Lk, s.Hc, s.B, k.stride_t, k.stride_h, k.stride_b, "k"))) return rc;
  if ((rc = make_tmap(&p.tm_v, at(a->v), s.D, s.Lk, s.Hc, s.B, a->v.stride_t, a->v.stride_h, a->v.stride_b, "v")))
    return rc;
  if ((rc = make_tmap(&p.tm_do, at(a->dout), s.D, s.Lq, s.Hc, s.B, a->dout.stride_t, a->dout.stride_h,
                      a->dout.stride_b, "dout")))
    return rc;
  const bool has_mask = a->key_mask != nullptr;
  const size_t smem_dq = bwd_dq_smem_bytes(s.D, s.Lk, has_mask), smem_kv = bwd_dkdv_smem_bytes(s.D, s.Lk, has_mask);
  e = prepare_bwd_bf16(s.D, smem_dq, smem_kv);
  if (e != cudaSuccess) return cuda_fail(e, "bwd_bf16 setup");
  if ((rc = launch_pre())) return rc;
  e = launch_bwd_bf16(p, s.D, s.Hc, s.B, smem_dq, smem_kv, st);
  if (e != cudaSuccess) return cuda_fail(e, "bwd_bf16 launch");
  return LTXATTN_OK;
}

// ---------------------------------------------------------------------------
// device discovery and status

int ltxattn_device_count(int32_t* count) {
  if (!count) return fail(LTXATTN_ERR_ARG, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *count = n;
  return LTXATTN_OK;
}

int ltxattn_device_query(int32_t device, ltxattn_device_info* info) {
  if (!info) return fail(LTXATTN_ERR_ARG, "info is NULL");
  memset(info, 0, sizeof *info);
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  snprintf(info->name, sizeof info->name, "%s", prop.name);
  info->device = device;
  info->cc_major = prop.major;
  info->cc_minor = prop.minor;
  info->sm_count = prop.multiProcessorCount;
  info->total_memory_bytes = (int64_t)prop.totalGlobalMem;
  info->max_smem_per_block_optin = (int32_t)prop.sharedMemPerBlockOptin;
  info->l2_bytes = prop.l2CacheSize;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrClockRate, device) == cudaSuccess) info->sm_clock_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMemoryClockRate, device) == cudaSuccess) info->mem_clock_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrGlobalMemoryBusWidth, device) == cudaSuccess)
    info->mem_bus_width_bits = v;
  int prev = 0;
  if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(device) == cudaSuccess) {
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) info->free_memory_bytes = (int64_t)fr;
    cudaSetDevice(prev);
  }
  info->supported = (prop.major == 10 && prop.minor == 0) ? 1 : 0;
  return LTXATTN_OK;
}

int ltxattn_device_status(int32_t clear, int32_t* site) {
  int* w = device_error_word();
  if (!w) return fail(LTXATTN_ERR_CUDA, "no device error word");
  // every stream of the device, including non-blocking ones that a plain
  // cudaMemcpy would not wait for
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "synchronising the device");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (clear && v != 0) {
    const int z = 0;
    e = cudaMemcpy(w, &z, sizeof z, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  if (site) *site = v >> 8;
  if ((v & 0xff) == kErrTimeout)
    return fail(LTXATTN_ERR_TIMEOUT, "a kernel wait gave up (site %d)", v >> 8);
  return LTXATTN_OK;
}

}  // extern "C"
