/*
 * ltxattn_oracle.c -- CPU restatement of the LTX 2.5 DiT attention core.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
 * this file; only tests/, __graft_entry__.smoke() (as the checker) and the
 * bench's cpu_baseline / --impl reference leg use it.
 *
 * What it restates (paths relative to the loading-awesome/LTX-2.5-Swift tree):
 *
 *   Sources/LTXModules/DiTAttention.swift:369-382   SDPA core.  The `.explicit`
 *       arm is the arithmetic that is visible in the reference:
 *           logits  = (q . k^T) * scale          (fp32)
 *           weights = softmax(logits, axis: -1)  (fp32)
 *           out     = (weights . v) -> q.dtype
 *       with scale = 1/sqrt(dimHead) (:372).  The `.fused` arm calls MLX's
 *       flash kernel for the same function.
 *   Sources/LTXModules/DiTAttention.swift:206-234   split RoPE on contiguous
 *       halves; tables cast to the activation dtype; bf16 x bf16 products.
 *   Sources/LTXModules/GemmaTextEncoder.swift:292-323 and
 *   Sources/LTXFoundation/TextConditioningLayout.swift:98-107   mask semantics:
 *       additive mask, 0 for an allowed key and -FLT_MAX (not -inf) for a
 *       masked one; a row with no allowed key is un-masked entirely.
 *   Sources/LTXModules/GradientCheckpoint.swift:48-67 and
 *   Sources/LTXModules/LoRATrainingStep.swift:283-304   the backward is the
 *       autodiff VJP of the function above; restated here in closed form.
 *
 * Parity status: the reference (Swift + MLX on Metal) cannot run on this
 * machine or on the GPU box, so this restatement is pinned by (1) the
 * reference's own known-answer test MLXCapabilityTests.fusedAttention
 * (Tests/LTXModulesTests/MLXCapabilityTests.swift:78-91) and (2) golden
 * vectors produced by an independent fp64 implementation (torch, see
 * tests/golden/make_golden.py) of the same explicit-path formula.
 *
 * Layouts: every tensor is contiguous [B, H, T, D] float32; the key mask is
 * [B, Lk] uint8 (nonzero = valid); RoPE tables are [Hr, T, D/2] float32 with
 * an explicit head stride (0 = shared by all heads) and batch stride.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* bf16 round-to-nearest-even, the conversion MLX applies on asType(.bfloat16) */
static inline float bf16_round(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {          /* inf / nan pass through */
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        uint32_t r = ((u >> 16) & 1u) + 0x7fffu;
        u = (u + r) & 0xffff0000u;
    }
    float y;
    memcpy(&y, &u, 4);
    return y;
}

void oracle_round_bf16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = bf16_round(x[i]);
}

/* ------------------------------------------------------------------ */
/* Seeded inputs: splitmix64 (the generator of Sources/ltx/Bench.swift:479-493)
 * feeding Box-Muller in fp64.  Output i uses the i-th pair of draws, so the
 * stream is counter-based: element i depends only on (seed, i). */
static inline uint64_t splitmix64_at(uint64_t seed, uint64_t index) {
    uint64_t z = seed + 0x9E3779B97F4A7C15ull * (index + 1ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void oracle_fill_normal(uint64_t seed, int64_t n, float* out) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = 0; i < n; ++i) {
        uint64_t a = splitmix64_at(seed, 2ull * (uint64_t)i);
        uint64_t b = splitmix64_at(seed, 2ull * (uint64_t)i + 1ull);
        double u1 = ((double)(a >> 11) + 1.0) * 0x1.0p-53;   /* (0, 1] */
        double u2 = (double)(b >> 11) * 0x1.0p-53;           /* [0, 1) */
        out[i] = (float)(sqrt(-2.0 * log(u1)) * cos(two_pi * u2));
    }
}

/* ------------------------------------------------------------------ */
/* Split RoPE, DiTAttention.swift:226-234:
 *   out[:D/2] = x1*cos - x2*sin ;  out[D/2:] = x2*cos + x1*sin
 * In bf16 mode every elementwise op rounds to bf16, as MLX does for a bf16
 * tensor times a bf16 table (the tables are narrowed first, :231-232). */
int oracle_rope(float* x, const float* cosv, const float* sinv,
                 int B, int H, int T, int D,
                 int64_t tab_stride_b, int64_t tab_stride_h, int round_bf16) {
    const int half = D / 2;
    for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
    for (int t = 0; t < T; ++t) {
        float* row = x + (((int64_t)b * H + h) * T + t) * D;
        const float* c = cosv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
        const float* s = sinv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
        for (int i = 0; i < half; ++i) {
            float x1 = row[i], x2 = row[i + half];
            float cc = c[i], ss = s[i];
            if (round_bf16) {
                cc = bf16_round(cc); ss = bf16_round(ss);
                float a = bf16_round(x1 * cc), bb = bf16_round(x2 * ss);
                float e = bf16_round(x2 * cc), f = bf16_round(x1 * ss);
                row[i] = bf16_round(a - bb);
                row[i + half] = bf16_round(e + f);
            } else {
                row[i] = x1 * cc - x2 * ss;
                row[i + half] = x2 * cc + x1 * ss;
            }
        }
    }
    return 0;
}

/* q / k preparation, DiTAttention.swift:358-367: rmsNorm over the whole inner
 * dim (:190-204, MLX's kernel arithmetic: mean square, r = 1/sqrt(mean + eps),
 * y = T(w * T(x * r))), the head split (:346-348) and split RoPE (:206-234).
 * x: [B][T][H*D]; w: [H*D]; tables as oracle_rope ([Bt][Ht][T][D/2], cos NULL
 * for none); out: [B][H][T][D].  The mean square accumulates in fp64 here
 * (the device's fp32 tree sum may differ from it in the last ulp of r). */
int oracle_qk_prep(const float* x, const float* w, int B, int T, int H, int D, float eps,
                   const float* cosv, const float* sinv, int64_t tab_stride_b, int64_t tab_stride_h,
                   int round_bf16, float* out) {
    const int inner = H * D, half = D / 2;
    for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) {
        const float* xr = x + ((int64_t)b * T + t) * inner;
        double ss = 0.0;
        for (int i = 0; i < inner; ++i) ss += (double)xr[i] * (double)xr[i];
        const float r = (float)(1.0 / sqrt((double)(float)(ss / inner) + (double)eps));
        for (int h = 0; h < H; ++h) {
            float* o = out + (((int64_t)b * H + h) * T + t) * D;
            for (int d = 0; d < D; ++d) {
                float n = xr[h * D + d] * r;
                if (round_bf16) n = bf16_round(n);
                float y = w[h * D + d] * n;
                if (round_bf16) y = bf16_round(y);
                o[d] = y;
            }
            if (cosv) {
                const float* c = cosv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
                const float* sn = sinv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
                for (int i = 0; i < half; ++i) {
                    const float x1 = o[i], x2 = o[i + half];
                    float cc = c[i], ss2 = sn[i];
                    if (round_bf16) {
                        cc = bf16_round(cc); ss2 = bf16_round(ss2);
                        const float a = bf16_round(x1 * cc), bb = bf16_round(x2 * ss2);
                        const float e = bf16_round(x2 * cc), f = bf16_round(x1 * ss2);
                        o[i] = bf16_round(a - bb);
                        o[i + half] = bf16_round(e + f);
                    } else {
                        o[i] = x1 * cc - x2 * ss2;
                        o[i + half] = x2 * cc + x1 * ss2;
                    }
                }
            }
        }
    }
    return 0;
}

/* Rotary tables, DiTForward.rotary (DiTForward.swift:641-678) with
 * frequencyGrid (:455-466):
 *   freq[i] = (float)(theta^(i/(count-1)) * pi/2), count = inner/(2*n_pos),
 *             the exponent and power in fp64 (the last exponent is exactly 1);
 *   middle  = (lo + hi) / 2 and frac = middle / max_pos[d], fp32;
 *   angle   = freq[i] * (frac*2 - 1), fp32, positional dimension fastest
 *             (column i*n_pos + d), after `pad` leading identity pairs
 *             (cos 1, sin 0) that fill inner/2;
 *   cos/sin in fp32, split per head: out[h][t][c] = table[t][h*per + c].
 * positions: [n_pos][tokens][2] (lo, hi).  Outputs [heads][tokens][per]. */
int oracle_rotary_tables(const float* positions, const float* max_pos, int n_pos, int tokens,
                         int inner, int heads, double theta, float* cos_out, float* sin_out) {
    const int count = inner / (2 * n_pos);
    const int half = inner / 2;
    const int pad = half - count * n_pos;
    const int per = half / heads;
    if (count < 2 || pad < 0 || half % heads) return 1;
    float* freq = (float*)malloc(sizeof(float) * (size_t)count);
    if (!freq) return 2;
    const double step = 1.0 / (double)(count - 1);
    for (int i = 0; i < count; ++i) {
        const double e = (i == count - 1) ? 1.0 : (double)i * step;
        freq[i] = (float)(pow(theta, e) * 3.14159265358979323846 / 2.0);
    }
    for (int t = 0; t < tokens; ++t) {
        for (int j = 0; j < half; ++j) {
            float c = 1.0f, sn = 0.0f;
            if (j >= pad) {
                const int k = j - pad, i = k / n_pos, d = k % n_pos;
                const float lo = positions[((int64_t)d * tokens + t) * 2];
                const float hi = positions[((int64_t)d * tokens + t) * 2 + 1];
                const float middle = (lo + hi) / 2.0f;
                const float frac = middle / max_pos[d];
                const float ang = freq[i] * (frac * 2.0f - 1.0f);
                c = cosf(ang);
                sn = sinf(ang);
            }
            const int64_t o = ((int64_t)(j / per) * tokens + t) * per + (j % per);
            cos_out[o] = c;
            sin_out[o] = sn;
        }
    }
    free(freq);
    return 0;
}

/* Transpose of the rotation, for gradients w.r.t. the un-rotated input
 * (the VJP treats the bf16 roundings as identity, as autodiff does). */
int oracle_rope_bwd(float* dx, const float* cosv, const float* sinv,
                     int B, int H, int T, int D,
                     int64_t tab_stride_b, int64_t tab_stride_h, int round_tables_bf16) {
    const int half = D / 2;
    for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
    for (int t = 0; t < T; ++t) {
        float* row = dx + (((int64_t)b * H + h) * T + t) * D;
        const float* c = cosv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
        const float* s = sinv + b * tab_stride_b + h * tab_stride_h + (int64_t)t * half;
        for (int i = 0; i < half; ++i) {
            double cc = round_tables_bf16 ? bf16_round(c[i]) : c[i];
            double ss = round_tables_bf16 ? bf16_round(s[i]) : s[i];
            double g1 = row[i], g2 = row[i + half];
            row[i] = (float)(g1 * cc + g2 * ss);
            row[i + half] = (float)(g2 * cc - g1 * ss);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Which keys a batch row may attend to.  Masked keys take an additive
 * -FLT_MAX; in fp32 that absorbs any finite logit, so after the max
 * subtraction their weight is exactly zero whenever one key is allowed.
 * A batch whose mask allows no key is un-masked (GemmaTextEncoder.swift:306-319). */
static void allowed_keys(const uint8_t* mask, int64_t mask_stride_b, int b, int Lk,
                         unsigned char* allowed) {
    int any = 0;
    for (int j = 0; j < Lk; ++j) {
        allowed[j] = mask ? (mask[b * mask_stride_b + j] != 0) : 1;
        any |= allowed[j];
    }
    if (!any)
        for (int j = 0; j < Lk; ++j) allowed[j] = 1;
}

/* Self-attention of the Gemma text encoder (GemmaTextEncoder.swift:218-233,
 * 292-323): query i may attend key j when j <= i (causal), i - j < window (a
 * sliding layer, window > 0) and key j is not padding; a query row left with
 * no such key attends every key instead (the reference's un-masking of fully
 * masked rows).  Grouped KV heads: query head h reads KV head h / (Hq / Hkv).
 * q [B][Hq][L][D], k / v [B][Hkv][L][D], valid [B][L] (NULL: all valid);
 * fp64 accumulation; lse natural-log over the attended keys. */
int oracle_attn_fwd_gemma(const float* q, const float* k, const float* v, const uint8_t* valid,
                          int B, int Hq, int Hkv, int L, int D, double scale, int causal, int window,
                          float* out, float* lse) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || L <= 0 || D <= 0) return 1;
    const int group = Hq / Hkv;
    double* logit = (double*)malloc(sizeof(double) * (size_t)L);
    unsigned char* allow = (unsigned char*)malloc((size_t)L);
    if (!logit || !allow) { free(logit); free(allow); return 2; }
    for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h)
    for (int i = 0; i < L; ++i) {
        int any = 0;
        for (int j = 0; j < L; ++j) {
            int ok = valid ? (valid[(int64_t)b * L + j] != 0) : 1;
            if (causal && j > i) ok = 0;
            if (window > 0 && i - j >= window) ok = 0;
            allow[j] = (unsigned char)ok;
            any |= ok;
        }
        if (!any) memset(allow, 1, (size_t)L);
        const float* qr = q + (((int64_t)b * Hq + h) * L + i) * D;
        const float* kh = k + ((int64_t)b * Hkv + h / group) * L * D;
        const float* vh = v + ((int64_t)b * Hkv + h / group) * L * D;
        double mx = -INFINITY;
        for (int j = 0; j < L; ++j) {
            if (!allow[j]) { logit[j] = -INFINITY; continue; }
            double sdot = 0.0;
            for (int d = 0; d < D; ++d) sdot += (double)qr[d] * (double)kh[(int64_t)j * D + d];
            logit[j] = sdot * scale;
            if (logit[j] > mx) mx = logit[j];
        }
        double sum = 0.0;
        for (int j = 0; j < L; ++j) {
            logit[j] = allow[j] ? exp(logit[j] - mx) : 0.0;
            sum += logit[j];
        }
        float* o = out + (((int64_t)b * Hq + h) * L + i) * D;
        for (int d = 0; d < D; ++d) {
            double acc = 0.0;
            for (int j = 0; j < L; ++j) acc += logit[j] * (double)vh[(int64_t)j * D + d];
            o[d] = (float)(acc / sum);
        }
        if (lse) lse[((int64_t)b * Hq + h) * L + i] = (float)(mx + log(sum));
    }
    free(logit);
    free(allow);
    return 0;
}

/* Forward, fp64 accumulation (the parity oracle).  lse is the natural-log
 * log-sum-exp of the scaled logits over allowed keys, [B, H, Lq]. */
int oracle_attn_fwd(const float* q, const float* k, const float* v,
                    const uint8_t* mask, int64_t mask_stride_b,
                    int B, int H, int Lq, int Lk, int D, double scale,
                    float* out, float* lse, int threads) {
    if (B <= 0 || H <= 0 || Lq < 0 || Lk <= 0 || D <= 0) return 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    int64_t rows = (int64_t)B * H * Lq;
#pragma omp parallel
    {
        double* logit = (double*)malloc(sizeof(double) * Lk);
        double* acc = (double*)malloc(sizeof(double) * D);
        unsigned char* allowed = (unsigned char*)malloc(Lk);
        int last_b = -1;
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            int b = (int)(r / ((int64_t)H * Lq));
            int h = (int)((r / Lq) % H);
            if (b != last_b) { allowed_keys(mask, mask_stride_b, b, Lk, allowed); last_b = b; }
            const float* qr = q + r * D;
            const float* kh = k + ((int64_t)b * H + h) * Lk * D;
            const float* vh = v + ((int64_t)b * H + h) * Lk * D;
            double mx = -INFINITY;
            for (int j = 0; j < Lk; ++j) {
                if (!allowed[j]) { logit[j] = -INFINITY; continue; }
                double s = 0.0;
                for (int d = 0; d < D; ++d) s += (double)qr[d] * (double)kh[(int64_t)j * D + d];
                logit[j] = s * scale;
                if (logit[j] > mx) mx = logit[j];
            }
            double sum = 0.0;
            for (int d = 0; d < D; ++d) acc[d] = 0.0;
            for (int j = 0; j < Lk; ++j) {
                if (!allowed[j]) continue;
                double p = exp(logit[j] - mx);
                sum += p;
                for (int d = 0; d < D; ++d) acc[d] += p * (double)vh[(int64_t)j * D + d];
            }
            for (int d = 0; d < D; ++d) out[r * D + d] = (float)(acc[d] / sum);
            if (lse) lse[r] = (float)(mx + log(sum));
        }
        free(logit); free(acc); free(allowed);
    }
    return 0;
}

/* Forward in fp32 arithmetic: the reference's explicit arm as written
 * (fp32 logits, fp32 softmax, fp32 PV), blocked over query rows so that the
 * [rows, Lk] logit block stays in cache.  This is the timed CPU baseline.
 * Key-major loops let the compiler vectorise over D and over keys. */
int oracle_attn_fwd_f32(const float* q, const float* k, const float* v,
                        const uint8_t* mask, int64_t mask_stride_b,
                        int B, int H, int Lq, int Lk, int D, float scale,
                        float* out, float* lse, int threads) {
    if (B <= 0 || H <= 0 || Lq < 0 || Lk <= 0 || D <= 0) return 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    enum { QB = 32 };
    int nqb = (Lq + QB - 1) / QB;
    int64_t units = (int64_t)B * H * nqb;
#pragma omp parallel
    {
        float* logit = (float*)malloc(sizeof(float) * (size_t)QB * Lk);
        float* acc = (float*)malloc(sizeof(float) * (size_t)QB * D);
        unsigned char* allowed = (unsigned char*)malloc(Lk);
        int last_b = -1;
#pragma omp for schedule(dynamic, 1)
        for (int64_t u = 0; u < units; ++u) {
            int b = (int)(u / ((int64_t)H * nqb));
            int h = (int)((u / nqb) % H);
            int q0 = (int)(u % nqb) * QB;
            int nq = Lq - q0 < QB ? Lq - q0 : QB;
            if (b != last_b) { allowed_keys(mask, mask_stride_b, b, Lk, allowed); last_b = b; }
            const float* qh = q + (((int64_t)b * H + h) * Lq + q0) * D;
            const float* kh = k + ((int64_t)b * H + h) * Lk * D;
            const float* vh = v + ((int64_t)b * H + h) * Lk * D;
            for (int i = 0; i < nq; ++i) {
                const float* qr = qh + (int64_t)i * D;
                float* lr = logit + (int64_t)i * Lk;
                for (int j = 0; j < Lk; ++j) {
                    const float* kr = kh + (int64_t)j * D;
                    float s = 0.f;
                    for (int d = 0; d < D; ++d) s += qr[d] * kr[d];
                    lr[j] = allowed[j] ? s * scale : -INFINITY;
                }
                float mx = -INFINITY;
                for (int j = 0; j < Lk; ++j) mx = lr[j] > mx ? lr[j] : mx;
                float sum = 0.f;
                for (int j = 0; j < Lk; ++j) { float p = expf(lr[j] - mx); lr[j] = p; sum += p; }
                float inv = 1.f / sum;
                for (int j = 0; j < Lk; ++j) lr[j] *= inv;
                if (lse) lse[((int64_t)b * H + h) * Lq + q0 + i] = mx + logf(sum);
                float* ar = acc + (int64_t)i * D;
                for (int d = 0; d < D; ++d) ar[d] = 0.f;
                for (int j = 0; j < Lk; ++j) {
                    float p = lr[j];
                    const float* vr = vh + (int64_t)j * D;
                    for (int d = 0; d < D; ++d) ar[d] += p * vr[d];
                }
                float* orow = out + (((int64_t)b * H + h) * Lq + q0 + i) * D;
                for (int d = 0; d < D; ++d) orow[d] = ar[d];
            }
        }
        free(logit); free(acc); free(allowed);
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Backward of out = softmax(scale * q k^T + mask) v, fp64 accumulation.
 * Closed form of the VJP MLX's autodiff applies (LoRATrainingStep.swift:283):
 *   P  = softmax(...)           dV = P^T dO
 *   dP = dO V^T                 dS = P o (dP - rowsum(P o dP))
 *   dQ = scale dS K             dK = scale dS^T Q
 * q and k here are the tensors that entered the SDPA (already rotated). */
int oracle_attn_bwd(const float* q, const float* k, const float* v,
                    const uint8_t* mask, int64_t mask_stride_b, const float* dout,
                    int B, int H, int Lq, int Lk, int D, double scale,
                    float* dq, float* dk, float* dv, int threads) {
    if (B <= 0 || H <= 0 || Lq < 0 || Lk <= 0 || D <= 0) return 1;
    if (D > 256) return 3; /* per-row accumulators are sized for D <= 256 */
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    double* P = (double*)malloc(sizeof(double) * (size_t)Lq * Lk);
    double* dS = (double*)malloc(sizeof(double) * (size_t)Lq * Lk);
    unsigned char* allowed = (unsigned char*)malloc(Lk);
    if (!P || !dS || !allowed) { free(P); free(dS); free(allowed); return 2; }
    enum { KB = 16 };
    for (int b = 0; b < B; ++b) {
        allowed_keys(mask, mask_stride_b, b, Lk, allowed);
        for (int h = 0; h < H; ++h) {
            const int64_t bh = (int64_t)b * H + h;
            const float* qh = q + bh * Lq * D;
            const float* kh = k + bh * Lk * D;
            const float* vh = v + bh * Lk * D;
            const float* doh = dout + bh * Lq * D;
            /* rows: P = softmax, dS = P o (dP - rowsum(P o dP)), dQ = scale dS K */
#pragma omp parallel for schedule(static)
            for (int i = 0; i < Lq; ++i) {
                double* pr = P + (int64_t)i * Lk;
                double* dsr = dS + (int64_t)i * Lk;
                const float* qi = qh + (int64_t)i * D;
                const float* gi = doh + (int64_t)i * D;
                double mx = -INFINITY;
                for (int j = 0; j < Lk; ++j) {
                    if (!allowed[j]) { pr[j] = -INFINITY; continue; }
                    double s = 0.0;
                    for (int d = 0; d < D; ++d) s += (double)qi[d] * kh[(int64_t)j * D + d];
                    pr[j] = s * scale;
                    if (pr[j] > mx) mx = pr[j];
                }
                double sum = 0.0;
                for (int j = 0; j < Lk; ++j) { pr[j] = allowed[j] ? exp(pr[j] - mx) : 0.0; sum += pr[j]; }
                double delta = 0.0;
                for (int j = 0; j < Lk; ++j) {
                    pr[j] /= sum;
                    double dp = 0.0;
                    for (int d = 0; d < D; ++d) dp += (double)gi[d] * vh[(int64_t)j * D + d];
                    dsr[j] = dp;
                    delta += pr[j] * dp;
                }
                for (int j = 0; j < Lk; ++j) dsr[j] = pr[j] * (dsr[j] - delta);
                double acc[256];
                for (int d = 0; d < D; ++d) acc[d] = 0.0;
                for (int j = 0; j < Lk; ++j) {
                    const double g = dsr[j];
                    if (g == 0.0) continue;
                    for (int d = 0; d < D; ++d) acc[d] += g * kh[(int64_t)j * D + d];
                }
                for (int d = 0; d < D; ++d) dq[bh * Lq * D + (int64_t)i * D + d] = (float)(scale * acc[d]);
            }
            /* key blocks: dK = scale dS^T Q, dV = P^T dO */
            const int nkb = (Lk + KB - 1) / KB;
#pragma omp parallel for schedule(dynamic, 1)
            for (int kb = 0; kb < nkb; ++kb) {
                const int j0 = kb * KB, j1 = j0 + KB < Lk ? j0 + KB : Lk;
                double ak[KB][256], av[KB][256];
                for (int jj = 0; jj < j1 - j0; ++jj)
                    for (int d = 0; d < D; ++d) ak[jj][d] = av[jj][d] = 0.0;
                for (int i = 0; i < Lq; ++i) {
                    const float* qi = qh + (int64_t)i * D;
                    const float* gi = doh + (int64_t)i * D;
                    for (int j = j0; j < j1; ++j) {
                        const double g = dS[(int64_t)i * Lk + j], pj = P[(int64_t)i * Lk + j];
                        if (g == 0.0 && pj == 0.0) continue;
                        for (int d = 0; d < D; ++d) {
                            ak[j - j0][d] += g * qi[d];
                            av[j - j0][d] += pj * gi[d];
                        }
                    }
                }
                for (int j = j0; j < j1; ++j)
                    for (int d = 0; d < D; ++d) {
                        dk[bh * Lk * D + (int64_t)j * D + d] = (float)(scale * ak[j - j0][d]);
                        dv[bh * Lk * D + (int64_t)j * D + d] = (float)av[j - j0][d];
                    }
            }
        }
    }
    free(P); free(dS); free(allowed);
    return 0;
}

/* dK and dV of selected keys of one unmasked head, streaming over the query rows
 * so that no Lq x Lk matrix is held (the 29,760-token configuration's P would
 * take 7 GB).  The same closed-form VJP as oracle_attn_bwd, with the row terms
 * supplied by the caller from a forward of the same head:
 *     P_ij = exp(scale * q_i.k_j - lse_i),   lse_i the natural log-sum-exp
 *     delta_i = sum_d dout_id * out_id       (= sum_j P_ij dP_ij)
 *     dV_j = sum_i P_ij dout_i,   dK_j = scale sum_i P_ij (dout_i.v_j - delta_i) q_i
 * q, dout [Lq, D]; k, v [Lk, D]; keys[n_keys] the key indices; dk, dv [n_keys, D].
 * fp64 accumulation. */
int oracle_attn_bwd_keys(const float* q, const float* k, const float* v, const float* dout,
                         const float* lse, const float* delta, int Lq, int Lk, int D, double scale,
                         const int* keys, int n_keys, float* dk, float* dv, int threads) {
    if (Lq <= 0 || Lk <= 0 || D <= 0 || n_keys < 0) return 1;
    if (D > 256) return 3;
    for (int n = 0; n < n_keys; ++n)
        if (keys[n] < 0 || keys[n] >= Lk) return 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#pragma omp parallel for schedule(dynamic, 1)
    for (int n = 0; n < n_keys; ++n) {
        const float* kj = k + (int64_t)keys[n] * D;
        const float* vj = v + (int64_t)keys[n] * D;
        double ak[256], av[256];
        for (int d = 0; d < D; ++d) ak[d] = av[d] = 0.0;
        for (int i = 0; i < Lq; ++i) {
            const float* qi = q + (int64_t)i * D;
            const float* gi = dout + (int64_t)i * D;
            double s = 0.0, dp = 0.0;
            for (int d = 0; d < D; ++d) {
                s += (double)qi[d] * kj[d];
                dp += (double)gi[d] * vj[d];
            }
            const double p = exp(s * scale - (double)lse[i]);
            const double ds = p * (dp - (double)delta[i]);
            for (int d = 0; d < D; ++d) {
                ak[d] += ds * qi[d];
                av[d] += p * gi[d];
            }
        }
        for (int d = 0; d < D; ++d) {
            dk[(int64_t)n * D + d] = (float)(scale * ak[d]);
            dv[(int64_t)n * D + d] = (float)av[d];
        }
    }
    return 0;
}

int oracle_abi_version(void) { return 1; }
