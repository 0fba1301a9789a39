/*
 * abi_host.c -- calls libltxattn_cuda the way a Swift (or any C) host does:
 * through include/ltxattn.h alone, with device memory from the CUDA runtime,
 * no Python and no torch.  Built and run by tests/test_c_host_gpu.py.
 *
 * One bf16 self-attention call with split RoPE and the log-sum-exp
 * (ltxattn_fwd, the SDPA of DiTAttention.swift:369-382 with the RoPE of
 * :364-367), then its backward (ltxattn_bwd, the VJP of
 * LoRATrainingStep.swift:283-304), on operands drawn from the reference
 * bench's splitmix64 stream (Sources/ltx/Bench.swift:479-493).  Every input
 * and output goes to the file named by argv[1]; the test recomputes them with
 * the CPU oracle.  Exit status 0 only if every call returned LTXATTN_OK and the
 * device error word is clean.
 *
 * File layout: "LTXA", int32 B, H, T, D, then bf16 arrays q, k, v, cos, sin,
 * out, float32 lse, bf16 dout, dq, dk, dv (all [B, H, T, D] contiguous; the
 * tables [T, D/2]; lse [B, H, T]).
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ltxattn.h"

#define CHECK_CUDA(x)                                                                          \
  do {                                                                                         \
    cudaError_t e_ = (x);                                                                      \
    if (e_ != cudaSuccess) {                                                                   \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_));       \
      return 2;                                                                                \
    }                                                                                          \
  } while (0)

#define CHECK_LTX(x)                                                                           \
  do {                                                                                         \
    int r_ = (x);                                                                              \
    if (r_ != LTXATTN_OK) {                                                                    \
      fprintf(stderr, "%s:%d %s -> %d: %s\n", __FILE__, __LINE__, #x, r_, ltxattn_last_error()); \
      return 3;                                                                                \
    }                                                                                          \
  } while (0)

static uint16_t bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* the reference bench's operands: uniform in [-1, 1), rounded to bf16 */
static void bench_bits(uint64_t seed, size_t n, uint16_t* out) {
  uint64_t state = seed + 0x9E3779B97F4A7C15ull;
  for (size_t i = 0; i < n; ++i) {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float unit = (float)(z >> 40) / (float)(1u << 24);
    out[i] = bf16_bits((unit - 0.5f) * 2.0f);
  }
}

static ltxattn_tensor view(void* p, int H, int T, int D) {
  ltxattn_tensor t;
  t.data = p;
  t.stride_b = (int64_t)H * T * D;
  t.stride_h = (int64_t)T * D;
  t.stride_t = D;
  return t;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s out.bin\n", argv[0]);
    return 1;
  }
  const int B = 1, H = 2, T = 200, D = 128;
  const size_t n = (size_t)B * H * T * D, nt = (size_t)T * (D / 2), nl = (size_t)B * H * T;

  int32_t count = 0;
  CHECK_LTX(ltxattn_device_count(&count));
  if (count < 1) {
    fprintf(stderr, "no CUDA device\n");
    return 4;
  }
  ltxattn_device_info info;
  CHECK_LTX(ltxattn_device_query(0, &info));
  fprintf(stderr, "device 0: %s, sm_%d%d, %d SMs, supported %d\n", info.name, info.cc_major, info.cc_minor,
          info.sm_count, info.supported);
  CHECK_CUDA(cudaSetDevice(0));

  uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * (4 * n + 2 * nt));
  uint16_t *hq = h, *hk = h + n, *hv = h + 2 * n, *hdo = h + 3 * n, *hc = h + 4 * n, *hs = hc + nt;
  bench_bits(0x5EED + 2, n, hq);
  bench_bits(0x5EED + 3, n, hk);
  bench_bits(0x5EED + 4, n, hv);
  bench_bits(0x5EED + 5, n, hdo);
  for (int t = 0; t < T; ++t)
    for (int j = 0; j < D / 2; ++j) {
      const double ang = t * pow(10000.0, -(double)j / (D / 2));
      hc[t * (D / 2) + j] = bf16_bits((float)cos(ang));
      hs[t * (D / 2) + j] = bf16_bits((float)sin(ang));
    }

  void *q, *k, *v, *dout, *out, *dq, *dk, *dv, *cs, *sn;
  float* lse;
  CHECK_CUDA(cudaMalloc(&q, 2 * n));
  CHECK_CUDA(cudaMalloc(&k, 2 * n));
  CHECK_CUDA(cudaMalloc(&v, 2 * n));
  CHECK_CUDA(cudaMalloc(&dout, 2 * n));
  CHECK_CUDA(cudaMalloc(&out, 2 * n));
  CHECK_CUDA(cudaMalloc(&dq, 2 * n));
  CHECK_CUDA(cudaMalloc(&dk, 2 * n));
  CHECK_CUDA(cudaMalloc(&dv, 2 * n));
  CHECK_CUDA(cudaMalloc(&cs, 2 * nt));
  CHECK_CUDA(cudaMalloc(&sn, 2 * nt));
  CHECK_CUDA(cudaMalloc((void**)&lse, 4 * nl));
  CHECK_CUDA(cudaMemcpy(q, hq, 2 * n, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(k, hk, 2 * n, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(v, hv, 2 * n, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dout, hdo, 2 * n, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(cs, hc, 2 * nt, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(sn, hs, 2 * nt, cudaMemcpyHostToDevice));
  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

  ltxattn_rotary rot;
  memset(&rot, 0, sizeof rot);
  rot.cos = cs;
  rot.sin = sn;
  rot.stride_b = 0;
  rot.stride_h = 0;
  rot.stride_t = D / 2;
  rot.tokens = T;

  /* forward: q and k rotated with the same table (keyRotary ?? rotary) */
  ltxattn_fwd_args fa;
  memset(&fa, 0, sizeof fa);
  fa.dtype = LTXATTN_BF16;
  fa.batch = B;
  fa.heads = H;
  fa.q_len = T;
  fa.kv_len = T;
  fa.head_dim = D;
  fa.q = view(q, H, T, D);
  fa.k = view(k, H, T, D);
  fa.v = view(v, H, T, D);
  fa.out = view(out, H, T, D);
  fa.scale = 1.0f / sqrtf((float)D);
  fa.q_rotary = rot;
  fa.lse = lse;
  fa.lse_stride_b = (int64_t)H * T;
  fa.lse_stride_h = T;
  void* fws = NULL;
  fa.workspace_bytes = ltxattn_fwd_workspace(&fa);
  if (fa.workspace_bytes) CHECK_CUDA(cudaMalloc(&fws, fa.workspace_bytes));
  fa.workspace = fws;
  CHECK_LTX(ltxattn_fwd(&fa, stream));

  /* backward of the same call */
  ltxattn_bwd_args ba;
  memset(&ba, 0, sizeof ba);
  ba.dtype = LTXATTN_BF16;
  ba.batch = B;
  ba.heads = H;
  ba.q_len = T;
  ba.kv_len = T;
  ba.head_dim = D;
  ba.q = fa.q;
  ba.k = fa.k;
  ba.v = fa.v;
  ba.out = fa.out;
  ba.dout = view(dout, H, T, D);
  ba.lse = lse;
  ba.lse_stride_b = fa.lse_stride_b;
  ba.lse_stride_h = fa.lse_stride_h;
  ba.dq = view(dq, H, T, D);
  ba.dk = view(dk, H, T, D);
  ba.dv = view(dv, H, T, D);
  ba.scale = fa.scale;
  ba.q_rotary = rot;
  void* bws = NULL;
  ba.workspace_bytes = ltxattn_bwd_workspace(&ba);
  if (ba.workspace_bytes) CHECK_CUDA(cudaMalloc(&bws, ba.workspace_bytes));
  ba.workspace = bws;
  CHECK_LTX(ltxattn_bwd(&ba, stream));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  int32_t site = 0;
  CHECK_LTX(ltxattn_device_status(1, &site));

  uint16_t* r = (uint16_t*)malloc(2 * n * 4);
  float* hl = (float*)malloc(4 * nl);
  CHECK_CUDA(cudaMemcpy(r, out, 2 * n, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(r + n, dq, 2 * n, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(r + 2 * n, dk, 2 * n, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(r + 3 * n, dv, 2 * n, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hl, lse, 4 * nl, cudaMemcpyDeviceToHost));

  FILE* f = fopen(argv[1], "wb");
  if (!f) return 5;
  const int32_t dims[4] = {B, H, T, D};
  fwrite("LTXA", 1, 4, f);
  fwrite(dims, 4, 4, f);
  fwrite(hq, 2, n, f);
  fwrite(hk, 2, n, f);
  fwrite(hv, 2, n, f);
  fwrite(hc, 2, nt, f);
  fwrite(hs, 2, nt, f);
  fwrite(r, 2, n, f);         /* out */
  fwrite(hl, 4, nl, f);       /* lse */
  fwrite(hdo, 2, n, f);       /* dout */
  fwrite(r + n, 2, 3 * n, f); /* dq, dk, dv */
  fclose(f);

  cudaFree(q); cudaFree(k); cudaFree(v); cudaFree(dout); cudaFree(out); cudaFree(dq); cudaFree(dk);
  cudaFree(dv); cudaFree(cs); cudaFree(sn); cudaFree(lse); cudaFree(fws); cudaFree(bws);
  cudaStreamDestroy(stream);
  free(h); free(r); free(hl);
  return 0;
}
