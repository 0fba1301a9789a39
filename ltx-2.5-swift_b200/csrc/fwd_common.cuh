// fwd_common.cuh -- launch shape, constants and the UMMA issue helpers shared
// by the bf16 forward kernels (fwd_sm100.cu, fwd_short_sm100.cu).
#pragma once

#include "ltxattn_internal.h"
#include "sm100.cuh"

namespace ltx {
namespace {

constexpr int kThreads = 384;
constexpr uint32_t kLaunchRegs = 168;   // what ptxas allots under __launch_bounds__(384, 1)
constexpr uint32_t kProducerRegs = 88;
constexpr uint32_t kSoftmaxRegs = 208;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kProducerRegs <= kThreads * kLaunchRegs,
              "register re-split exceeds the launch allocation");
constexpr int kBlockM = kFwdBlockM;             // query rows per CTA (two Q tiles)
constexpr uint32_t kChunkBytes = 128u * 128u;  // one 64-element-wide chunk of a 128-row tile
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLn2 = 0.69314718055994530942f;

// S = Q K^T for one 128x128 tile: D/16 MMAs of K = 16.  qd / kd are base
// descriptors of the Q and K tiles; k-step kk sits in 64-wide chunk kk/4 at
// byte (kk%4)*32 of each 128-byte row.
template <int D>
__device__ __forceinline__ void issue_s(uint32_t tS, SDesc qd, SDesc kd) {
  constexpr uint32_t idesc = idesc_bf16_f32(128, 128, 0, 0);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = ((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4;
    umma_ss2(tS, qd.lo + off, qd.hi, kd.lo + off, kd.hi, idesc, kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V for one half of a tile (keys 64*half .. 64*half+63): 4 MMAs of
// K = 16 keys; P from TMEM (8 columns per k-step), V MN-major (16 keys = 16
// rows of 128 B; d-chunks kChunkBytes apart).
template <int D>
__device__ __forceinline__ void issue_pv_half(uint32_t tO, uint32_t tP, SDesc vd, bool accumulate, int half) {
  constexpr uint32_t idesc = idesc_bf16_f32(128, D, 0, 1);
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    const int kk = half * 4 + k4;
    umma_ts2(tO, tP + kk * 8, vd.lo + ((kk * 16 * 128) >> 4), vd.hi, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

}  // namespace
}  // namespace ltx
