// flash_common.cuh -- pieces shared by the two flash-attention kernels
// (attn_fwd_sm100.cu: head_dim 64/128; attn_wide_sm100.cu: head_dim 256/384):
// shared-memory operand descriptors for 128-row tiles stored as 64-column
// SW128 panels, the lazy-rescale threshold and the FMA-pipe exp2.
#pragma once

#include "sm100_ptx.cuh"

namespace ax {

constexpr uint32_t kPanelBytes = 128 * 128;  // 128 rows x 128 B (64 fp16)
constexpr float kRescaleThreshold = 8.0f;     // log2 units: O is rescaled when max grows > 2^8
// Of every 8 adjacent column pairs, this many take exp2 on the FMA pipe
// (polynomial) and the rest on the MUFU pipe.
#ifndef AX_POLY_PAIRS
#define AX_POLY_PAIRS 2
#endif
constexpr int kPolyPairsPer8 = AX_POLY_PAIRS;

// 2^x on the FMA pipe for a pair of values.  Range reduction x = j + f with
// j = round(x) obtained by adding 1.5*2^23 (the integer lands in the low
// mantissa bits), f in [-1/2, 1/2]; 2^f by a degree-4 minimax polynomial
// (relative error 3.6e-6, coefficients from gen_exp2_poly.py); 2^j by adding
// j to the exponent field.  x is clamped at -126 so the result stays normal;
// masked entries (-inf) come out as 2^-126, which is 0 once stored as fp16
// and negligible in the fp32 row sum.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = add2(x, make_float2(kMagic, kMagic));
  const float2 j = add2(t, make_float2(-kMagic, -kMagic));
  const float2 f = add2(x, make_float2(-j.x, -j.y));
  float2 p = fma2(make_float2(0.009782912209630013f, 0.009782912209630013f), f,
                  make_float2(0.055976882576942444f, 0.055976882576942444f));
  p = fma2(p, f, make_float2(0.24020710587501526f, 0.24020710587501526f));
  p = fma2(p, f, make_float2(0.6931136250495911f, 0.6931136250495911f));
  p = fma2(p, f, make_float2(1.0f, 1.0f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// K-major operand (rows x 128 fp16 as two 64-column SW128 panels): k-step kk
// (16 columns) starts in panel kk/4 at byte (kk%4)*32.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk) {
  return sw128_desc(tile + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
}
// MN-major V operand: k-step kk covers keys [16kk, 16kk+16) = 2 groups of 8
// rows (1024 B apart); the two 64-wide head_dim panels are kPanelBytes apart.
__device__ __forceinline__ uint64_t vmajor_desc(uint32_t tile, int kk) {
  return sw128_desc(tile + kk * 2048, kPanelBytes, 1024);
}

}  // namespace ax
