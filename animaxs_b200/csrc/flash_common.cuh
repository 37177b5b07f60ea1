// flash_common.cuh -- pieces shared by the two flash-attention kernels
// (attn_fwd_sm100.cu: head_dim 64/128; attn_wide_sm100.cu: head_dim 256/384):
// shared-memory operand descriptors for 128-row tiles stored as 64-column
// SW128 panels, the lazy-rescale threshold and the FMA-pipe exp2.
#pragma once

#include "kernels.h"
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


// ---- MMA issue for 128-row tiles (attn_fwd_sm100.cu, attn_s3_sm100.cu) ----
constexpr uint32_t kIdescQKTile = idesc_f16_f32(128, 128, false);  // B = K tile, K-major
template <int HD>
constexpr uint32_t kIdescPVTile = idesc_f16_f32(128, HD, true);     // B = V tile, MN-major, N = HD

// Descriptors advance by constant offsets of their start-address field
// (bits 0-13, address >> 4; every operand lies below 256 KiB of shared memory,
// so the field never carries).  The loops are unrolled and run on the whole MMA
// warp (one elected lane issues): the issue rate sits on the critical path.
template <int HD>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_tile, uint32_t k_tile) {
  const uint64_t a0 = kmajor_desc(q_tile, 0), b0 = kmajor_desc(k_tile, 0);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4);
    umma_f16_ss_warp(d_tmem, a0 + off, b0 + off, kIdescQKTile, kk > 0 ? 1u : 0u);
  }
}
// Half `hf` of O (+)= P V: k-steps 4*hf .. 4*hf+3 (keys [64*hf, 64*hf+64)).
// kFp32P: P is held as P_hi (columns [0, 64) of the S tile) plus P_lo
// (columns [64, 128)) and both are multiplied into the same accumulator.
template <int HD, bool kFp32P>
__device__ __forceinline__ void issue_pv_half(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_tile,
                                              int hf, bool accumulate) {
  const uint64_t b0 = vmajor_desc(v_tile, 0);
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    const int kk = hf * 4 + k4;
    umma_f16_ts_warp(d_tmem, p_tmem + kk * 8, b0 + static_cast<uint64_t>((kk * 2048) >> 4), kIdescPVTile<HD>,
                (accumulate || kk > 0) ? 1u : 0u);
  }
  if constexpr (kFp32P) {
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      const int kk = hf * 4 + k4;
      umma_f16_ts_warp(d_tmem, p_tmem + 64 + kk * 8, b0 + static_cast<uint64_t>((kk * 2048) >> 4),
                       kIdescPVTile<HD>, 1u);
    }
  }
}

__device__ __forceinline__ int kv_tiles_for(int tile_q0, int q_len, int valid, int causal) {
  if (tile_q0 >= q_len) return 0;
  int e = valid;
  if (causal) e = min(e, tile_q0 + kTileM);
  return (e + kTileN - 1) / kTileN;
}

}  // namespace ax
