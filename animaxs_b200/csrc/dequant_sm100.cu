// dequant_sm100.cu -- W8 / W4 projection weights decoded to fp16 in HBM.
//
// The reference keeps DiT / encoder weights as W8 or W4 codes with an fp16
// scale and zero per row and per 64 columns (scripts/pack_anima.py:217-296)
// and decodes them either into an fp16 buffer for the library GEMM
// (LinearExecutor.swift:153-189 -> dequant_w4_to_half / dequant_w8_to_half,
// AnimaKernels.metal:19-67) or inside its own quantized GEMM.  Here the decode
// is a separate HBM-bound pass (0.5 or 1 byte read + 2 bytes written per
// value) ahead of the tcgen05 projection GEMM: the weight is 2-6 % of a DiT
// projection's bytes and is read once per call, so fusing the decode into
// the GEMM's operand path would save well under the GEMM's own time.
//
// value = half(float(q) * float(scale) + float(zero)) with the multiply and
// the add rounded separately (no fused multiply-add), which is what the
// reference's decoders compute (scripts/animapk_cuda/quant.py:32-76).
//
// One thread per 16 consecutive columns of a row: 8 (W4) or 16 (W8) code
// bytes in one load, two 16-byte stores out.  A block covers whole rows (two
// rows of k = 2048 per block iteration, more when k is smaller), so no index
// division sits in the loop.  Rows whose packed start is not 8- / 16-byte
// aligned (odd k for W4, user strides) and the last partial chunk of a row go
// byte by byte.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "kernels.h"

namespace ax {
namespace {

constexpr int kThreads = 256;
constexpr int kCols = 16;  // columns per thread and chunk

// float(q) for 0 <= q < 2^23 without the int->float unit: 2^23 + q is exact in
// fp32 (the mantissa holds q), and subtracting 2^23 back is exact.
__device__ __forceinline__ float code_to_float(uint32_t q) {
  return __fsub_rn(__uint_as_float(0x4B000000u | q), 8388608.f);
}

__device__ __forceinline__ float decode_one(uint32_t q, float sc, float ze) {
  return __fadd_rn(__fmul_rn(code_to_float(q), sc), ze);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);  // each half rounded to nearest-even
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int kBits>
__global__ void __launch_bounds__(kThreads, 4) dequant_kernel(const uint8_t* __restrict__ packed,
                                                           const __half* __restrict__ scale,
                                                           const __half* __restrict__ zero,
                                                           __half* __restrict__ out, int rows, int k,
                                                           int64_t packed_stride, int64_t out_stride,
                                                           bool vec_out) {
  const int chunks = (k + kCols - 1) / kCols;
  const int groups = (k + 63) >> 6;
  // Rows per block iteration and this thread's (row, first chunk) in it.
  const int rpb = chunks >= kThreads ? 1 : kThreads / chunks;
  const int sub = chunks >= kThreads ? 0 : static_cast<int>(threadIdx.x) / chunks;
  const int c_first = chunks >= kThreads ? static_cast<int>(threadIdx.x) : static_cast<int>(threadIdx.x) - sub * chunks;
  const int c_step = chunks >= kThreads ? kThreads : chunks;
  if (sub >= rpb) return;
  constexpr int kLoadBytes = kCols * kBits / 8;  // 8 (W4) or 16 (W8)
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * rpb + sub; r < rows;
       r += static_cast<int64_t>(gridDim.x) * rpb) {
    const uint8_t* src_row = packed + r * packed_stride;
    __half* dst_row = out + r * out_stride;
    const bool vec_in = (reinterpret_cast<uintptr_t>(src_row) & (kLoadBytes - 1)) == 0;
    for (int c = c_first; c < chunks; c += c_step) {
      const int c0 = c * kCols;
      const int g = c0 >> 6;  // 16 columns never straddle a group of 64
      const float sc = __half2float(scale[r * groups + g]);
      const float ze = __half2float(zero[r * groups + g]);
      const uint8_t* src = src_row + c0 * kBits / 8;
      __half* dst = dst_row + c0;
      const int n = min(kCols, k - c0);
      if (n == kCols && vec_in) {
        uint32_t h[8];
        if (kBits == 4) {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // byte j: column 2j low nibble, 2j + 1 high nibble
            h[j] = pack2(decode_one((w.x >> (8 * j)) & 0xFu, sc, ze), decode_one((w.x >> (8 * j + 4)) & 0xFu, sc, ze));
            h[4 + j] = pack2(decode_one((w.y >> (8 * j)) & 0xFu, sc, ze), decode_one((w.y >> (8 * j + 4)) & 0xFu, sc, ze));
          }
        } else {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            h[2 * j] = pack2(decode_one(ws[j] & 0xFFu, sc, ze), decode_one((ws[j] >> 8) & 0xFFu, sc, ze));
            h[2 * j + 1] = pack2(decode_one((ws[j] >> 16) & 0xFFu, sc, ze), decode_one(ws[j] >> 24, sc, ze));
          }
        }
        if (vec_out) {
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(h[0], h[1], h[2], h[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(h[4], h[5], h[6], h[7]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            dst[2 * j] = __ushort_as_half(static_cast<unsigned short>(h[j] & 0xFFFFu));
            dst[2 * j + 1] = __ushort_as_half(static_cast<unsigned short>(h[j] >> 16));
          }
        }
      } else {
        for (int j = 0; j < n; ++j) {
          const uint32_t b = src[kBits == 4 ? j / 2 : j];
          dst[j] = __float2half_rn(decode_one(kBits == 4 ? ((b >> (4 * (j & 1))) & 0xFu) : b, sc, ze));
        }
      }
    }
  }
}

// The common case -- k a multiple of 8, every packed row 4- (W4) / 8-byte
// (W8) aligned, a 16-byte aligned output.  A thread owns one 8-column chunk
// (4 or 8 code bytes, one 16-byte store: a warp stores 512 contiguous bytes)
// in a grid-strided set of rows, and keeps the loads of the next kPrefetch
// rows in flight while it decodes and stores the current one, so warps
// overlap memory with arithmetic instead of moving through load, decode and
// store in lock step.
//
// Arithmetic: q * scale is exact in fp32 (8-bit code times an 11-bit fp16
// significand), so one fused multiply-add rounds exactly once, like the
// reference's rounded multiply then rounded add.  A code byte becomes the
// float 2^23 + q with one byte permute (the byte below the 0x4B exponent
// byte), then 2^23 is subtracted exactly.
constexpr int kPrefetch = 4;
constexpr int kColsAligned = 8;

__device__ __forceinline__ float byte_to_float(uint32_t word, int j) {
  // result bytes: [0] = word byte j, [1] = [2] = 0, [3] = 0x4B  ->  2^23 + byte
  return __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | static_cast<unsigned>(j))), 8388608.f);
}

template <int kBits>
__global__ void __launch_bounds__(kThreads, 5) dequant_aligned_kernel(const uint8_t* __restrict__ packed,
                                                                      const __half* __restrict__ scale,
                                                                      const __half* __restrict__ zero,
                                                                      __half* __restrict__ out, int rows, int k,
                                                                      int64_t packed_stride, int64_t out_stride) {
  using Codes = typename std::conditional<kBits == 4, uint32_t, uint2>::type;
  const int chunks = k / kColsAligned;
  const int groups = (k + 63) >> 6;
  const int rpb = chunks >= kThreads ? 1 : kThreads / chunks;
  const int sub = chunks >= kThreads ? 0 : static_cast<int>(threadIdx.x) / chunks;
  const int c_first = chunks >= kThreads ? static_cast<int>(threadIdx.x) : static_cast<int>(threadIdx.x) - sub * chunks;
  const int c_step = chunks >= kThreads ? kThreads : chunks;
  if (sub >= rpb) return;
  const int step = static_cast<int>(gridDim.x) * rpb;  // < 2^31: at most 5 x SMs x 256 rows
  const int first = static_cast<int>(blockIdx.x) * rpb + sub;
  if (first >= rows) return;
  // Row-to-row pointer increments (no per-row 64-bit multiplies).
  const int64_t code_delta = step * packed_stride;
  const int64_t sz_delta = static_cast<int64_t>(step) * groups;
  const int64_t out_delta = step * out_stride;
  for (int c = c_first; c < chunks; c += c_step) {
    const int c0 = c * kColsAligned;
    const uint8_t* lc = packed + first * packed_stride + c0 * kBits / 8;  // next row to load
    const __half* ls = scale + static_cast<int64_t>(first) * groups + (c0 >> 6);
    const __half* lz = zero + static_cast<int64_t>(first) * groups + (c0 >> 6);
    __half* dst = out + first * out_stride + c0;                         // next row to store
    Codes w[kPrefetch];
    __half sh[kPrefetch], zh[kPrefetch];
    int r_load = first;
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
      if (r_load < rows) {
        w[u] = __ldg(reinterpret_cast<const Codes*>(lc));
        sh[u] = ls[0];
        zh[u] = lz[0];
        lc += code_delta;
        ls += sz_delta;
        lz += sz_delta;
      }
      r_load += step;
    }
    for (int r = first; r < rows;) {
#pragma unroll
      for (int u = 0; u < kPrefetch; ++u) {
        if (r >= rows) break;
        const float sc = __half2float(sh[u]);
        const float ze = __half2float(zh[u]);
        uint32_t h[4];
        if constexpr (kBits == 4) {
          // byte j of the word: column 2j in the low nibble, 2j + 1 in the high
          const uint32_t lo = w[u] & 0x0F0F0F0Fu, hi = (w[u] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            h[j] = pack2(__fmaf_rn(byte_to_float(lo, j), sc, ze), __fmaf_rn(byte_to_float(hi, j), sc, ze));
        } else {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t wj = j == 0 ? w[u].x : w[u].y;
            h[2 * j] = pack2(__fmaf_rn(byte_to_float(wj, 0), sc, ze), __fmaf_rn(byte_to_float(wj, 1), sc, ze));
            h[2 * j + 1] = pack2(__fmaf_rn(byte_to_float(wj, 2), sc, ze), __fmaf_rn(byte_to_float(wj, 3), sc, ze));
          }
        }
        if (r_load < rows) {  // refill this slot kPrefetch rows ahead
          w[u] = __ldg(reinterpret_cast<const Codes*>(lc));
          sh[u] = ls[0];
          zh[u] = lz[0];
          lc += code_delta;
          ls += sz_delta;
          lz += sz_delta;
        }
        r_load += step;
        *reinterpret_cast<uint4*>(dst) = make_uint4(h[0], h[1], h[2], h[3]);
        dst += out_delta;
        r += step;
      }
    }
  }
}

}  // namespace

cudaError_t launch_dequant(int bits, const void* packed, const void* scale, const void* zero, void* out,
                           int rows, int k, int64_t packed_stride, int64_t out_stride, int sms,
                           cudaStream_t stream) {
  const int chunks = (k + kCols - 1) / kCols;
  const int rpb = chunks >= kThreads ? 1 : kThreads / chunks;
  // One block iteration per `rpb` rows; 4 blocks per SM (the residency the
  // launch bounds guarantee), the row loop grid-strided.
  const int64_t want = (static_cast<int64_t>(rows) + rpb - 1) / rpb;
  const int grid = static_cast<int>(want < static_cast<int64_t>(sms) * 4 ? want : static_cast<int64_t>(sms) * 4);
  const bool vec_out = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (out_stride % 8 == 0);
  const auto* p = static_cast<const uint8_t*>(packed);
  const auto* s = static_cast<const __half*>(scale);
  const auto* z = static_cast<const __half*>(zero);
  auto* o = static_cast<__half*>(out);
  const int64_t load_bytes = bits == 4 ? 4 : 8;
  // (row counters are 32-bit there: keep rows + the row step below 2^31)
  if (vec_out && k % kColsAligned == 0 && packed_stride % load_bytes == 0 &&
      reinterpret_cast<uintptr_t>(packed) % load_bytes == 0 && rows < (1 << 30)) {
    const int ac = k / kColsAligned;
    const int arpb = ac >= kThreads ? 1 : kThreads / ac;
    const int64_t slots = (static_cast<int64_t>(rows) + arpb - 1) / arpb;
    const int64_t cap = static_cast<int64_t>(sms) * 5;  // the residency the launch bounds give
    const int g2 = static_cast<int>(slots < cap ? slots : cap);
    if (bits == 4)
      dequant_aligned_kernel<4><<<g2, kThreads, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride);
    else
      dequant_aligned_kernel<8><<<g2, kThreads, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride);
    return cudaGetLastError();
  }
  if (bits == 4)
    dequant_kernel<4><<<grid, kThreads, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride, vec_out);
  else
    dequant_kernel<8><<<grid, kThreads, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride, vec_out);
  return cudaGetLastError();
}

}  // namespace ax
