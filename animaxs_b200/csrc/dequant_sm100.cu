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
// One thread per 8 consecutive columns of a row: 4 (W4) or 8 (W8) code bytes
// in, one 16-byte store out; a warp covers 256 columns, so loads and stores are
// contiguous.  Rows whose packed start is not 4- / 8-byte aligned (odd k for
// W4, user strides) and the last partial chunk of a row go byte by byte.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace ax {
namespace {

__device__ __forceinline__ __half decode_one(uint32_t q, float sc, float ze) {
  return __float2half_rn(__fadd_rn(__fmul_rn(static_cast<float>(q), sc), ze));
}

template <int kBits>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ packed,
                                                      const __half* __restrict__ scale,
                                                      const __half* __restrict__ zero,
                                                      __half* __restrict__ out, int rows, int k,
                                                      int64_t packed_stride, int64_t out_stride,
                                                      bool vec_out) {
  const int chunks = (k + 7) >> 3;
  const int groups = (k + 63) >> 6;
  const int64_t total = static_cast<int64_t>(rows) * chunks;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(t / chunks);
    const int c0 = static_cast<int>(t - static_cast<int64_t>(r) * chunks) * 8;
    const int g = c0 >> 6;  // 8 columns never straddle a group of 64
    const float sc = __half2float(scale[static_cast<int64_t>(r) * groups + g]);
    const float ze = __half2float(zero[static_cast<int64_t>(r) * groups + g]);
    const uint8_t* src = packed + static_cast<int64_t>(r) * packed_stride + (kBits == 4 ? c0 / 2 : c0);
    __half* dst = out + static_cast<int64_t>(r) * out_stride + c0;
    const int n = min(8, k - c0);
    __align__(16) __half v[8];
    if (n == 8 && (reinterpret_cast<uintptr_t>(src) & (kBits == 4 ? 3 : 7)) == 0) {
      if (kBits == 4) {
        const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(src));
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = decode_one((w >> (4 * j)) & 0xFu, sc, ze);
      } else {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = decode_one((w.x >> (8 * j)) & 0xFFu, sc, ze);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[4 + j] = decode_one((w.y >> (8 * j)) & 0xFFu, sc, ze);
      }
    } else {
      for (int j = 0; j < n; ++j) {
        const uint32_t b = src[kBits == 4 ? j / 2 : j];
        v[j] = decode_one(kBits == 4 ? ((b >> (4 * (j & 1))) & 0xFu) : b, sc, ze);
      }
    }
    if (n == 8 && vec_out) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
    } else {
      for (int j = 0; j < n; ++j) dst[j] = v[j];
    }
  }
}

}  // namespace

cudaError_t launch_dequant(int bits, const void* packed, const void* scale, const void* zero, void* out,
                           int rows, int k, int64_t packed_stride, int64_t out_stride, int sms,
                           cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(rows) * ((k + 7) / 8);
  // Enough 256-thread blocks for 8 per SM (the whole GPU busy), fewer for
  // small matrices; the loop is grid-strided.
  const int64_t want = (total + 255) / 256;
  const int grid = static_cast<int>(want < static_cast<int64_t>(sms) * 8 ? want : static_cast<int64_t>(sms) * 8);
  const bool vec_out = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (out_stride % 8 == 0);
  const auto* p = static_cast<const uint8_t*>(packed);
  const auto* s = static_cast<const __half*>(scale);
  const auto* z = static_cast<const __half*>(zero);
  auto* o = static_cast<__half*>(out);
  if (bits == 4)
    dequant_kernel<4><<<grid, 256, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride, vec_out);
  else
    dequant_kernel<8><<<grid, 256, 0, stream>>>(p, s, z, o, rows, k, packed_stride, out_stride, vec_out);
  return cudaGetLastError();
}

}  // namespace ax
