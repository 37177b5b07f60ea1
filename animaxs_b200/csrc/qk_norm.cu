// qk_norm.cu -- per-(token, head) RMSNorm (+ split-half RoPE) for q and k.
//
// Replaces the reference's rmsnorm_heads_half (AnimaKernels.metal:660-689) and
// rms_rope_split_half (AnimaKernels.metal:696-729): fp32 statistics
// rsqrt(mean(x^2) + eps), a shared [128] weight, then the rotation
//   out[p]    = cos*a + (-sin)*b
//   out[p+64] = sin*a +   cos*b        (a = x[p]*inv*w[p], b = x[p+64]*inv*w[p+64])
// with the [token][64][2][2] table blocks [cos, -sin, sin, cos].
//
// Layout: one 16-lane half-warp per row of 128 fp16 (256 B); each lane moves
// one 128-bit vector (8 halves).  The partner of pair p lives 8 lanes away, so
// the rotation is one shuffle.  Purely HBM-bound: 512 B of traffic per row.
#include "kernels.h"

namespace ax {
namespace {

__global__ void __launch_bounds__(256) qk_norm_kernel(const NormParams p) {
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long rowid = gid >> 4;
  const int l16 = threadIdx.x & 15;
  const unsigned mask = 0xFFFFu << (threadIdx.x & 16);
  const long long rows0 = p.job[0].rows;
  const long long total = rows0 + (p.njobs > 1 ? p.job[1].rows : 0);
  if (rowid >= total) return;  // uniform across the half-warp
  const bool second = rowid >= rows0;
  const NormJob& J = second ? p.job[1] : p.job[0];
  long long r = second ? rowid - rows0 : rowid;
  const int hh = static_cast<int>(r % J.heads);
  r /= J.heads;
  const int tok = static_cast<int>(r % J.tokens);
  const long long bb = r / J.tokens;

  const __half* src = J.in + bb * J.in_batch + static_cast<long long>(tok) * J.in_tok +
                      static_cast<long long>(hh) * J.in_head + l16 * 8;
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
  float x[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h2[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) ss += __shfl_xor_sync(mask, ss, off);
  const float inv = rsqrtf(ss * (1.0f / 128.0f) + p.eps);

  float a[8];
  if (J.weight != nullptr) {
    const uint4 wr = *reinterpret_cast<const uint4*>(J.weight + l16 * 8);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wr);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(w2[i]);
      a[2 * i] = x[2 * i] * inv * f.x;
      a[2 * i + 1] = x[2 * i + 1] * inv * f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = x[i] * inv;
  }

  float out[8];
  if (p.rope != nullptr) {
    const bool first_half = l16 < 8;
    const float4* tab = reinterpret_cast<const float4*>(p.rope) +
                        static_cast<long long>(tok) * 64 + (l16 & 7) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float partner = __shfl_xor_sync(mask, a[i], 8);
      const float4 blk = __ldg(tab + i);  // {cos, -sin, sin, cos}
      // first half: own = a (x[p]),  partner = b (x[p+64])
      // second half: own = b,        partner = a
      out[i] = first_half ? (blk.x * a[i] + blk.y * partner) : (blk.z * partner + blk.x * a[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = a[i];
  }

  uint4 res;
  __half2* r2 = reinterpret_cast<__half2*>(&res);
#pragma unroll
  for (int i = 0; i < 4; ++i) r2[i] = __floats2half2_rn(out[2 * i], out[2 * i + 1]);
  __half* dst = J.out + bb * J.out_batch + static_cast<long long>(tok) * J.out_tok +
                static_cast<long long>(hh) * J.out_head + l16 * 8;
  *reinterpret_cast<uint4*>(dst) = res;
}

}  // namespace

cudaError_t launch_qk_norm(const NormParams& p, cudaStream_t stream) {
  const long long total = p.job[0].rows + (p.njobs > 1 ? p.job[1].rows : 0);
  if (total <= 0) return cudaSuccess;
  const long long threads = total * 16;
  const long long blocks = (threads + 255) / 256;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  qk_norm_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ax
