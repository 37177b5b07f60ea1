// qk_norm.cu -- per-(token, head) RMSNorm (+ split-half RoPE) for q and k.
//
// Replaces the reference's rmsnorm_heads_half (AnimaKernels.metal:660-689) and
// rms_rope_split_half (AnimaKernels.metal:696-729): fp32 statistics
// rsqrt(mean(x^2) + eps), a shared [128] weight, then the rotation
//   out[p]    = cos*a + (-sin)*b
//   out[p+64] = sin*a +   cos*b        (a = x[p]*inv*w[p], b = x[p+64]*inv*w[p+64])
// with the [token][64][2][2] table blocks [cos, -sin, sin, cos].
//
// Layout: one CTA per (token, batch); one 16-lane half-warp per head row of 128
// fp16 (256 B), one 128-bit vector per lane.  The partner of pair p lives 8
// lanes away (one shuffle).  A lane's RoPE coefficients (8 pairs) are loaded
// once and reused for every head of the token, q and k alike.  HBM-bound:
// 512 B of traffic per row.
#include "kernels.h"

namespace ax {
namespace {

constexpr int kNormThreads = 128;

__device__ __forceinline__ void norm_row(uint4 raw, __half* dst, const __half* weight, float eps,
                                         bool rope, const float (&c)[8], const float (&ns)[8],
                                         const float (&sn)[8], int l16, unsigned mask) {
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
  const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
  float a[8];
  if (weight != nullptr) {
    const uint4 wr = *reinterpret_cast<const uint4*>(weight + l16 * 8);
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
  if (rope) {
    const bool first_half = l16 < 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float partner = __shfl_xor_sync(mask, a[i], 8);
      // first half: own = a (x[p]), partner = b (x[p+64]); second half: own = b, partner = a
      out[i] = first_half ? (c[i] * a[i] + ns[i] * partner) : (sn[i] * partner + c[i] * a[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = a[i];
  }
  uint4 res;
  __half2* r2 = reinterpret_cast<__half2*>(&res);
#pragma unroll
  for (int i = 0; i < 4; ++i) r2[i] = __floats2half2_rn(out[2 * i], out[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = res;
}

// One CTA per (token, batch).  The token's rows -- every q head, then every k
// head -- are dealt to the 8 half-warps four at a time; a half-warp issues its
// four 128-bit loads before doing any math so that enough bytes are in flight
// to cover HBM latency.
__global__ void __launch_bounds__(kNormThreads) qk_norm_kernel(const NormParams p) {
  const int tok = blockIdx.x;
  const int bb = blockIdx.y;
  const int hw = threadIdx.x >> 4;
  const int l16 = threadIdx.x & 15;
  const unsigned mask = 0xFFFFu << (threadIdx.x & 16);
  const bool rope = p.rope != nullptr;
  float c[8], ns[8], sn[8];
  if (rope) {
    const float4* tab = reinterpret_cast<const float4*>(p.rope) +
                        static_cast<long long>(tok) * 64 + (l16 & 7) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 blk = __ldg(tab + i);  // {cos, -sin, sin, cos}
      c[i] = blk.x;
      ns[i] = blk.y;
      sn[i] = blk.z;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = ns[i] = sn[i] = 0.f;
  }
  const NormJob& J0 = p.job[0];
  const NormJob& J1 = p.job[1];
  const int r0 = (tok < J0.tokens && bb < J0.batch) ? J0.heads : 0;
  const int r1 = (p.njobs > 1 && tok < J1.tokens && bb < J1.batch) ? J1.heads : 0;
  const int rows = r0 + r1;
  constexpr int kHalfWarps = kNormThreads / 16;
  constexpr int kUnroll = 4;
  for (int base = 0; base < rows; base += kHalfWarps * kUnroll) {
    uint4 raw[kUnroll];
    __half* dst[kUnroll];
    const __half* w[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int r = base + hw + kHalfWarps * u;
      dst[u] = nullptr;
      w[u] = nullptr;
      if (r < rows) {
        const bool second = r >= r0;
        const NormJob& J = second ? J1 : J0;
        const int head = second ? r - r0 : r;
        const __half* src = J.in + bb * J.in_batch + static_cast<long long>(tok) * J.in_tok +
                            static_cast<long long>(head) * J.in_head + l16 * 8;
        dst[u] = J.out + bb * J.out_batch + static_cast<long long>(tok) * J.out_tok +
                 static_cast<long long>(head) * J.out_head + l16 * 8;
        w[u] = J.weight;
        raw[u] = *reinterpret_cast<const uint4*>(src);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (dst[u] != nullptr) norm_row(raw[u], dst[u], w[u], p.eps, rope, c, ns, sn, l16, mask);
  }
}

}  // namespace

cudaError_t launch_qk_norm(const NormParams& p, cudaStream_t stream) {
  int tokens = 0, batch = 0;
  for (int i = 0; i < p.njobs; ++i) {
    tokens = max(tokens, p.job[i].tokens);
    batch = max(batch, p.job[i].batch);
  }
  if (tokens <= 0 || batch <= 0) return cudaSuccess;
  if (batch > 65535) return cudaErrorInvalidValue;
  qk_norm_kernel<<<dim3(tokens, batch), kNormThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ax
