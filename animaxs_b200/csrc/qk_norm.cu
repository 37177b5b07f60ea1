// qk_norm.cu -- per-(token, head) RMSNorm (+ split-half RoPE) for q and k.
//
// Replaces the reference's rmsnorm_heads_half (AnimaKernels.metal:660-689) and
// rms_rope_split_half (AnimaKernels.metal:696-729): fp32 statistics
// rsqrt(mean(x^2) + eps), a shared [128] weight, then the rotation
//   out[p]    = cos*a + (-sin)*b
//   out[p+64] = sin*a +   cos*b        (a = x[p]*inv*w[p], b = x[p+64]*inv*w[p+64])
// with the [token][64][2][2] table blocks [cos, -sin, sin, cos].
//
// HBM-bound (512 B of traffic per 128-element row).  8 lanes work on one row:
// lane l takes elements [8l, 8l+8) and [64+8l, 64+8l+8), i.e. both members of
// rotation pairs 8l..8l+7, so the rotation needs no data exchange and only the
// sum of squares is reduced (3 shuffles).  One CTA per (token, batch): its
// rows (the token's q heads, then its k heads) are dealt to row slots of 8
// lanes, four rows per slot, and every thread issues all of its loads before
// any math so that enough bytes are in flight to cover HBM latency (measured
// 4.9 TB/s on the fused DiT paths).  A lane's 8 rotation blocks are loaded once
// per token and reused by every head.  Results go out with 16-byte stores.
#include "kernels.h"
#include "sm100_ptx.cuh"

namespace ax {
namespace {

constexpr int kMaxNormThreads = 64;  // up to 8 row slots x 8 lanes
constexpr int kRowUnroll = 4;        // rows in flight per thread

__device__ __forceinline__ void norm_row(const uint4 ra, const uint4 rb, __half* dst,
                                         const __half* weight, float eps, bool rope,
                                         const float (&c)[8], const float (&ns)[8],
                                         const float (&sn)[8], int l8, unsigned mask) {
  float a[8], b[8];
  const __half2* ha = reinterpret_cast<const __half2*>(&ra);
  const __half2* hb = reinterpret_cast<const __half2*>(&rb);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fa = __half22float2(ha[i]);
    const float2 fb = __half22float2(hb[i]);
    a[2 * i] = fa.x;
    a[2 * i + 1] = fa.y;
    b[2 * i] = fb.x;
    b[2 * i + 1] = fb.y;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(b[i], b[i], fmaf(a[i], a[i], ss));
  ss += __shfl_xor_sync(mask, ss, 4);
  ss += __shfl_xor_sync(mask, ss, 2);
  ss += __shfl_xor_sync(mask, ss, 1);
  const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
  if (weight != nullptr) {
    const uint4 wa = *reinterpret_cast<const uint4*>(weight + l8 * 8);
    const uint4 wb = *reinterpret_cast<const uint4*>(weight + 64 + l8 * 8);
    const __half2* w2a = reinterpret_cast<const __half2*>(&wa);
    const __half2* w2b = reinterpret_cast<const __half2*>(&wb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __half22float2(w2a[i]);
      const float2 fb = __half22float2(w2b[i]);
      a[2 * i] *= inv * fa.x;
      a[2 * i + 1] *= inv * fa.y;
      b[2 * i] *= inv * fb.x;
      b[2 * i + 1] *= inv * fb.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] *= inv;
      b[i] *= inv;
    }
  }
  uint4 oa, ob;
  __half2* pa = reinterpret_cast<__half2*>(&oa);
  __half2* pb = reinterpret_cast<__half2*>(&ob);
  if (rope) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = 2 * i, f = 2 * i + 1;
      pa[i] = __floats2half2_rn(c[e] * a[e] + ns[e] * b[e], c[f] * a[f] + ns[f] * b[f]);
      pb[i] = __floats2half2_rn(sn[e] * a[e] + c[e] * b[e], sn[f] * a[f] + c[f] * b[f]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pa[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
      pb[i] = __floats2half2_rn(b[2 * i], b[2 * i + 1]);
    }
  }
  *reinterpret_cast<uint4*>(dst + l8 * 8) = oa;
  *reinterpret_cast<uint4*>(dst + 64 + l8 * 8) = ob;
}

__global__ void __launch_bounds__(kMaxNormThreads) qk_norm_kernel(const NormParams p) {
  const int tok = blockIdx.x;
  const int bb = blockIdx.y;
  const int slot = threadIdx.x >> 3;
  const int l8 = threadIdx.x & 7;
  const unsigned mask = 0xFFu << (threadIdx.x & 24);
  const bool rope = p.rope != nullptr;
  float c[8], ns[8], sn[8];
  if (rope) {
    const float4* tab = reinterpret_cast<const float4*>(p.rope) + static_cast<long long>(tok) * 64 + l8 * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) { const float4 blk = __ldg(tab + i); c[i] = blk.x; ns[i] = blk.y; sn[i] = blk.z; }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = ns[i] = sn[i] = 0.f;
  }
  const NormJob& J0 = p.job[0];
  const NormJob& J1 = p.job[1];
  const int r0 = (tok < J0.tokens && bb < J0.batch) ? J0.heads : 0;
  const int r1 = (p.njobs > 1 && tok < J1.tokens && bb < J1.batch) ? J1.heads : 0;
  const int rows = r0 + r1;
  const int kSlots = blockDim.x / 8;
  for (int base = 0; base < rows; base += kSlots * kRowUnroll) {
    uint4 ra[kRowUnroll], rb[kRowUnroll];
    __half* dst[kRowUnroll];
    const __half* w[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      const int r = base + slot + kSlots * u;
      dst[u] = nullptr; w[u] = nullptr;
      if (r < rows) {
        const bool second = r >= r0;
        const NormJob& J = second ? J1 : J0;
        const int head = second ? r - r0 : r;
        const __half* src = J.in + bb * J.in_batch + static_cast<long long>(tok) * J.in_tok + static_cast<long long>(head) * J.in_head;
        dst[u] = J.out + bb * J.out_batch + static_cast<long long>(tok) * J.out_tok + static_cast<long long>(head) * J.out_head;
        w[u] = J.weight;
        ra[u] = *reinterpret_cast<const uint4*>(src + l8 * 8);
        rb[u] = *reinterpret_cast<const uint4*>(src + 64 + l8 * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u)
      if (dst[u] != nullptr) norm_row(ra[u], rb[u], dst[u], w[u], p.eps, rope, c, ns, sn, l8, mask);
  }
}

}  // namespace

cudaError_t launch_qk_norm(NormParams p, cudaStream_t stream) {
  int tokens = 0, batch = 0, rows = 0;
  for (int i = 0; i < p.njobs; ++i) {
    tokens = max(tokens, p.job[i].tokens);
    batch = max(batch, p.job[i].batch);
    rows += p.job[i].heads;
  }
  if (tokens <= 0 || batch <= 0 || rows <= 0) return cudaSuccess;
  if (batch > 65535) return cudaErrorInvalidValue;
  // Enough 8-lane slots for kRowUnroll rows each, whole warps, at most 8 slots.
  int slots = (rows + kRowUnroll - 1) / kRowUnroll;
  slots = slots < 4 ? 4 : (slots > 8 ? 8 : slots);
  const int threads = slots * 8 <= 32 ? 32 : 64;
  qk_norm_kernel<<<dim3(tokens, batch), threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ax
