// qk_norm.cu -- per-(token, head) RMSNorm (+ split-half RoPE) for q and k.
//
// Replaces the reference's rmsnorm_heads_half (AnimaKernels.metal:660-689),
// rms_rope_split_half (AnimaKernels.metal:696-729) and, at head_dim 64, the LLM
// adapter's rms_rope_adapter64 (AnimaKernels.metal:733-763): fp32 statistics
// rsqrt(mean(x^2) + eps), a shared [head_dim] weight, then the rotation of the
// pairs (p, p + D/2), D = head_dim:
//   out[p]     = cos*a + (-sin)*b
//   out[p+D/2] = sin*a +   cos*b        (a = x[p]*inv*w[p], b = x[p+D/2]*inv*w[p+D/2])
// with the [token][D/2][2][2] table blocks [cos, -sin, sin, cos].
//
// 4*D bytes of HBM traffic per row.  8 lanes work on one row: lane l takes
// E = D/16 elements [E*l, E*l+E) and [D/2+E*l, D/2+E*l+E), i.e. both members
// of rotation pairs E*l..E*l+E-1, so the rotation needs no data exchange and
// only the sum of squares is reduced (3 shuffles).  One CTA per (token,
// batch): its rows (the token's q heads, then its k heads) are dealt to row
// slots of 8 lanes, four rows per slot, and every thread issues all of its
// loads before any math so that enough bytes are in flight to cover HBM
// latency.  The kernel is bound by L1 requests and issue slots rather than
// DRAM, so it keeps those down: a lane's E rotation blocks are loaded once per
// token, a quarter by each of the warp's 4 row slots and the rest passed by
// shuffle; the two jobs' weights are loaded once per thread; the weight and
// rotation products run as packed f32x2 instructions (per-element IEEE
// results as the scalar forms, with the same fused multiply-add contraction).
// Measured 4.8 TB/s for the fused DiT self-attention prologue, 5.4 TB/s for
// the cross-attention one.
#include "kernels.h"
#include "sm100_ptx.cuh"

namespace ax {
namespace {

constexpr int kMaxNormThreads = 64;  // up to 8 row slots x 8 lanes
constexpr int kRowUnroll = 4;        // rows in flight per thread

// E = HD/16 consecutive fp16 of each half of a row: one lane's share.
template <int E>
struct Chunk {
  uint32_t w[E / 2];
};
template <int E>
__device__ __forceinline__ Chunk<E> load_chunk(const __half* p) {
  Chunk<E> c;
  if constexpr (E == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    c.w[0] = v.x; c.w[1] = v.y; c.w[2] = v.z; c.w[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    c.w[0] = v.x; c.w[1] = v.y;
  }
  return c;
}
template <int E>
__device__ __forceinline__ void store_chunk(__half* p, const Chunk<E>& c) {
  if constexpr (E == 8) {
    *reinterpret_cast<uint4*>(p) = make_uint4(c.w[0], c.w[1], c.w[2], c.w[3]);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(c.w[0], c.w[1]);
  }
}

template <int HD>
__device__ __forceinline__ void norm_row(const Chunk<HD / 16> ra, const Chunk<HD / 16> rb, __half* dst,
                                         bool has_w, const Chunk<HD / 16>& wa, const Chunk<HD / 16>& wb,
                                         float eps, bool rope,
                                         const float (&c)[HD / 16], const float (&ns)[HD / 16],
                                         const float (&sn)[HD / 16], int l8, unsigned mask) {
  constexpr int E = HD / 16;
  constexpr int H2 = HD / 2;
  float a[E], b[E];
#pragma unroll
  for (int i = 0; i < E / 2; ++i) {
    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&ra.w[i]));
    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&rb.w[i]));
    a[2 * i] = fa.x;
    a[2 * i + 1] = fa.y;
    b[2 * i] = fb.x;
    b[2 * i + 1] = fb.y;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss = fmaf(b[i], b[i], fmaf(a[i], a[i], ss));
  ss += __shfl_xor_sync(mask, ss, 4);
  ss += __shfl_xor_sync(mask, ss, 2);
  ss += __shfl_xor_sync(mask, ss, 1);
  const float inv = rsqrtf(ss * (1.0f / HD) + eps);
  if (has_w) {
    const float2 inv2 = make_float2(inv, inv);
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&wa.w[i]));
      const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&wb.w[i]));
      // a *= inv * w, two elements per instruction
      const float2 xa = mul2(make_float2(a[2 * i], a[2 * i + 1]), mul2(inv2, fa));
      const float2 xb = mul2(make_float2(b[2 * i], b[2 * i + 1]), mul2(inv2, fb));
      a[2 * i] = xa.x;
      a[2 * i + 1] = xa.y;
      b[2 * i] = xb.x;
      b[2 * i + 1] = xb.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      a[i] *= inv;
      b[i] *= inv;
    }
  }
  Chunk<E> oa, ob;
  if (rope) {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const int e = 2 * i, f = 2 * i + 1;
      // x = fma(cos, a, -sin * b), y = fma(sin, a, cos * b)
      const float2 A = make_float2(a[e], a[f]), B = make_float2(b[e], b[f]), C = make_float2(c[e], c[f]);
      const float2 X = fma2(C, A, mul2(make_float2(ns[e], ns[f]), B));
      const float2 Y = fma2(make_float2(sn[e], sn[f]), A, mul2(C, B));
      __half2 x = __floats2half2_rn(X.x, X.y);
      __half2 y = __floats2half2_rn(Y.x, Y.y);
      oa.w[i] = *reinterpret_cast<uint32_t*>(&x);
      ob.w[i] = *reinterpret_cast<uint32_t*>(&y);
    }
  } else {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      __half2 x = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
      __half2 y = __floats2half2_rn(b[2 * i], b[2 * i + 1]);
      oa.w[i] = *reinterpret_cast<uint32_t*>(&x);
      ob.w[i] = *reinterpret_cast<uint32_t*>(&y);
    }
  }
  store_chunk<E>(dst + l8 * E, oa);
  store_chunk<E>(dst + H2 + l8 * E, ob);
}

template <int HD>
__global__ void __launch_bounds__(kMaxNormThreads) qk_norm_kernel(const NormParams p) {
  constexpr int E = HD / 16;
  constexpr int H2 = HD / 2;
  const int tok = blockIdx.x;
  const int bb = blockIdx.y;
  const int slot = threadIdx.x >> 3;
  const int l8 = threadIdx.x & 7;
  const unsigned mask = 0xFFu << (threadIdx.x & 24);
  const bool rope = p.rope != nullptr;
  float c[E], ns[E], sn[E];
  if (rope) {
    // The 4 row slots of a warp need the same blocks: slot s loads blocks
    // [E/4 s, E/4 (s+1)) of its lane's E and the others come by shuffle.
    const float4* tab = reinterpret_cast<const float4*>(p.rope) + static_cast<long long>(tok) * H2 + l8 * E;
    constexpr int Q = E / 4;
    const int s4 = (threadIdx.x >> 3) & 3;
    float4 mine[Q];
#pragma unroll
    for (int i = 0; i < Q; ++i) mine[i] = __ldg(tab + s4 * Q + i);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int src = (threadIdx.x & 7) + 8 * (i / Q);
      c[i] = __shfl_sync(0xffffffffu, mine[i % Q].x, src);
      ns[i] = __shfl_sync(0xffffffffu, mine[i % Q].y, src);
      sn[i] = __shfl_sync(0xffffffffu, mine[i % Q].z, src);
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) c[i] = ns[i] = sn[i] = 0.f;
  }
  const NormJob& J0 = p.job[0];
  const NormJob& J1 = p.job[1];
  Chunk<E> wa0{}, wb0{}, wa1{}, wb1{};
  const bool hw0 = J0.weight != nullptr;
  const bool hw1 = p.njobs > 1 && J1.weight != nullptr;
  if (hw0) {
    wa0 = load_chunk<E>(J0.weight + l8 * E);
    wb0 = load_chunk<E>(J0.weight + H2 + l8 * E);
  }
  if (hw1) {
    wa1 = load_chunk<E>(J1.weight + l8 * E);
    wb1 = load_chunk<E>(J1.weight + H2 + l8 * E);
  }
  const int r0 = (tok < J0.tokens && bb < J0.batch) ? J0.heads : 0;
  const int r1 = (p.njobs > 1 && tok < J1.tokens && bb < J1.batch) ? J1.heads : 0;
  const int rows = r0 + r1;
  const int kSlots = blockDim.x / 8;
  for (int base = 0; base < rows; base += kSlots * kRowUnroll) {
    Chunk<E> ra[kRowUnroll], rb[kRowUnroll];
    __half* dst[kRowUnroll];
    bool sec[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      const int r = base + slot + kSlots * u;
      dst[u] = nullptr; sec[u] = false;
      if (r < rows) {
        const bool second = r >= r0;
        const NormJob& J = second ? J1 : J0;
        const int head = second ? r - r0 : r;
        const __half* src = J.in + bb * J.in_batch + static_cast<long long>(tok) * J.in_tok + static_cast<long long>(head) * J.in_head;
        dst[u] = J.out + bb * J.out_batch + static_cast<long long>(tok) * J.out_tok + static_cast<long long>(head) * J.out_head;
        sec[u] = second;
        ra[u] = load_chunk<E>(src + l8 * E);
        rb[u] = load_chunk<E>(src + H2 + l8 * E);
      }
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u)
      if (dst[u] != nullptr) {
        if (sec[u])
          norm_row<HD>(ra[u], rb[u], dst[u], hw1, wa1, wb1, p.eps, rope, c, ns, sn, l8, mask);
        else
          norm_row<HD>(ra[u], rb[u], dst[u], hw0, wa0, wb0, p.eps, rope, c, ns, sn, l8, mask);
      }
  }
}

}  // namespace

cudaError_t launch_qk_norm(NormParams p, cudaStream_t stream) {
  int tokens = 0, batch = 0, rows_all = 0, rows = 0;
  for (int i = 0; i < p.njobs; ++i) {
    tokens = max(tokens, p.job[i].tokens);
    batch = max(batch, p.job[i].batch);
    rows_all += p.job[i].heads;
  }
  if (tokens <= 0 || batch <= 0 || rows_all <= 0) return cudaSuccess;
  // Rows of the typical CTA: the jobs that cover every (token, batch).  A job
  // with fewer tokens (cross-attention's 512-token k beside 4096 q tokens)
  // adds rows to its CTAs only, which then take a second round of row slots,
  // instead of halving the rows in flight of all the others.
  for (int i = 0; i < p.njobs; ++i)
    if (p.job[i].tokens == tokens && p.job[i].batch == batch) rows += p.job[i].heads;
  if (rows == 0) rows = rows_all;
  if (batch > 65535) return cudaErrorInvalidValue;
  // Enough 8-lane slots for kRowUnroll rows each, whole warps, at most 8 slots.
  int slots = (rows + kRowUnroll - 1) / kRowUnroll;
  slots = slots < 4 ? 4 : (slots > 8 ? 8 : slots);
  const int threads = slots * 8 <= 32 ? 32 : 64;
  if (p.head_dim == 128)
    qk_norm_kernel<128><<<dim3(tokens, batch), threads, 0, stream>>>(p);
  else if (p.head_dim == 64)
    qk_norm_kernel<64><<<dim3(tokens, batch), threads, 0, stream>>>(p);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace ax
