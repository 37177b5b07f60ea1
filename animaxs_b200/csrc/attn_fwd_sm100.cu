// attn_fwd_sm100.cu -- flash attention for head_dim 128 on B200 (sm_100a).
//
// Replaces the reference's attention operator (AnimaXS/Runtime/Metal/
// AttentionExecutor.swift:122-302, whose DiT fast path is the Metal kernel
// dit_flash_attention_h128_q4_k32, AnimaKernels.metal:2193-2318, and whose
// general path is MPS QK^T -> attention_softmax_rows (:1051-1100) -> MPS PV).
// Same math: O = softmax(Q K^T * scale + mask) V with fp32 softmax statistics,
// here as an online (flash) softmax over 128-key tiles.
//
// One CTA = one 128-row query tile of one (batch, head).  Six warps:
//   warps 0-3  softmax: thread t owns query row t (= TMEM lane t); reads S from
//              TMEM, applies causal / key-padding masks, keeps the running
//              max / sum in fp32, rescales the O accumulator in TMEM, writes
//              P (fp16) into a 128B-swizzled shared tile, and finally
//              normalises O and stores it.
//   warp 4     TMA producer: Q once, then K_j / V_j tiles into a 2-stage ring.
//   warp 5     MMA issuer (one thread) + TMEM owner: S_j = Q K_j^T into one of
//              two TMEM S buffers, O += P_j V_j into the TMEM O accumulator,
//              both tcgen05.mma kind::f16 with operands in shared memory.
// TMEM: columns [0,128) S buffer 0, [128,256) S buffer 1, [256,384) O.
//
// Pipelining: QK^T for tile j+1 runs on the tensor core while the softmax
// warps work on tile j; PV for tile j is issued as soon as P_j is written.
#include "kernels.h"
#include "sm100_ptx.cuh"

namespace ax {
namespace {

constexpr uint32_t kTileBytes = kTileM * kHeadDim * 2;  // 32 KiB: one 128x128 fp16 tile
constexpr uint32_t kPanelBytes = 128 * 128;             // 128 rows x 128 B (64 fp16)
constexpr uint32_t kSmQ = 0;
constexpr uint32_t kSmK = kSmQ + kTileBytes;            // 2 stages
constexpr uint32_t kSmV = kSmK + 2 * kTileBytes;        // 2 stages
constexpr uint32_t kSmP = kSmV + 2 * kTileBytes;
constexpr uint32_t kSmBar = kSmP + kTileBytes;
constexpr uint32_t kSmemBytes = kSmBar + 256 + 1024;    // + barriers + alignment slack

enum : int {
  kBarQ = 0,
  kBarKFull = 1,   // +stage
  kBarKEmpty = 3,  // +stage
  kBarVFull = 5,   // +stage
  kBarVEmpty = 7,  // +stage
  kBarSFull = 9,   // +buffer
  kBarSFree = 11,  // +buffer
  kBarPFull = 13,
  kBarORdy = 14,
  kBarDone = 15,
  kNumBars = 16
};
constexpr uint32_t kSlotTmem = kNumBars * 8;   // byte offset (from kSmBar) of the TMEM address
constexpr uint32_t kSlotAbort = kSlotTmem + 4;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0;
constexpr uint32_t kColO = 256;
constexpr uint32_t kIdescQK = idesc_f16_f32(128, 128, false);  // B = K tile, K-major
constexpr uint32_t kIdescPV = idesc_f16_f32(128, 128, true);   // B = V tile, MN-major

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

__device__ __forceinline__ void rescale32(uint32_t (&r)[32], float a) {
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * a);
}

__global__ void __launch_bounds__(192, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base + kSmQ, sK = base + kSmK, sV = base + kSmV, sP = base + kSmP;
  const uint32_t bar0 = base + kSmBar;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + kSmBar + kSlotTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kSmBar + kSlotAbort);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = p.causal ? (p.n_q_tiles - 1 - static_cast<int>(blockIdx.x))
                          : static_cast<int>(blockIdx.x);
  const int h = p.head_offset + static_cast<int>(blockIdx.y);
  const int b = static_cast<int>(blockIdx.z);
  const int kvh = h / p.heads_per_kv;
  const int q0 = qt * kTileM;

  int valid = p.kv_valid;
  if (p.kv_valid_dev != nullptr) valid = p.kv_valid_dev[b];
  valid = min(max(valid, 1), p.kv_len);
  int kv_end = valid;
  if (p.causal) kv_end = min(kv_end, q0 + kTileM);
  const int n_kv = (kv_end + kTileN - 1) / kTileN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      const uint32_t cnt = (i == kBarSFree || i == kBarSFree + 1 || i == kBarPFull) ? 128u : 1u;
      mbar_init(BAR(i), cnt);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 5) {
    tmem_alloc(bar0 + kSlotTmem, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int armed_k[2] = {0, 0}, armed_v[2] = {0, 0};
      mbar_arrive_expect_tx(BAR(kBarQ), kTileBytes);
      tma_load_4d(sQ, &tm_q, BAR(kBarQ), 0, q0, h, b);
      tma_load_4d(sQ + kPanelBytes, &tm_q, BAR(kBarQ), 64, q0, h, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(BAR(kBarKEmpty + st), ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(BAR(kBarKFull + st), kTileBytes);
        tma_load_4d(sK + st * kTileBytes, &tm_k, BAR(kBarKFull + st), 0, j * kTileN, kvh, b);
        tma_load_4d(sK + st * kTileBytes + kPanelBytes, &tm_k, BAR(kBarKFull + st), 64,
                    j * kTileN, kvh, b);
        ++armed_k[st];
        if (!mbar_wait(BAR(kBarVEmpty + st), ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(BAR(kBarVFull + st), kTileBytes);
        tma_load_4d(sV + st * kTileBytes, &tm_v, BAR(kBarVFull + st), 0, j * kTileN, kvh, b);
        tma_load_4d(sV + st * kTileBytes + kPanelBytes, &tm_v, BAR(kBarVFull + st), 64,
                    j * kTileN, kvh, b);
        ++armed_v[st];
      }
      // Never leave the CTA with a tensor copy still landing in shared memory:
      // wait (bounded, ignoring the abort flag) for every phase armed above.
      int local_abort = 0;
      mbar_wait(BAR(kBarQ), 0, &local_abort, nullptr);
      for (int st = 0; st < 2; ++st) {
        local_abort = 0;
        if (armed_k[st]) mbar_wait(BAR(kBarKFull + st), (armed_k[st] - 1) & 1, &local_abort, nullptr);
        local_abort = 0;
        if (armed_v[st]) mbar_wait(BAR(kBarVFull + st), (armed_v[st] - 1) & 1, &local_abort, nullptr);
      }
    }
  } else if (warp == 5) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      bool ok = mbar_wait(BAR(kBarQ), 0, abort_flag, p.status);
      tc_fence_after();
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(BAR(kBarKFull + st), ph, abort_flag, p.status)) break;
          if (!mbar_wait(BAR(kBarSFree + st), ph ^ 1u, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t d_s = tmem + kColS0 + st * 128;
          const uint32_t kt = sK + st * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ss(d_s, kmajor_desc(sQ, kk), kmajor_desc(kt, kk), kIdescQK, kk > 0 ? 1u : 0u);
          tc_commit(BAR(kBarSFull + st));
          tc_commit(BAR(kBarKEmpty + st));
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int st = jj & 1;
          const uint32_t ph = (jj >> 1) & 1;
          if (!mbar_wait(BAR(kBarPFull), static_cast<uint32_t>(jj & 1), abort_flag, p.status)) break;
          if (!mbar_wait(BAR(kBarVFull + st), ph, abort_flag, p.status)) break;
          tc_fence_after();
          const uint32_t vt = sV + st * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ss(tmem + kColO, kmajor_desc(sP, kk), vmajor_desc(vt, kk), kIdescPV,
                        (jj > 0 || kk > 0) ? 1u : 0u);
          tc_commit(BAR(kBarVEmpty + st));
          tc_commit(BAR(kBarORdy));
        }
      }
      // All MMAs this thread issued must retire before TMEM is released.
      tc_commit(BAR(kBarDone));
      int local_abort = 0;
      mbar_wait(BAR(kBarDone), 0, &local_abort, nullptr);
    }
  } else {
    // ------------------------------------------------------------- softmax --
    const int t = threadIdx.x;  // query row within the tile == TMEM lane
    const int row = q0 + t;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = mbar_wait(BAR(kBarSFull + sb), ph, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t s[4][32];
      const uint32_t s_addr = tmem + lane_base + kColS0 + sb * 128;
      tmem_ld32(s_addr + 0, s[0]);
      tmem_ld32(s_addr + 32, s[1]);
      tmem_ld32(s_addr + 64, s[2]);
      tmem_ld32(s_addr + 96, s[3]);
      tmem_ld_wait(s[0]);
      asm volatile("" : AX_RW32(s[1])::"memory");
      asm volatile("" : AX_RW32(s[2])::"memory");
      asm volatile("" : AX_RW32(s[3])::"memory");
      tc_fence_before();
      mbar_arrive(BAR(kBarSFree + sb));

      const int key0 = j * kTileN;
      const bool need_mask = (key0 + kTileN > valid) || (p.causal && key0 + kTileN - 1 > row);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        float v = __uint_as_float(s[c >> 5][c & 31]);
        if (need_mask) {
          const int key = key0 + c;
          if (key >= valid || (p.causal && key > row)) v = -INFINITY;
        }
        s[c >> 5][c & 31] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m, mx * sl2);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2_approx(m - m_use);
      float rs = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(s[c >> 5][c & 31]), sl2, -m_use));
        const float p1 = ex2_approx(fmaf(__uint_as_float(s[(c + 1) >> 5][(c + 1) & 31]), sl2, -m_use));
        rs += p0 + p1;
        pk[c >> 1] = pack_half2(p0, p1);
      }
      l = l * alpha + rs;
      m = m_new;

      if (j >= 1) {
        // PV(j-1) must have retired: the O accumulator is stable and P is free.
        ok = mbar_wait(BAR(kBarORdy), static_cast<uint32_t>((j - 1) & 1), abort_flag, p.status);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t o[32];
            const uint32_t o_addr = tmem + lane_base + kColO + c4 * 32;
            tmem_ld32(o_addr, o);
            tmem_ld_wait(o);
            rescale32(o, alpha);
            tmem_st32(o_addr, o);
          }
          tmem_st_wait();
        }
      }
      // P row t -> 128B-swizzled K-major tile (two 64-key panels).
      const uint32_t prow = sP + static_cast<uint32_t>(t) * 128u;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        const uint32_t addr = prow + (ch >> 3) * kPanelBytes + ((((ch & 7) ^ (t & 7))) << 4);
        st_shared_v4(addr, pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(kBarPFull));
    }
    if (ok) {
      ok = mbar_wait(BAR(kBarORdy), static_cast<uint32_t>((n_kv - 1) & 1), abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      __half* orow = p.o + static_cast<long long>(b) * p.o_batch +
                     static_cast<long long>(row) * p.o_tok +
                     static_cast<long long>(h - p.o_head_base) * p.o_head;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kColO + c4 * 32, o);
        tmem_ld_wait(o);
        if (row < p.q_len) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = pack_half2(__uint_as_float(o[i * 8 + 0]) * inv_l, __uint_as_float(o[i * 8 + 1]) * inv_l);
            v.y = pack_half2(__uint_as_float(o[i * 8 + 2]) * inv_l, __uint_as_float(o[i * 8 + 3]) * inv_l);
            v.z = pack_half2(__uint_as_float(o[i * 8 + 4]) * inv_l, __uint_as_float(o[i * 8 + 5]) * inv_l);
            v.w = pack_half2(__uint_as_float(o[i * 8 + 6]) * inv_l, __uint_as_float(o[i * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + i * 8) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
#undef BAR
}

}  // namespace

cudaError_t launch_attn_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const AttnFwdParams& p, int heads_in_launch, int batch,
                            cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_sm100_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid(p.n_q_tiles, heads_in_launch, batch);
  attn_fwd_sm100_kernel<<<grid, 192, kSmemBytes, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace ax
