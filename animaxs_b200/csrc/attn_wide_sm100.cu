// attn_wide_sm100.cu -- flash attention for head_dim 256 and 384 on B200 (sm_100a).
//
// The reference's attention operator takes any head dim (AttentionExecutor.swift:
// 122-302; head-major inputs go through the MPS path at :220-300).  Besides the
// DiT / Qwen / adapter heads (64, 128: attn_fwd_sm100.cu) its one wide caller is
// the VAE decoder's middle attention (VAEDecoder.swift:351-410): one head of 384
// channels over the 64x64 latent positions, Q/K/V contiguous [positions, 384]
// blocks, non-causal, scale 1/sqrt(384).  Same math as the other kernel:
// O = softmax(Q K^T * scale + mask) V with fp32 statistics, online over 128-key
// tiles.
//
// One CTA owns one 128-row query tile.  A 384-wide O does not fit twice in
// TMEM beside a score tile, so TMEM holds S [0,128) and O [128, 128+HD) (512
// columns at HD 384), and P goes to shared memory (a 128x128 fp16 K-major
// tile, the A operand of PV).  That frees S as soon as the softmax has read it:
// the MMA warp issues QK(j+1) while the softmax still computes P(j), then
// PV(j), so the tensor core runs QK(j+1), PV(j), QK(j+2), PV(j+1), ... and
// the softmax hides under the QKs.  Q stays resident in shared memory
// (HD/128 chunks of 128x128); K and V stream through one ring of 128-key x
// 128-column chunks in the order the MMAs consume them: K(0), then per tile j
// K(j+1) (S accumulates over the head-dim chunks) and V(j) (chunk c feeds O
// columns [128c, 128c+128)).  Ten warps:
//   warps 0-3 / 4-7  softmax: warpgroup g takes keys [64g, 64g+64) of every S
//                    tile (= P panel g) and O columns [g*HD/2, (g+1)*HD/2);
//                    thread t owns query row t (TMEM lane t).  The two halves
//                    of a row exchange their maxima through shared memory.
//   warp 8           MMA issuer + TMEM owner.
//   warp 9           TMA producer.
//
// Key split.  A 4096-position VAE image has 32 query tiles: one CTA each would
// leave 116 of 148 SMs idle.  When there are few query tiles the launch splits
// each tile's keys over a thread-block cluster of n_split (2 or 4) CTAs; each
// computes an unnormalised partial O with its own row max m and sum l, and the
// cluster merges them through distributed shared memory, with no global
// workspace: the CTA of split s finishes rows [R*s, R*s + R), R = 128 /
// n_split; every CTA sends those rows' raw O and (m, l) to it, and it stores
// sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M) (M = max_s m_s).  The receive
// buffers overlay the Q/P/ring region, idle once every CTA's MMAs and copies
// are done (the first cluster barrier).
//
// Measured on B200 and not kept: the same kernel as a tcgen05 CTA pair
// (cta_group::2, M = 256, each CTA loading half of every K/V chunk) halves the
// MMA instructions, but with a single S buffer the pair waits on the slower
// of two softmaxes plus the cross-SM signal latency every tile, and ran
// 10% (one image: 2x, clusters of 8) slower.
#include <atomic>

#include "api_internal.h"
#include "flash_common.cuh"
#include "kernels.h"

namespace ax {
namespace {

constexpr int kThreads = 320;                  // 2 softmax warpgroups, MMA warp, TMA warp
constexpr int kSoftmaxThreads = 256;
constexpr uint32_t kChunk = 2 * kPanelBytes;   // 128 rows x 128 fp16 = two SW128 panels (32 KiB)

template <int HD>
struct WideSmem {
  static constexpr int kNC = HD / 128;                   // 128-column chunks of the head dim
  static constexpr int kStages = HD == 384 ? 3 : 4;      // K/V chunk ring (what 227 KiB leaves)
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kP = kNC * kChunk;           // P: 128 rows x 128 keys, K-major SW128
  static constexpr uint32_t kRing = kP + kChunk;
  static constexpr uint32_t kBar = kRing + kStages * kChunk;
  static constexpr uint32_t kXch = kBar + 256;           // 2 x 128 floats: row max / row sum exchange
  static constexpr uint32_t kBytes = kXch + 1024 + 1024; // + alignment slack
};
constexpr int kMaxStages = 4;
static_assert(WideSmem<384>::kBytes <= 227 * 1024, "shared memory exceeds the 227 KiB opt-in");
// Merge buffers (offset 0): receive 128 x HD fp32, statistics 1 KiB, one 32-row
// fp16 store stage; the ns == 1 store stage (128 x HD fp16) is smaller.
static_assert(128u * 384 * 4 + 1024 + 32 * 384 * 2 <= WideSmem<384>::kBar, "merge buffers overflow");
static_assert(128u * 256 * 4 + 1024 + 32 * 256 * 2 <= WideSmem<256>::kBar, "merge buffers overflow");

enum : int {
  kBarQ = 0,
  kBarFull = 1,                       // +stage
  kBarEmpty = kBarFull + kMaxStages,  // +stage
  kBarSFull = kBarEmpty + kMaxStages, // S(j) in TMEM
  kBarSFree,                          // the softmax holds S(j) in registers: QK(j+1) may overwrite it
  kBarPFull,                          // 256 arrivals: P(j) in shared memory
  kBarPFree,                          // PV(j) retired: P may be rewritten, O rescaled
  kBarODone,                          // the last PV retired
  kBarDone,
  kNumBars
};
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;
static_assert(kSlotAbort + 4 <= 256, "barrier block overflows its 256 bytes");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128;
constexpr uint32_t kIdescQK = idesc_f16_f32(128, 128, false);  // B = K chunk, K-major
constexpr uint32_t kIdescPV = idesc_f16_f32(128, 128, true);   // A = P (K-major), B = V chunk, MN-major

// Named barrier id of the two softmax warpgroups (0 is __syncthreads').
constexpr uint32_t kSoftmaxBar = 1;

__device__ __forceinline__ bool softmax_bar_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "n"(kSoftmaxBar), "n"(kSoftmaxThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ int kv_tiles(int tile_q0, int q_len, int valid, int causal) {
  if (tile_q0 >= q_len) return 0;
  int e = valid;
  if (causal) e = min(e, tile_q0 + kTileM);
  return (e + kTileN - 1) / kTileN;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_wide_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v,
                           const __grid_constant__ CUtensorMap tm_o, const AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  using L = WideSmem<HD>;
  constexpr int NC = L::kNC;
  const uint32_t sQ = base + L::kQ, sP = base + L::kP, sRing = base + L::kRing;
  const uint32_t bar0 = base + L::kBar;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + L::kBar + kSlotTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kBar + kSlotAbort);
  volatile float* xch = reinterpret_cast<volatile float*>(gbase + L::kXch);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Cluster dims (n_split, 1, 1): the n_split CTAs of one query tile are consecutive.
  const int ns = p.n_split;
  const int rank = ns > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int item = static_cast<int>(blockIdx.x) / ns;
  const int qi = item % p.n_q_tiles;
  const int hb = item / p.n_q_tiles;
  const int q0 = (p.causal ? (p.n_q_tiles - 1 - qi) : qi) * kTileM;  // causal: longest first
  const int h = p.head_offset + hb % p.heads_in_launch;
  const int b = hb / p.heads_in_launch;
  const int kvh = h / p.heads_per_kv;
  int valid = p.kv_valid;
  if (p.kv_valid_dev != nullptr) valid = p.kv_valid_dev[b];
  valid = min(max(valid, 1), p.kv_len);
  const int n_all = kv_tiles(q0, p.q_len, valid, p.causal);
  const int j_begin = rank * n_all / ns;
  const int n_my = (rank + 1) * n_all / ns - j_begin;  // key tiles of this CTA (may be 0)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(BAR(i), i == kBarPFull ? kSoftmaxThreads : 1u);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 8) {
    tmem_alloc(bar0 + kSlotTmem, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ producer --
    if (lane == 0 && n_my > 0) {
      int armed_q = 0, armed[kMaxStages] = {};
      bool ok = true;
      mbar_arrive_expect_tx(BAR(kBarQ), NC * kChunk);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        tma_load_4d(sQ + c * kChunk, &tm_q, BAR(kBarQ), 128 * c, q0, h, b);
        tma_load_4d(sQ + c * kChunk + kPanelBytes, &tm_q, BAR(kBarQ), 128 * c + 64, q0, h, b);
      }
      armed_q = 1;
      uint32_t g = 0;  // chunks loaded so far: stage g % kStages
      // The NC chunks of key tile `jt` of K or V, in ring order.
      auto load_tile = [&](const CUtensorMap* tm, int jt) {
        const int key0 = (j_begin + jt) * kTileN;
        for (int c = 0; c < NC; ++c, ++g) {
          const uint32_t st = g % L::kStages;
          if (!(ok = mbar_wait(BAR(kBarEmpty + st), ((g / L::kStages) & 1u) ^ 1u, abort_flag, p.status)))
            return;
          const uint32_t dst = sRing + st * kChunk;
          mbar_arrive_expect_tx(BAR(kBarFull + st), kChunk);
          tma_load_4d(dst, tm, BAR(kBarFull + st), 128 * c, key0, kvh, b);
          tma_load_4d(dst + kPanelBytes, tm, BAR(kBarFull + st), 128 * c + 64, key0, kvh, b);
          ++armed[st];
        }
      };
      // The order the MMA warp consumes them: K(0), then K(j+1), V(j).
      load_tile(&tm_k, 0);
      for (int j = 0; ok && j < n_my; ++j) {
        if (j + 1 < n_my) load_tile(&tm_k, j + 1);
        if (ok) load_tile(&tm_v, j);
      }
      // Never leave with a tensor copy still landing in shared memory.
      if (armed_q) mbar_wait_drain(BAR(kBarQ), 0);
      for (int st = 0; st < L::kStages; ++st)
        if (armed[st]) mbar_wait_drain(BAR(kBarFull + st), (armed[st] - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 8) {
    // ----------------------------------------------------------------- MMA --
    // Whole warp runs the loop; one elected lane issues each MMA and commit.
    if (n_my > 0) {
      bool ok = mbar_wait_warp(BAR(kBarQ), 0, abort_flag, p.status);
      uint32_t g = 0;  // chunks consumed so far
      // S = Q K_jt^T, accumulated over the head-dim chunks.
      auto qk = [&]() {
        for (int c = 0; c < NC; ++c, ++g) {
          const uint32_t st = g % L::kStages;
          if (!(ok = mbar_wait_warp(BAR(kBarFull + st), (g / L::kStages) & 1u, abort_flag, p.status)))
            return;
          tc_fence_after();
          const uint64_t a0 = kmajor_desc(sQ + c * kChunk, 0);
          const uint64_t b0 = kmajor_desc(sRing + st * kChunk, 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4);
            umma_f16_ss_warp(tmem + 0, a0 + off, b0 + off, kIdescQK, (c > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_warp(BAR(kBarEmpty + st));
        }
        tc_commit_warp(BAR(kBarSFull));
      };
      if (ok) qk();
      for (int j = 0; ok && j < n_my; ++j) {
        if (j + 1 < n_my) {
          // QK(j+1) overwrites S once the softmax holds S(j) in registers.
          if (!(ok = mbar_wait_warp(BAR(kBarSFree), j & 1u, abort_flag, p.status))) break;
          tc_fence_after();
          qk();
          if (!ok) break;
        }
        // O[:, 128c:128c+128] += P(j) V_j[:, 128c:128c+128], P from shared memory.
        if (!(ok = mbar_wait_warp(BAR(kBarPFull), j & 1u, abort_flag, p.status))) break;
        tc_fence_after();
        const uint64_t a0 = kmajor_desc(sP, 0);
        for (int c = 0; c < NC; ++c, ++g) {
          const uint32_t st = g % L::kStages;
          if (!(ok = mbar_wait_warp(BAR(kBarFull + st), (g / L::kStages) & 1u, abort_flag, p.status))) break;
          tc_fence_after();
          const uint64_t b0 = vmajor_desc(sRing + st * kChunk, 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t aoff = static_cast<uint64_t>(((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4);
            umma_f16_ss_warp(tmem + kColO + 128 * c, a0 + aoff,
                             b0 + static_cast<uint64_t>((kk * 2048) >> 4), kIdescPV,
                             (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_warp(BAR(kBarEmpty + st));
        }
        if (!ok) break;
        tc_commit_warp(BAR(kBarPFree));
      }
      if (ok) tc_commit_warp(BAR(kBarODone));
    }
    // All MMAs this warp issued must retire before TMEM and shared memory are reused.
    tc_commit_warp(BAR(kBarDone));
    mbar_wait_drain(BAR(kBarDone), 0);
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax --
    const int wg = warp >> 2;          // key half of S / column half of O
    const int t = threadIdx.x & 127;   // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + wg * 64;
    const uint32_t o_addr = tmem + lane_base + kColO + wg * (HD / 2);
    // Row t of P panel wg (keys [64wg, 64wg+64)); 16-byte unit u of a 128-byte
    // SW128 row sits at unit u ^ (row % 8).
    const uint32_t p_row = sP + wg * kPanelBytes + t * 128;
    const int row = q0 + t;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_my; ++j) {
      bool got = ok && mbar_wait(BAR(kBarSFull), j & 1u, abort_flag, p.status);
      // The other half read the previous tile's xch entry before its P(j-1) arrival.
      if (got && j > 0) got = mbar_wait(BAR(kBarPFull), (j - 1) & 1u, abort_flag, p.status);
      got = __all_sync(0xffffffffu, got);
      uint32_t s[2][32];
      float pm = -INFINITY;
      if (got) {
        tc_fence_after();
        tmem_ld32(s_addr + 0, s[0]);
        tmem_ld32(s_addr + 32, s[1]);
        tmem_ld_wait(s[0]);
        asm volatile("" : AX_RW32(s[1])::"memory");
        const int key0 = (j_begin + j) * kTileN + wg * 64;
        if ((key0 + 64 > valid) || (p.causal && key0 + 63 > row)) {
          const int lim = p.causal ? min(valid, row + 1) : valid;  // keys >= lim are masked
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (key0 + c >= lim) s[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
#define SV(c) __uint_as_float(s[(c) >> 5][(c) & 31])
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mx[i] = fmax3(SV(i), SV(i + 8), SV(i + 16));
          mx[i] = fmax3(mx[i], SV(i + 24), SV(i + 32));
          mx[i] = fmax3(mx[i], SV(i + 40), SV(i + 48));
          mx[i] = fmaxf(mx[i], SV(i + 56));
        }
#undef SV
        pm = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) * sl2;
        xch[wg * 128 + t] = pm;
      }
      // Every thread has S(j) in registers (and its max in xch); the barrier
      // also makes the abort decision common.
      tc_fence_before();
      ok = softmax_bar_and(got);
      if (!ok) break;
      if (threadIdx.x == 0) mbar_arrive(BAR(kBarSFree));
      const float tmax = fmaxf(pm, xch[(wg ^ 1) * 128 + t]);
      const float m_new = fmaxf(m, tmax);
      const bool grow = m_new > m + kRescaleThreshold;  // also true on the first tile
      const float alpha = grow ? ex2_approx(m - m_new) : 1.f;
      if (grow) {
        l *= alpha;
        m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      const float2 sl2v = make_float2(sl2, sl2);
      const float2 nmv = make_float2(neg_m, neg_m);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                       make_float2(0.f, 0.f)};
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float2 x = fma2(make_float2(__uint_as_float(s[c >> 5][c & 31]),
                                          __uint_as_float(s[c >> 5][(c + 1) & 31])),
                              sl2v, nmv);
        float2 pr;
        if (((c >> 1) & 7) < kPolyPairsPer8) {
          pr = ex2_poly2(x);
        } else {
          pr.x = ex2_approx(x.x);
          pr.y = ex2_approx(x.y);
        }
        acc[(c >> 1) & 3] = add2(acc[(c >> 1) & 3], pr);
        pk[c >> 1] = pack_half2(pr.x, pr.y);
      }
      // PV(j-1) must have retired before P is rewritten and O rescaled.
      bool free_p = true;
      if (j > 0) {
        free_p = mbar_wait(BAR(kBarPFree), (j - 1) & 1u, abort_flag, p.status);
        free_p = __all_sync(0xffffffffu, free_p);
      }
      if (free_p) {
        tc_fence_after();
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int c4 = 0; c4 < HD / 64; ++c4) {
            uint32_t o[32];
            tmem_ld32(o_addr + c4 * 32, o);
            tmem_ld_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + c4 * 32, o);
          }
          tmem_st_wait();
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          st_shared_v4(p_row + ((u ^ (t & 7)) << 4), pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        fence_proxy_async_smem();  // P is read by the tensor core (async proxy)
        tc_fence_before();
        mbar_arrive(BAR(kBarPFull));
      }
      const float2 a = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
      l += a.x + a.y;
      // A failed wait here surfaces at the next tile's barrier (or the ODone wait).
      ok = free_p;
    }
    if (ok && n_my > 0) {
      ok = mbar_wait(BAR(kBarODone), 0, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) tc_fence_after();
    }
    // Row sum over both halves.  (The other half's last read of xch preceded
    // its P arrival, which the last PV, hence ODone, waited for.)
    xch[wg * 128 + t] = l;
    named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
    const float l_row = l + xch[(wg ^ 1) * 128 + t];
    const bool have = ok && n_my > 0;
    const int st_id = threadIdx.x;  // 0..255 over both softmax warpgroups
    const int oh = h - p.o_head_base;
    if (ns == 1) {
      // Normalise and stage O as fp16 in the tensor-store box layout (HD/64
      // panels of 128 rows x 128 B, 128-byte swizzle) over the idle Q region,
      // then one thread stores it with TMA (rows past q_len are clipped).
      if (have) {
        const float inv_l = 1.f / l_row;
#pragma unroll 1
        for (int c4 = 0; c4 < HD / 64; ++c4) {
          uint32_t o[32];
          tmem_ld32(o_addr + c4 * 32, o);
          tmem_ld_wait(o);
          const int col = wg * (HD / 2) + c4 * 32;
          const uint32_t prow = base + (col >> 6) * 16384 + t * 128;
          const int u0 = (col & 63) >> 3;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            st_shared_v4(prow + (((u0 + i) ^ (t & 7)) << 4),
                         pack_half2(__uint_as_float(o[i * 8 + 0]) * inv_l, __uint_as_float(o[i * 8 + 1]) * inv_l),
                         pack_half2(__uint_as_float(o[i * 8 + 2]) * inv_l, __uint_as_float(o[i * 8 + 3]) * inv_l),
                         pack_half2(__uint_as_float(o[i * 8 + 4]) * inv_l, __uint_as_float(o[i * 8 + 5]) * inv_l),
                         pack_half2(__uint_as_float(o[i * 8 + 6]) * inv_l, __uint_as_float(o[i * 8 + 7]) * inv_l));
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
      if (st_id == 0 && have) {
        for (int pnl = 0; pnl < HD / 64; ++pnl)
          for (int r32 = 0; r32 < 4 && q0 + 32 * r32 < p.q_len; ++r32)
            tma_store_4d(&tm_o, base + pnl * 16384 + r32 * 4096, 64 * pnl, q0 + 32 * r32, oh, b);
        tma_store_commit();
        tma_store_wait_all();
      }
    } else {
      // Cluster merge by rows: rank r finishes rows [R*r, R*r + R) of the tile,
      // R = 128 / n_split.  Each CTA sends the raw O and (m, l) of those rows to
      // rank r; a warp's lanes are consecutive rows, so in the quad-major
      // receive layout [sender][column quad][row][4] every remote store
      // instruction writes 512 contiguous bytes.  The producer and MMA warps
      // take the same two cluster barriers below.
      const int R = 128 / ns;
      const uint32_t sRecv = base;
      const uint32_t sStats = base + 128u * HD * 4;   // [sender][row] (m, l)
      const uint32_t sStage = sStats + 1024;          // 32 rows x HD fp16, store box layout
      fence_proxy_async_smem();
      cluster_sync();  // 1: every CTA's copies and MMAs are done: its ring may be overwritten
      const int owner = t / R, r_loc = t % R;
      if (wg == 0)
        st_cluster_v2f(mapa_shared(sStats + (rank * R + r_loc) * 8, owner), have ? m : -INFINITY,
                       have ? l_row : 0.f);
#pragma unroll 1
      for (int c4 = 0; c4 < HD / 64; ++c4) {
        uint32_t o[32];
        if (have) {
          tmem_ld32(o_addr + c4 * 32, o);
          tmem_ld_wait(o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        const int cq0 = (wg * (HD / 2) + c4 * 32) >> 2;
        const uint32_t dst = mapa_shared(sRecv + ((rank * (HD / 4) + cq0) * R + r_loc) * 16, owner);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_cluster_v4(dst + i * R * 16, o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      }
      cluster_sync();  // 2: every sender's rows have arrived
      // out = sum_s O_s * 2^(m_s - M) / L, M = max_s m_s, L = sum_s l_s 2^(m_s - M);
      // 32 rows per round, staged as fp16 and stored with TMA.
      for (int r0 = 0; r0 < R; r0 += 32) {
        const int r = r0 + (st_id & 31);  // this thread's row in every pass of the round
        float wgt[4] = {0.f, 0.f, 0.f, 0.f};
        {
          float M = -INFINITY, Lsum = 0.f;
          for (int sdr = 0; sdr < ns; ++sdr) {
            const float2 ml = ld_shared_v2f(sStats + (sdr * R + r) * 8);
            if (ml.y > 0.f) M = fmaxf(M, ml.x);
          }
          for (int sdr = 0; sdr < ns; ++sdr) {
            const float2 ml = ld_shared_v2f(sStats + (sdr * R + r) * 8);
            if (ml.y > 0.f) {
              wgt[sdr] = ex2_approx(ml.x - M);
              Lsum += ml.y * wgt[sdr];
            }
          }
          const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
          for (int sdr = 0; sdr < ns; ++sdr) wgt[sdr] *= inv;
        }
        const int rr = st_id & 31;
#pragma unroll 1
        for (int cq = st_id >> 5; cq < HD / 4; cq += kSoftmaxThreads / 32) {
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sdr = 0; sdr < ns; ++sdr) {
            const float4 x = ld_shared_v4f(sRecv + ((sdr * (HD / 4) + cq) * R + r) * 16);
            a.x += wgt[sdr] * x.x;
            a.y += wgt[sdr] * x.y;
            a.z += wgt[sdr] * x.z;
            a.w += wgt[sdr] * x.w;
          }
          const uint32_t unit = static_cast<uint32_t>(((cq & 15) >> 1) ^ (rr & 7));
          st_shared_v2(sStage + (cq >> 4) * 4096 + rr * 128 + (unit << 4) + (cq & 1) * 8,
                       pack_half2(a.x, a.y), pack_half2(a.z, a.w));
        }
        fence_proxy_async_smem();
        named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
        const int row0 = q0 + rank * R + r0;
        if (st_id == 0 && row0 < p.q_len) {
          for (int pnl = 0; pnl < HD / 64; ++pnl)
            tma_store_4d(&tm_o, sStage + pnl * 4096, 64 * pnl, row0, oh, b);
          tma_store_commit();
          tma_store_wait_all();
        }
        named_bar_sync(kSoftmaxBar, kSoftmaxThreads);  // the stage may be refilled
      }
    }
  }
  if (ns > 1 && warp >= 8) {
    fence_proxy_async_smem();
    cluster_sync();
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
#undef BAR
}

template <int HD>
cudaError_t launch_wide_hd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const AttnFwdParams& p, int heads_in_launch, int batch, int dev,
                           cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  cudaError_t e;
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load(std::memory_order_acquire) & bit) == 0) {
    e = cudaFuncSetAttribute(attn_wide_sm100_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             WideSmem<HD>::kBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  static std::atomic<int> sm_count[64];
  int sms = sm_count[dev & 63].load(std::memory_order_relaxed);
  if (sms == 0) {
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sm_count[dev & 63].store(sms, std::memory_order_relaxed);
  }
  AttnFwdParams q = p;
  q.heads_in_launch = heads_in_launch;
  q.n_q_tiles = (p.q_len + kTileM - 1) / kTileM;
  const long long items = static_cast<long long>(q.n_q_tiles) * heads_in_launch * batch;
  if (items <= 0) return cudaSuccess;
  // Split the keys while the launch would leave half the SMs idle and every
  // split keeps at least two key tiles.
  const int kv_tiles_max = (p.kv_len + kTileN - 1) / kTileN;
  int ns = 1;
  while (ns < 4 && items * ns * 2 <= sms && kv_tiles_max >= 4 * ns) ns *= 2;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = WideSmem<HD>::kBytes;
  cfg.stream = stream;
  // Clusters of ns CTAs with ~226 KiB of shared memory each must fit in a GPC.
  static std::atomic<int> cluster_ok[64][3];  // [dev][log2 ns]: 0 unknown, 1 yes, 2 no
  while (ns > 1) {
    const int li = ns == 2 ? 1 : 2;
    int known = cluster_ok[dev & 63][li].load(std::memory_order_relaxed);
    if (known == 0) {
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = ns;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.gridDim = dim3(static_cast<unsigned>(ns));
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, attn_wide_sm100_kernel<HD>, &cfg);
      if (e != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
      }
      known = clusters > 0 ? 1 : 2;
      cluster_ok[dev & 63][li].store(known, std::memory_order_relaxed);
    }
    if (known == 1) break;
    ns /= 2;
  }
  if (items * ns > 0x7fffffffLL) return cudaErrorInvalidValue;
  q.n_split = ns;
  cfg.gridDim = dim3(static_cast<unsigned>(items * ns));
  if (ns > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ns;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  } else {
    cfg.attrs = nullptr;
    cfg.numAttrs = 0;
  }
  // Output view [batch][heads][q_len][HD] for the tensor stores (box 64 x 32).
  CUtensorMap to;
  if (ax_make_tmap(nullptr, &to, p.o, HD, p.q_len, p.head_offset + heads_in_launch - p.o_head_base, batch,
                   p.o_tok, p.o_head, p.o_batch, 32) != ANIMAXS_OK)
    return cudaErrorInvalidValue;
  e = cudaLaunchKernelEx(&cfg, attn_wide_sm100_kernel<HD>, tq, tk, tv, to, q);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attn_wide(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnFwdParams& p, int heads_in_launch, int batch, int dev,
                             cudaStream_t stream) {
  if (p.head_dim == 384) return launch_wide_hd<384>(tq, tk, tv, p, heads_in_launch, batch, dev, stream);
  if (p.head_dim == 256) return launch_wide_hd<256>(tq, tk, tv, p, heads_in_launch, batch, dev, stream);
  return cudaErrorInvalidValue;
}

}  // namespace ax
