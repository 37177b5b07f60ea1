// attn_s3_sm100.cu -- flash attention for head_dim 64 / 128 on B200 (sm_100a): one
// query tile per work item, three score buffers in TMEM.
//
// The same operator and the same per-row arithmetic as attn_fwd_sm100.cu
// (AttentionExecutor.swift:122-302; AnimaKernels.metal:2193-2318): an online
// softmax over 128-key tiles with fp32 statistics, the lazy O rescale (only
// when a row's max grows by more than 2^8), exp2 on the MUFU and FMA pipes in
// the same column pairs, P written as fp16 over the consumed scores and
// multiplied in the same two halves.  Each row goes through exactly the
// arithmetic of a chain of attn_fwd_sm100.cu, so the two kernels produce the
// same bits (P is published once per tile here: the softmax does not wait for
// the tensor core, so half-tile publication would gain nothing).
//
// What differs is the pipeline.  attn_fwd_sm100.cu runs two query tiles per
// CTA with one score buffer each, so every tile's chain is softmax(j) ->
// PV(j) -> QK(j+1) -> softmax(j+1): the tensor core's QK for the next key
// tile waits for this tile's P.  Here one query tile owns three score buffers
// (TMEM S0, S1, S2 = columns [0, 384), O = [384, 512)): QK(j+1..j+3) are
// issued while softmax(j) runs, so the softmax warpgroup goes from tile to
// tile without waiting for the tensor core, and the tensor core (1024 cycles
// of MMA per tile: QK 512 + PV 512) runs under it.
//
// Warps (256 threads, one CTA per SM, persistent over work items):
//   0-3  softmax: thread t owns query row t (= TMEM lane t)
//   4    MMA issuer + TMEM owner: QK(0..2), then per tile PV(j) (P from TMEM)
//        and QK(j+3) into the buffer PV(j) has just read
//   5    TMA producer: Q, then K_0..K_2 and per tile V_j, K_{j+3}, into a
//        3-stage K ring and a 2-stage V ring
//   6    PV tracker: consumes every V-stage release (= PV retired) in order and
//        publishes the count in shared memory, so that a softmax thread that
//        must rescale O (rare) can wait for exactly the PVs it needs
//   7    idle
// Used for the launches that deal single tiles; paired launches run
// attn_fwd_sm100.cu, whose two softmax warpgroups per SM hide each other's
// latencies (one warp per SM sub-partition cannot).  In the fused
// head-sharded gather (peer_sharded.cu) the epilogue also stores each output
// tile into every peer's buffer and counts the CTA's items on the peers'
// arrival words, as attn_fwd_sm100.cu does.
// Every wait is bounded (ANIMAXS_WAIT_TIMEOUT_NS); a timeout raises the CTA's
// abort flag and the device status bit, and the CTA drains and exits.
#include <atomic>

#include "api_internal.h"
#include "flash_common.cuh"
#include "kernels.h"

namespace ax {
namespace {

constexpr int kS3KStages = 3;
constexpr int kS3VStages = 2;
constexpr int kS3SBufs = 3;
template <int HD>
struct S3Smem {
  static constexpr uint32_t kTile = kTileM * HD * 2;  // 32 KiB (HD 128) / 16 KiB (HD 64)
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kTile;
  static constexpr uint32_t kV = kK + kS3KStages * kTile;
  static constexpr uint32_t kBar = kV + kS3VStages * kTile;
  // Output stage: per softmax warp, 32 rows x 64 columns fp16 (4 KiB) in the
  // tensor-store layout.
  static constexpr uint32_t kStage = kBar + 1024;
  static constexpr uint32_t kBytes = kStage + 4 * 4096 + 1024;  // + alignment slack
};
static_assert(S3Smem<128>::kBytes <= 227 * 1024, "shared memory exceeds the 227 KiB opt-in");
constexpr int kS3Threads = 256;

// The K ring has one stage per score buffer: K tile t lives in stage t % 3
// and is read only by QK(t) into buffer t % 3, so the barrier that tells the
// softmax that S(t) is ready also tells the producer that the stage is free.
// Likewise V tile t is read only by PV(t): the release of its stage marks
// PV(t) retired, which is what warp 6 counts.
static_assert(kS3KStages == kS3SBufs, "K stage t % 3 must be released by the commit of S buffer t % 3");
enum : int {
  kS3BarQ = 0,
  kS3BarKFull = 1,                          // +stage
  kS3BarVFull = kS3BarKFull + kS3KStages,   // +stage
  kS3BarVEmpty = kS3BarVFull + kS3VStages,  // +stage: PV of the stage's tile retired
  kS3BarSFull = kS3BarVEmpty + kS3VStages,  // +buffer: QK into the buffer retired (frees its K stage)
  kS3BarPFull = kS3BarSFull + kS3SBufs,     // +buffer (4 warp arrivals): P in the buffer
  kS3BarODone = kS3BarPFull + kS3SBufs,     // the item's last PV retired
  kS3BarQFree = kS3BarODone + 1,            // the item's last QK retired: Q may be reloaded
  kS3BarDone = kS3BarQFree + 1,
  kS3NumBars = kS3BarDone + 1
};
constexpr uint32_t kS3SlotTmem = kS3NumBars * 8;
constexpr uint32_t kS3SlotAbort = kS3SlotTmem + 4;
constexpr uint32_t kS3SlotPvDone = kS3SlotTmem + 8;  // PVs retired so far (warp 6)
static_assert(kS3SlotPvDone + 4 <= 1024, "barrier block overflows");
constexpr uint32_t kS3ColO = 384;
constexpr uint32_t kS3TmemCols = 512;

__device__ __forceinline__ uint32_t ld_acquire_cta(const volatile uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(const_cast<uint32_t*>(p))) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(volatile uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(const_cast<uint32_t*>(p))), "r"(v) : "memory");
}

// kPeers: the fused head-sharded gather's instantiation (peer stores and
// arrivals); a separate instantiation, so that the others carry no trace of it.
template <int HD, bool kPeers>
__global__ void __launch_bounds__(kS3Threads, 1)
    attn_s3_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                         const AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  using L = S3Smem<HD>;
  constexpr uint32_t kTileBytes = L::kTile;
  const uint32_t sQ = base + L::kQ, sK = base + L::kK, sV = base + L::kV;
  const uint32_t bar0 = base + L::kBar;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + L::kBar + kS3SlotTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kBar + kS3SlotAbort);
  volatile uint32_t* pv_done = reinterpret_cast<volatile uint32_t*>(gbase + L::kBar + kS3SlotPvDone);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work item w -> (query tile, head, batch); causal launches take the
  // longest tiles (the last ones) first.
  struct Item {
    int q0, h, b, kvh, valid, n;
  };
  auto item_of = [&](int w) {
    Item it;
    const int ti = w % p.n_q_tiles;
    const int hb = w / p.n_q_tiles;
    const int tile = p.causal ? (p.n_q_tiles - 1 - ti) : ti;
    it.h = p.head_offset + hb % p.heads_in_launch;
    it.b = hb / p.heads_in_launch;
    it.kvh = it.h / p.heads_per_kv;
    it.q0 = tile * kTileM;
    int valid = p.kv_valid;
    if (p.kv_valid_dev != nullptr) valid = p.kv_valid_dev[it.b];
    it.valid = min(max(valid, 1), p.kv_len);
    it.n = kv_tiles_for(it.q0, p.q_len, it.valid, p.causal);
    return it;
  };
  const int w0 = static_cast<int>(blockIdx.x);
  const int wstep = static_cast<int>(gridDim.x);
  // Fused head-sharded gather: store into the peers only after a completed handshake.
  const bool peers_go = kPeers && p.n_peers > 0 && (p.peer_go == nullptr || *p.peer_go == p.peer_go_value);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kS3NumBars; ++i)
      mbar_init(BAR(i), (i >= kS3BarPFull && i < kS3BarPFull + kS3SBufs) ? 4u : 1u);
    *abort_flag = 0;
    *pv_done = 0;
    mbar_fence_init();
  }
  if (warp == 4) {
    tmem_alloc(bar0 + kS3SlotTmem, kS3TmemCols);
    tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 5) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int armed_q = 0, armed_k[kS3KStages] = {}, armed_v[kS3VStages] = {};
      uint32_t gk = 0, gv = 0;  // K / V tiles loaded so far (ring position)
      // Tile number g of a ring with n stages lives in stage g % n; the wait for
      // a free stage is on the phase its previous occupant's release completed.
      auto load = [&](bool is_k, uint32_t g, int row0, int kvh, int b) -> bool {
        const uint32_t nst = is_k ? kS3KStages : kS3VStages;
        const uint32_t st = g % nst;
        const uint32_t ph = (g / nst) & 1u;
        const uint32_t full = BAR((is_k ? kS3BarKFull : kS3BarVFull) + st);
        const uint32_t dst = (is_k ? sK : sV) + st * kTileBytes;
        const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
        // The stage's previous tile (g - nst) is free once its only reader
        // retired: QK(g - 3) for K (S buffer st's commit), PV(g - 2) for V.
        if (!mbar_wait(BAR((is_k ? kS3BarSFull : kS3BarVEmpty) + st), ph ^ 1u, abort_flag, p.status))
          return false;
        mbar_arrive_expect_tx(full, kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) tma_load_4d(dst + c * kPanelBytes, tm, full, 64 * c, row0, kvh, b);
        ++(is_k ? armed_k[st] : armed_v[st]);
        return true;
      };
      bool ok = true;
      int it = 0;
      for (int w = w0; ok && w < p.n_items; w += wstep, ++it) {
        const Item I = item_of(w);
        // Q is reloaded once the previous item's last QK has retired.
        if (it > 0 && !(ok = mbar_wait(BAR(kS3BarQFree), static_cast<uint32_t>((it - 1) & 1),
                                       abort_flag, p.status)))
          break;
        mbar_arrive_expect_tx(BAR(kS3BarQ), kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_4d(sQ + c * kPanelBytes, &tm_q, BAR(kS3BarQ), 64 * c, I.q0, I.h, I.b);
        ++armed_q;
        // K/V in the order the MMA warp consumes them: K_0..K_2, then per tile
        // V_j, K_{j+3}.
        for (int j = 0; ok && j < min(kS3SBufs, I.n); ++j) ok = load(true, gk++, j * kTileN, I.kvh, I.b);
        for (int j = 0; ok && j < I.n; ++j) {
          if (!(ok = load(false, gv++, j * kTileN, I.kvh, I.b))) break;
          if (j + kS3SBufs < I.n && !(ok = load(true, gk++, (j + kS3SBufs) * kTileN, I.kvh, I.b))) break;
        }
      }
      // Never leave the CTA with a tensor copy still landing in shared memory:
      // wait (bounded, ignoring the abort flag) for every phase armed above.
      if (armed_q) mbar_wait_drain(BAR(kS3BarQ), (armed_q - 1) & 1);
      for (int st = 0; st < kS3KStages; ++st)
        if (armed_k[st]) mbar_wait_drain(BAR(kS3BarKFull + st), (armed_k[st] - 1) & 1);
      for (int st = 0; st < kS3VStages; ++st)
        if (armed_v[st]) mbar_wait_drain(BAR(kS3BarVFull + st), (armed_v[st] - 1) & 1);
    }
  } else if (warp == 4) {
    // ----------------------------------------------------------------- MMA --
    // The whole warp runs this loop; one elected lane issues each MMA and commit.
    uint32_t gk = 0, gv = 0;  // K / V tiles consumed so far
    uint32_t gt = 0;          // tiles of earlier items (score-buffer uses)
    bool ok = true;
    uint32_t it = 0;
    // QK of tile t (a running count) into buffer t % 3, with the next K tile.
    auto qk = [&](uint32_t t) -> bool {
      const uint32_t kst = gk % kS3KStages;
      if (!mbar_wait_warp(BAR(kS3BarKFull + kst), (gk / kS3KStages) & 1u, abort_flag, p.status)) return false;
      tc_fence_after();
      const uint32_t sb = t % kS3SBufs;
      issue_qk<HD>(tmem + sb * 128, sQ, sK + kst * kTileBytes);
      tc_commit_warp(BAR(kS3BarSFull + sb));  // S ready; K stage kst (= sb) free
      ++gk;
      return true;
    };
    for (int w = w0; ok && w < p.n_items; w += wstep, ++it) {
      const Item I = item_of(w);
      const int n = I.n;
      if (!(ok = mbar_wait_warp(BAR(kS3BarQ), it & 1u, abort_flag, p.status))) break;
      for (int j = 0; ok && j < min(kS3SBufs, n); ++j) ok = qk(gt + j);
      if (!ok) break;
      if (n <= kS3SBufs) tc_commit_warp(BAR(kS3BarQFree));  // the item's last QK
      for (int j = 0; j < n; ++j) {
        const uint32_t t = gt + j;
        const uint32_t sb = t % kS3SBufs;
        const uint32_t vst = gv % kS3VStages;
        if (!(ok = mbar_wait_warp(BAR(kS3BarVFull + vst), (gv / kS3VStages) & 1u, abort_flag, p.status))) break;
        const uint32_t vt = sV + vst * kTileBytes;
        // P(t) in buffer sb: the buffer's PFull barrier completes once per use.
        // An item's first PV overwrites O; its first P is published only after
        // the softmax threads' previous epilogue has read O out of TMEM.
        if (!(ok = mbar_wait_warp(BAR(kS3BarPFull + sb), (t / kS3SBufs) & 1u, abort_flag, p.status))) break;
        tc_fence_after();
        issue_pv_half<HD, false>(tmem + kS3ColO, tmem + sb * 128, vt, 0, j > 0);
        issue_pv_half<HD, false>(tmem + kS3ColO, tmem + sb * 128, vt, 1, true);
        if (j == n - 1) tc_commit_warp(BAR(kS3BarODone));
        tc_commit_warp(BAR(kS3BarVEmpty + vst));  // PV(t) retired: V stage free, counted by warp 6
        ++gv;
        // QK(t+3) overwrites buffer sb after PV(t) (same thread, issue order).
        if (j + kS3SBufs < n) {
          if (!(ok = qk(t + kS3SBufs))) break;
          if (j + kS3SBufs == n - 1) tc_commit_warp(BAR(kS3BarQFree));  // the item's last QK
        }
      }
      gt += n;
    }
    // All MMAs this warp issued must retire before TMEM is released.
    tc_commit_warp(BAR(kS3BarDone));
    mbar_wait_drain(BAR(kS3BarDone), 0);
    __syncwarp();
  } else if (warp == 6) {
    // ---------------------------------------------------------- PV tracker --
    // Consume the V-stage releases (one per PV, tile c in stage c % 2) in
    // order, so that no wait can mistake an older phase for the one it
    // wants, and publish the count of retired PVs.
    uint32_t total = 0;
    for (int w = w0; w < p.n_items; w += wstep) total += item_of(w).n;
    for (uint32_t c = 0; c < total; ++c) {
      if (!mbar_wait_warp(BAR(kS3BarVEmpty + c % kS3VStages), (c / kS3VStages) & 1u, abort_flag, p.status))
        break;
      if (lane == 0) {
        tc_fence_before();
        st_release_cta(pv_done, c + 1);
      }
      __syncwarp();
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------- softmax --
    const int t = threadIdx.x;       // row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + kS3ColO;
    const float sl2 = p.scale_log2;
    // Bounded wait until warp 6 has counted `need` retired PVs.
    auto pv_wait = [&](uint32_t need) -> bool {
      if (ld_acquire_cta(pv_done) >= need) return true;
      const uint64_t t0 = globaltimer_ns();
      uint32_t k = 0;
      while (true) {
        if (ld_acquire_cta(pv_done) >= need) return true;
        if ((++k & 15u) == 0) {
          if (*abort_flag) return false;
          if (globaltimer_ns() - t0 > ANIMAXS_WAIT_TIMEOUT_NS) {
            *abort_flag = 1;
            if (p.status) atomicOr(p.status, kStatusTimeout);
            return false;
          }
        }
      }
    };
    bool ok = true;
    uint32_t gt = 0;  // tiles of earlier items (score-buffer uses)
    uint32_t e = 0;   // epilogues done in earlier items
    for (int w = w0; ok && w < p.n_items; w += wstep) {
      const Item I = item_of(w);
      const int row = I.q0 + t;
      const int n = I.n;
      const int valid = I.valid;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const uint32_t tt = gt + j;
        const uint32_t sb = tt % kS3SBufs;
        const uint32_t s_addr = tmem + lane_base + sb * 128;
        ok = mbar_wait(BAR(kS3BarSFull + sb), (tt / kS3SBufs) & 1u, abort_flag, p.status);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t s[4][32];
        tmem_ld32(s_addr + 0, s[0]);
        tmem_ld32(s_addr + 32, s[1]);
        tmem_ld32(s_addr + 64, s[2]);
        tmem_ld32(s_addr + 96, s[3]);
        tmem_ld_wait(s[0]);
        asm volatile("" : AX_RW32(s[1])::"memory");
        asm volatile("" : AX_RW32(s[2])::"memory");
        asm volatile("" : AX_RW32(s[3])::"memory");

        const int key0 = j * kTileN;
        if ((key0 + kTileN > valid) || (p.causal && key0 + kTileN - 1 > row)) {
          const int lim = p.causal ? min(valid, row + 1) : valid;  // keys >= lim are masked
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (key0 + c >= lim) s[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
        // Row max: 8 independent chains of three-input max over 16 values each.
#define SV(c) __uint_as_float(s[(c) >> 5][(c) & 31])
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mx[i] = fmax3(SV(i), SV(i + 8), SV(i + 16));
#pragma unroll
          for (int c = 24; c < 120; c += 16) mx[i] = fmax3(mx[i], SV(c + i), SV(c + 8 + i));
          mx[i] = fmaxf(mx[i], SV(120 + i));
        }
#undef SV
        const float tmax = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                                 fmaxf(mx[6], mx[7])) * sl2;
        const float m_new = fmaxf(m, tmax);
        const bool grow = m_new > m + kRescaleThreshold;  // also true on the first tile
        const float alpha = grow ? ex2_approx(m - m_new) : 1.f;  // 0 on the first tile (m = -inf)
        if (grow) {
          l *= alpha;
          m = m_new;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O must hold PV(0..tt-1) and nothing more: wait until warp 6 has
          // seen them retire (PV(tt) starts only after this warp's arrival
          // below).
          ok = __all_sync(0xffffffffu, pv_wait(tt));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c4 = 0; c4 < HD / 32; ++c4) {
            uint32_t o[32];
            tmem_ld32(o_addr + c4 * 32, o);
            tmem_ld_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + c4 * 32, o);
          }
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        const float2 sl2v = make_float2(sl2, sl2);
        const float2 nmv = make_float2(neg_m, neg_m);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        uint32_t pk[2][32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int c = half * 64; c < half * 64 + 64; c += 2) {
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
            pk[half][(c >> 1) & 31] = pack_half2(pr.x, pr.y);
          }
          tmem_st32(s_addr + half * 32, pk[half]);
        }
        // Publish P (both halves): the warp's stores, then one arrival per warp.
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(kS3BarPFull + sb));
        const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const float2 a = add2(a01, a23);
        l += a.x + a.y;
      }
      if (ok && n > 0) {
        ok = mbar_wait(BAR(kS3BarODone), e & 1u, abort_flag, p.status);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          // Normalise and store O: each warp stages its 32 rows, 64 columns at a
          // time, in the tensor-store layout (16-byte unit u of row r at unit
          // u ^ (r % 8)) and its lane 0 writes them with one TMA store (rows
          // past q_len are clipped by the tensor map).
          tc_fence_after();
          const float inv_l = 1.f / l;
          const uint32_t wstage = base + L::kStage + static_cast<uint32_t>(warp) * 4096u;
          const uint32_t stage = wstage + lane * 128u;
#pragma unroll
          for (int rd = 0; rd < HD / 64; ++rd) {
            uint32_t o[2][32];
            tmem_ld32(o_addr + rd * 64, o[0]);
            tmem_ld32(o_addr + rd * 64 + 32, o[1]);
            tmem_ld_wait(o[0]);
            asm volatile("" : AX_RW32(o[1])::"memory");
            // The stage's previous store (last round or item) has been read.
            if (lane == 0) tma_store_wait_read();
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const uint32_t* ov = &o[u >> 2][(u & 3) * 8];
              st_shared_v4(stage + (((u ^ (lane & 7))) << 4),
                           pack_half2(__uint_as_float(ov[0]) * inv_l, __uint_as_float(ov[1]) * inv_l),
                           pack_half2(__uint_as_float(ov[2]) * inv_l, __uint_as_float(ov[3]) * inv_l),
                           pack_half2(__uint_as_float(ov[4]) * inv_l, __uint_as_float(ov[5]) * inv_l),
                           pack_half2(__uint_as_float(ov[6]) * inv_l, __uint_as_float(ov[7]) * inv_l));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_4d(&tm_o, wstage, 64 * rd, I.q0 + warp * 32, I.h - p.o_head_base, I.b);
              tma_store_commit();
            }
            if (peers_go) {
              // Fused head-sharded gather: the same 32 x 64 tile to the same
              // place in every peer's output over NVLink, 8 lanes per row
              // (128 contiguous bytes), 4 rows per step.  The stage is only
              // read here; the next round rewrites it after the __syncwarp
              // that follows lane 0's wait.
              const int u = lane & 7;
              const long long obase = static_cast<long long>(I.b) * p.o_batch +
                                      static_cast<long long>(I.h - p.o_head_base) * p.o_head + 64 * rd + 8 * u;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int r = 4 * i + (lane >> 3);
                const int grow = I.q0 + warp * 32 + r;
                const uint4 val = ld_shared_v4u(wstage + r * 128u + ((u ^ (r & 7)) << 4));
                if (grow < p.q_len) {
                  char* dst = reinterpret_cast<char*>(p.o + obase + static_cast<long long>(grow) * p.o_tok);
                  for (int pi = 0; pi < p.n_peers; ++pi)
                    *reinterpret_cast<uint4*>(dst + p.peer_delta[pi]) = val;
                }
              }
            }
          }
        }
        ++e;
      }
      gt += n;
    }
  }

  if (warp < 4 && lane == 0) tma_store_wait_all();  // the output stores have completed
  if (peers_go && warp < 4) __threadfence_system();  // peer stores before the arrival below
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, kS3TmemCols);
  }
  if (peers_go && threadIdx.x == 0 && *abort_flag == 0) {
    // This CTA's items are in every peer's output: count them on each peer's
    // arrival word for this rank (a CTA that timed out does not arrive, so the
    // peers' waits report the failure instead of reading a partial output).
    const int mine = static_cast<int>(blockIdx.x) < p.n_items
                         ? (p.n_items - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                         : 0;
    for (int pi = 0; pi < p.n_peers; ++pi) red_add_release_sys(p.peer_arrive[pi], static_cast<unsigned>(mine));
  }
#undef BAR
}

}  // namespace

// One query tile per work item (n_q_tiles = ceil(q_len / 128)); head dim 64
// or 128, no score probe, legacy numerics (launch_attn_fwd checks).
template <int HD>
static cudaError_t launch_s3_hd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                const AttnFwdParams& p, int heads_in_launch, int batch, int dev, int sms,
                                cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  cudaError_t e;
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load(std::memory_order_acquire) & bit) == 0) {
    for (auto fn : {attn_s3_sm100_kernel<HD, false>, attn_s3_sm100_kernel<HD, true>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, S3Smem<HD>::kBytes);
      if (e != cudaSuccess) return e;
    }
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  AttnFwdParams q = p;
  q.heads_in_launch = heads_in_launch;
  q.single_tiles = 1;
  q.n_q_tiles = (p.q_len + kTileM - 1) / kTileM;
  const long long items = static_cast<long long>(q.n_q_tiles) * heads_in_launch * batch;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
  q.n_items = static_cast<int>(items);
  const int grid = static_cast<int>(items < sms ? items : sms);
  // Output view [batch][heads][q_len][HD] for the tensor stores (box 64 x 32).
  CUtensorMap to;
  if (ax_make_tmap(nullptr, &to, p.o, HD, p.q_len, p.head_offset + heads_in_launch - p.o_head_base, batch,
                   p.o_tok, p.o_head, p.o_batch, 32) != ANIMAXS_OK)
    return cudaErrorInvalidValue;
  auto kernel = q.n_peers > 0 ? attn_s3_sm100_kernel<HD, true> : attn_s3_sm100_kernel<HD, false>;
  kernel<<<grid, kS3Threads, S3Smem<HD>::kBytes, stream>>>(tq, tk, tv, to, q);
  return cudaGetLastError();
}

cudaError_t launch_attn_s3(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const AttnFwdParams& p, int heads_in_launch, int batch, int dev, int sms,
                           cudaStream_t stream) {
  if (p.head_dim == 64) return launch_s3_hd<64>(tq, tk, tv, p, heads_in_launch, batch, dev, sms, stream);
  if (p.head_dim == 128) return launch_s3_hd<128>(tq, tk, tv, p, heads_in_launch, batch, dev, sms, stream);
  return cudaErrorInvalidValue;
}

}  // namespace ax
