// attn_fwd_sm100.cu -- flash attention for head_dim 128 on B200 (sm_100a).
//
// Replaces the reference's attention operator (AnimaXS/Runtime/Metal/
// AttentionExecutor.swift:122-302, whose DiT fast path is the Metal kernel
// dit_flash_attention_h128_q4_k32, AnimaKernels.metal:2193-2318, and whose
// general path is MPS QK^T -> attention_softmax_rows (:1051-1100) -> MPS PV).
// Same math: O = softmax(Q K^T * scale + mask) V with fp32 softmax statistics,
// computed as an online (flash) softmax over 128-key tiles.
//
// Persistent: one CTA per SM loops over work items; an item is two 128-row
// query tiles (A: rows q0..q0+127, B: q0+128..q0+255) of one (batch, head),
// both streaming the same K/V tiles.  Items are dealt round-robin (item w to
// CTA w % gridDim.x).  The producer loads the next item's Q, K and V while the
// current item drains, and the next item's first QK runs while the softmax
// warps still store the current item's O, so the per-item start-up (Q load,
// first QK) and epilogue -- measured ~6.5 us per 256-row CTA when every item
// was its own CTA -- overlap with work.  Twelve warps:
//   warps 0-3  softmax for tile A, warps 4-7 softmax for tile B: thread t owns
//              query row t of its tile (= TMEM lane t).  Per K/V tile it reads
//              S from TMEM, applies the causal / key-padding masks, updates the
//              running max (lazily: O is only rescaled when the max grows by
//              more than 2^8) and sum in fp32, and writes P = exp2(S*c - m) as
//              fp16 back into TMEM over the consumed S columns.  At the end it
//              normalises O and stores it.
//   warp 8     MMA issuer + TMEM owner: S_X = Q_X K_j^T (tcgen05.mma kind::f16,
//              both operands in shared memory) and O_X += P_X V_j with P read
//              straight from TMEM (A operand in TMEM).
//   warp 9     TMA producer: both Q tiles once, then K_j / V_j into 2-stage
//              rings, in the order the MMA warp consumes them.
//   warps 10-11 idle (they complete the third warpgroup for setmaxnreg).
// TMEM (512 columns): S_A [0,128), S_B [128,256) (P_X overlays the first 64
// columns of S_X), O_A [256,384), O_B [384,512).
//
// The tensor core alternates PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1): while one
// softmax warpgroup works on its tile, the tensor core runs the other tile's
// MMAs.  P is published in two halves (keys 0-63, 64-127) and PV is issued in
// the matching two halves, so the first half of PV runs while the softmax is
// still computing the second half of P.  tcgen05.mma ops from one thread
// execute in issue order, which is what lets QK_X(j+1) overwrite the TMEM
// columns PV_X(j) reads P_X(j) from.  Barrier phases count tiles and items
// across the whole persistent loop.
//
// Head-sharded calls over several GPUs (p.n_peers > 0) fuse the all-gather
// into the epilogue: each staged output tile is also stored into every peer's
// output over NVLink, and each CTA then adds its item count to every peer's
// arrival word (release, system scope) for the peer's closing wait.
#include <atomic>

#include "api_internal.h"
#include "flash_common.cuh"
#include "kernels.h"

namespace ax {
namespace {

// Ring depths.  A tile load measured ~4000 cycles from issue to arrival under
// full load; two stages each cover it (a third V stage, which still fits in
// 227 KiB, measured no faster).
constexpr int kKStages = 2;
constexpr int kVStages = 2;
// Shared-memory layout for head dim HD (64 or 128): a Q/K/V tile is 128 rows x HD
// fp16 = HD/64 swizzled 64-column panels.
template <int HD>
struct Smem {
  static constexpr uint32_t kTile = kTileM * HD * 2;     // 32 KiB (HD 128) / 16 KiB (HD 64)
  static constexpr uint32_t kQ = 0;                      // Q_A, Q_B
  static constexpr uint32_t kK = kQ + 2 * kTile;
  static constexpr uint32_t kV = kK + kKStages * kTile;
  static constexpr uint32_t kBar = kV + kVStages * kTile;
  // Output stage: per softmax warp, 32 rows x 64 columns fp16 (4 KiB) in the
  // tensor-store layout; 8 warps.
  static constexpr uint32_t kStage = kBar + 1024;
  static constexpr uint32_t kBytes = kStage + 8 * 4096 + 1024;  // + alignment slack
};
constexpr int kThreads = 384;  // warpgroups: softmax A, softmax B, MMA/TMA (+2 idle warps)

enum : int {
  kBarQ = 0,
  kBarKFull = 1,                         // +stage
  kBarKEmpty = kBarKFull + kKStages,     // +stage
  kBarVFull = kBarKEmpty + kKStages,     // +stage
  kBarVEmpty = kBarVFull + kVStages,     // +stage
  kBarSFull = kBarVEmpty + kVStages,     // +tile
  kBarPHalf = kBarSFull + 2,  // +2*tile + half (128 arrivals): P for keys [64*half, 64*half+64) in TMEM
  kBarODone = kBarPHalf + 4,  // +tile: the item's last PV_X retired
  kBarQFree = kBarODone + 2,  // the item's last QK retired: Q may be reloaded
  kBarDone = kBarQFree + 1,
  kNumBars = kBarDone + 1
};
static_assert(kNumBars * 8 + 8 <= 256, "barrier block overflows its 256 bytes");
static_assert(Smem<128>::kBytes <= 227 * 1024, "shared memory exceeds the 227 KiB opt-in");
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;  // O_A at kColO, O_B at kColO + HD
// Register split (setmaxnreg): the kernel launches 3 warpgroups at the
// compiler's per-thread count N (ptxas: 168); the two softmax warpgroups raise
// theirs to AX_SOFTMAX_REGS and the MMA/TMA warpgroup lowers its to
// AX_OTHER_REGS.  2*128*AX_SOFTMAX_REGS + 128*AX_OTHER_REGS must not exceed
// 384*N, or the raise would wait forever: build.py checks this against the
// ptxas report before it links the library.
#define AX_SOFTMAX_REGS 208
#define AX_OTHER_REGS 88

// kProbe: also record the scores' numerical health (animaxs_attn_set_score_probe);
// kFp32P: the FP32_SCORES_AND_SOFTMAX numerics (exp2 on the SFU only, P x V
// from P_hi + P_lo).  Separate instantiations, so that the production kernel
// carries no trace of either.
template <int HD, bool kProbe, bool kFp32P>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_o, const AttnFwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  using L = Smem<HD>;
  constexpr uint32_t kTileBytes = L::kTile;
  const uint32_t sQ = base + L::kQ, sK = base + L::kK, sV = base + L::kV;
  const uint32_t bar0 = base + L::kBar;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + L::kBar + kSlotTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kBar + kSlotAbort);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work item w -> (query-tile pair, head, batch); causal launches take the
  // longest pairs (the last ones) first.
  struct Item {
    int q0, h, b, kvh, valid, nA, nB, n_kv;
  };
  auto item_of = [&](int w) {
    Item it;
    const int pi = w % p.n_q_tiles;
    const int hb = w / p.n_q_tiles;
    const int pair = p.causal ? (p.n_q_tiles - 1 - pi) : pi;
    it.h = p.head_offset + hb % p.heads_in_launch;
    it.b = hb / p.heads_in_launch;
    it.kvh = it.h / p.heads_per_kv;
    // Single-tile items (p.single_tiles): one 128-row tile, processed as tile A.
    it.q0 = pair * (p.single_tiles ? kTileM : 2 * kTileM);
    int valid = p.kv_valid;
    if (p.kv_valid_dev != nullptr) valid = p.kv_valid_dev[it.b];
    it.valid = min(max(valid, 1), p.kv_len);
    it.nA = kv_tiles_for(it.q0, p.q_len, it.valid, p.causal);
    it.nB = p.single_tiles ? 0 : kv_tiles_for(it.q0 + kTileM, p.q_len, it.valid, p.causal);
    it.n_kv = max(it.nA, it.nB);
    return it;
  };
  const int w0 = static_cast<int>(blockIdx.x);
  const int wstep = static_cast<int>(gridDim.x);
  // Fused gather: store into the peers only after a completed handshake.
  const bool peers_go = p.n_peers > 0 && (p.peer_go == nullptr || *p.peer_go == p.peer_go_value);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(BAR(i), (i >= kBarPHalf && i < kBarPHalf + 4) ? 128u : 1u);
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

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(AX_OTHER_REGS));
  if (warp == 9) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int armed_q = 0, armed_k[kKStages] = {}, armed_v[kVStages] = {};
      uint32_t gk = 0, gv = 0;  // K / V tiles loaded so far (ring position)
      // Tile number g of a ring with n stages lives in stage g % n; the wait for
      // a free stage is on the phase its previous occupant's release completed.
      auto load = [&](bool is_k, uint32_t g, int row0, int kvh, int b) -> bool {
        const uint32_t nst = is_k ? kKStages : kVStages;
        const uint32_t st = g % nst;
        const uint32_t ph = (g / nst) & 1u;
        const uint32_t full = BAR((is_k ? kBarKFull : kBarVFull) + st);
        const uint32_t dst = (is_k ? sK : sV) + st * kTileBytes;
        const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
        if (!mbar_wait(BAR((is_k ? kBarKEmpty : kBarVEmpty) + st), ph ^ 1u, abort_flag, p.status))
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
        if (it > 0 && !(ok = mbar_wait(BAR(kBarQFree), static_cast<uint32_t>((it - 1) & 1),
                                       abort_flag, p.status)))
          break;
        // Q_B only when tile B has work (it is never read otherwise).
        const int qt = I.nB > 0 ? 2 : 1;
        mbar_arrive_expect_tx(BAR(kBarQ), qt * kTileBytes);
        for (int x = 0; x < qt; ++x)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_4d(sQ + x * kTileBytes + c * kPanelBytes, &tm_q, BAR(kBarQ), 64 * c,
                        I.q0 + x * kTileM, I.h, I.b);
        ++armed_q;
        // K/V in the order the MMA warp consumes them: K_0, then V_j, K_{j+1}.
        if (!(ok = load(true, gk++, 0, I.kvh, I.b))) break;
        for (int j = 0; ok && j < I.n_kv; ++j) {
          if (!(ok = load(false, gv++, j * kTileN, I.kvh, I.b))) break;
          if (j + 1 < I.n_kv && !(ok = load(true, gk++, (j + 1) * kTileN, I.kvh, I.b))) break;
        }
      }
      // Never leave the CTA with a tensor copy still landing in shared memory:
      // wait (bounded, ignoring the abort flag) for every phase armed above.
      if (armed_q) mbar_wait_drain(BAR(kBarQ), (armed_q - 1) & 1);
      for (int st = 0; st < kKStages; ++st)
        if (armed_k[st]) mbar_wait_drain(BAR(kBarKFull + st), (armed_k[st] - 1) & 1);
      for (int st = 0; st < kVStages; ++st)
        if (armed_v[st]) mbar_wait_drain(BAR(kBarVFull + st), (armed_v[st] - 1) & 1);
    }
  } else if (warp == 8) {
    // ----------------------------------------------------------------- MMA --
    // The whole warp runs this loop (waits, address arithmetic); one elected
    // lane issues each MMA and commit.
    const uint32_t sQA = sQ, sQB = sQ + kTileBytes;
    // Running counters (unsigned: ring stage and phase are bit operations).
    uint32_t gk = 0, gv = 0;  // K / V tiles consumed so far
    uint32_t tA = 0, tB = 0;  // tiles of A / B in earlier items (PHalf phases)
    bool ok = true;
    uint32_t it = 0;
    auto k_full = [&](uint32_t g) {
      return mbar_wait_warp(BAR(kBarKFull + g % kKStages), (g / kKStages) & 1u, abort_flag, p.status);
    };
    for (int w = w0; ok && w < p.n_items; w += wstep, ++it) {
      const Item I = item_of(w);
      const int nA = I.nA, nB = I.nB, n_kv = I.n_kv;
      if (!(ok = mbar_wait_warp(BAR(kBarQ), it & 1u, abort_flag, p.status))) break;
      if (!(ok = k_full(gk))) break;
      tc_fence_after();
      const uint32_t k0 = sK + (gk % kKStages) * kTileBytes;
      if (nA > 0) {
        issue_qk<HD>(tmem + 0, sQA, k0);
        tc_commit_warp(BAR(kBarSFull + 0));
      }
      if (nB > 0) {
        issue_qk<HD>(tmem + 128, sQB, k0);
        tc_commit_warp(BAR(kBarSFull + 1));
      }
      tc_commit_warp(BAR(kBarKEmpty + gk % kKStages));
      ++gk;
      if (n_kv == 1) tc_commit_warp(BAR(kBarQFree));  // the item's last QK
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t vst = gv % kVStages;
        const uint32_t vph = (gv / kVStages) & 1u;
        const int j1 = j + 1;
        const uint32_t vt = sV + vst * kTileBytes;
        const uint32_t kt1 = sK + (gk % kKStages) * kTileBytes;
        if (!(ok = mbar_wait_warp(BAR(kBarVFull + vst), vph, abort_flag, p.status))) break;
        if (j < nA) {
          // An item's first PV overwrites O_A.  The softmax threads publish the
          // item's first P only after their previous epilogue has read O_A out
          // of TMEM, so the PHalf wait below also orders that.
          const uint32_t pph = (tA + j) & 1u;
          if (!(ok = mbar_wait_warp(BAR(kBarPHalf + 0), pph, abort_flag, p.status))) break;
          tc_fence_after();
          issue_pv_half<HD, kFp32P>(tmem + kColO, tmem + 0, vt, 0, j > 0);
          if (!(ok = mbar_wait_warp(BAR(kBarPHalf + 1), pph, abort_flag, p.status))) break;
          tc_fence_after();
          issue_pv_half<HD, kFp32P>(tmem + kColO, tmem + 0, vt, 1, true);
          if (j == nA - 1) tc_commit_warp(BAR(kBarODone + 0));
        }
        if (j1 < n_kv) {
          if (!(ok = k_full(gk))) break;
          tc_fence_after();
        }
        if (j1 < nA) {
          issue_qk<HD>(tmem + 0, sQA, kt1);
          tc_commit_warp(BAR(kBarSFull + 0));
        }
        if (j < nB) {
          const uint32_t pph = (tB + j) & 1u;
          if (!(ok = mbar_wait_warp(BAR(kBarPHalf + 2), pph, abort_flag, p.status))) break;
          tc_fence_after();
          issue_pv_half<HD, kFp32P>(tmem + kColO + HD, tmem + 128, vt, 0, j > 0);
          if (!(ok = mbar_wait_warp(BAR(kBarPHalf + 3), pph, abort_flag, p.status))) break;
          tc_fence_after();
          issue_pv_half<HD, kFp32P>(tmem + kColO + HD, tmem + 128, vt, 1, true);
          if (j == nB - 1) tc_commit_warp(BAR(kBarODone + 1));
        }
        // V_j's last reader has been issued: release its stage now (the commit
        // fires when PV_B(j) retires), not after QK_B(j+1).
        tc_commit_warp(BAR(kBarVEmpty + vst));
        ++gv;
        if (j1 < nB) {
          issue_qk<HD>(tmem + 128, sQB, kt1);
          tc_commit_warp(BAR(kBarSFull + 1));
        }
        if (j1 < n_kv) {
          tc_commit_warp(BAR(kBarKEmpty + gk % kKStages));
          ++gk;
          if (j1 == n_kv - 1) tc_commit_warp(BAR(kBarQFree));  // the item's last QK
        }
      }
      tA += nA;
      tB += nB;
    }
    // All MMAs this warp issued must retire before TMEM is released.
    tc_commit_warp(BAR(kBarDone));
    mbar_wait_drain(BAR(kBarDone), 0);
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(AX_SOFTMAX_REGS));
    // ------------------------------------------------------------- softmax --
    const int X = warp >> 2;              // 0: tile A, 1: tile B
    const int t = threadIdx.x & 127;      // row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + X * 128;
    const uint32_t o_addr = tmem + lane_base + kColO + X * HD;
    const float sl2 = p.scale_log2;
    bool ok = true;
    uint32_t tX = 0;  // tiles of this query tile processed in earlier items
    uint32_t eX = 0;  // epilogues done in earlier items
    for (int w = w0; ok && w < p.n_items; w += wstep) {
      const Item I = item_of(w);
      const int row = I.q0 + X * kTileM + t;
      const int nX = X ? I.nB : I.nA;
      const int valid = I.valid;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < nX; ++j) {
        ok = mbar_wait(BAR(kBarSFull + X), (tX + j) & 1u, abort_flag, p.status);
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
        if constexpr (kProbe) {
          // Score health over this row's unmasked keys, as the reference's
          // attention_softmax_rows_probe (AnimaKernels.metal:1738-1830) records
          // it for the scaled scores: flags, max |score|, first flagged key.
          const int lim = p.causal ? min(valid, row + 1) : valid;
          const float scale = sl2 * 0.6931471805599453f;  // scale_log2 / log2(e)
          unsigned int pf = 0u, pmax = 0u, pfirst = 0xFFFFFFFFu;
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const float sv = __uint_as_float(s[c >> 5][c & 31]);
            if (key0 + c < lim) {
              unsigned int f = 0u;
              if (sv != sv) {
                f = 1u;
              } else if (isinf(sv)) {
                f = sv > 0.f ? 2u : 4u;
              } else {
                const float a = fabsf(sv) * scale;
                if (a > 65504.f) f = 8u;
                pmax = max(pmax, __float_as_uint(a));
              }
              if (f != 0u) {
                pf |= f;
                pfirst = min(pfirst, static_cast<unsigned int>(key0 + c));
              }
            }
          }
          pf = __reduce_or_sync(0xffffffffu, pf);
          pmax = __reduce_max_sync(0xffffffffu, pmax);
          pfirst = __reduce_min_sync(0xffffffffu, pfirst);
          if (lane == 0) {
            if (pf != 0u) {
              atomicOr(p.probe, pf);
              atomicMin(p.probe + 2, pfirst);
            }
            if (pmax != 0u) atomicMax(p.probe + 1, pmax);
          }
        }
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
          // PV_X(j-1) precedes QK_X(j) in the MMA stream, so it has retired and O
          // is stable; PV_X(j) starts only after this thread's first arrival below.
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
          uint32_t pl[kFp32P ? 32 : 1];
#pragma unroll
          for (int c = half * 64; c < half * 64 + 64; c += 2) {
            const float2 x = fma2(make_float2(__uint_as_float(s[c >> 5][c & 31]),
                                              __uint_as_float(s[c >> 5][(c + 1) & 31])),
                                  sl2v, nmv);
            float2 pr;
            if (!kFp32P && ((c >> 1) & 7) < kPolyPairsPer8) {
              pr = ex2_poly2(x);
            } else {
              pr.x = ex2_approx(x.x);
              pr.y = ex2_approx(x.y);
            }
            acc[(c >> 1) & 3] = add2(acc[(c >> 1) & 3], pr);
            pk[half][(c >> 1) & 31] = pack_half2(pr.x, pr.y);
            if constexpr (kFp32P) {
              // P_lo = fp16(P - P_hi); the difference is exact in fp32.
              const float2 hv = __half22float2(*reinterpret_cast<const __half2*>(&pk[half][(c >> 1) & 31]));
              pl[(c >> 1) & 31] = pack_half2(__fsub_rn(pr.x, hv.x), __fsub_rn(pr.y, hv.y));
            }
          }
          // Publish this half of P: the MMA warp starts its half of PV_X(j) while
          // the second half is still being computed.  (P_lo of keys [64h, 64h+64)
          // lands in S columns [64+32h, 96+32h), whose scores this thread
          // already holds in registers.)
          tmem_st32(s_addr + half * 32, pk[half]);
          if constexpr (kFp32P) tmem_st32(s_addr + 64 + half * 32, pl);
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(BAR(kBarPHalf + 2 * X + half));
        }
        const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const float2 a = add2(a01, a23);
        l += a.x + a.y;
      }
      if (ok && nX > 0) {
        ok = mbar_wait(BAR(kBarODone + X), eX & 1u, abort_flag, p.status);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          // Normalise and store O: each warp stages its 32 rows, 64 columns at a
          // time, in the tensor-store layout (16-byte unit u of row r at unit
          // u ^ (r % 8)) and its lane 0 writes them with one TMA store (rows
          // past q_len are clipped by the tensor map).  No cross-warp sync.
          tc_fence_after();
          const float inv_l = 1.f / l;
          const uint32_t stage = base + L::kStage + static_cast<uint32_t>(warp) * 4096u + lane * 128u;
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
              tma_store_4d(&tm_o, base + L::kStage + static_cast<uint32_t>(warp) * 4096u, 64 * rd,
                           I.q0 + X * kTileM + (warp & 3) * 32, I.h - p.o_head_base, I.b);
              tma_store_commit();
            }
            if (peers_go) {
              // Fused head-sharded gather: the same 32 x 64 tile to the same
              // place in every peer's output over NVLink, 8 lanes per row
              // (128 contiguous bytes), 4 rows per step.  The stage is only
              // read here; the next round rewrites it after the __syncwarp
              // that follows lane 0's wait.
              const uint32_t wstage = base + L::kStage + static_cast<uint32_t>(warp) * 4096u;
              const int u = lane & 7;
              const long long obase = static_cast<long long>(I.b) * p.o_batch +
                                      static_cast<long long>(I.h - p.o_head_base) * p.o_head + 64 * rd + 8 * u;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int r = 4 * i + (lane >> 3);
                const int grow = I.q0 + X * kTileM + (warp & 3) * 32 + r;
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
        ++eX;
      }
      tX += nX;
    }
  }

  if (warp < 8 && lane == 0) tma_store_wait_all();  // the output stores have completed
  if (peers_go && warp < 8) __threadfence_system();  // peer stores before the arrival below
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

int attn_fwd_rows_per_cta() { return 2 * kTileM; }

// Work items of a launch.  An item is normally a pair of 128-row query tiles
// sharing one K/V stream; when the pairs would leave more than half of the SMs
// idle, items are single tiles: twice the CTAs, so the launch finishes sooner.
// Such launches run attn_s3_sm100.cu (below); the single-tile items of this
// kernel (the score probe, fp32 numerics) leave the second softmax warpgroup
// idle.  A launch whose output tiles also go to peer GPUs deals single tiles
// as soon as the pairs alone would leave SMs idle: the pairs would all finish
// at once and expose the whole gather, while single tiles take two waves and
// the first wave's peer stores overlap the second wave.  Every row's
// arithmetic is the same in all forms, so the output is bit-identical.
static bool single_tile_items(int q_len, int heads_in_launch, int batch, int sms, bool peers) {
  const long long pairs = (q_len + 2 * kTileM - 1) / (2 * kTileM) * static_cast<long long>(heads_in_launch) * batch;
  return 2 * pairs <= sms || (peers && pairs < sms);
}
long long attn_fwd_work_items(int q_len, int heads_in_launch, int batch, int sms, bool peers) {
  const int rows = single_tile_items(q_len, heads_in_launch, batch, sms, peers) ? kTileM : 2 * kTileM;
  return static_cast<long long>((q_len + rows - 1) / rows) * heads_in_launch * batch;
}

template <int HD>
static cudaError_t launch_hd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnFwdParams& p, int heads_in_launch, int batch, int dev,
                             cudaStream_t stream) {
  // The dynamic shared-memory opt-in is a per-device function attribute.
  static std::atomic<uint64_t> configured{0};
  cudaError_t e;
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load(std::memory_order_acquire) & bit) == 0) {
    for (auto fn : {attn_fwd_sm100_kernel<HD, false, false>, attn_fwd_sm100_kernel<HD, true, false>,
                    attn_fwd_sm100_kernel<HD, false, true>, attn_fwd_sm100_kernel<HD, true, true>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<HD>::kBytes);
      if (e != cudaSuccess) return e;
    }
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  // Persistent grid: one CTA per SM (at most one per work item).
  static std::atomic<int> sm_count[64];
  int sms = sm_count[dev & 63].load(std::memory_order_relaxed);
  if (sms == 0) {
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sm_count[dev & 63].store(sms, std::memory_order_relaxed);
  }
  const bool single = single_tile_items(p.q_len, heads_in_launch, batch, sms, p.n_peers > 0);
  // Single-tile launches go to attn_s3_sm100.cu, whose one
  // query tile per CTA has three score buffers, so its softmax never waits for
  // the tensor core (config 1: 24.4 -> 20.6 us, a Qwen layer 15.0 -> 13.8 us;
  // same bits).  Paired launches stay here: with one softmax warp per SM
  // sub-partition the other kernel cannot hide its own latencies the way two
  // warpgroups hide each other's (batch-8 DiT self-attention 1035 vs 1104 us).
  if (single && p.probe == nullptr && !p.fp32_p)
    return launch_attn_s3(tq, tk, tv, p, heads_in_launch, batch, dev, sms, stream);
  AttnFwdParams q = p;
  q.heads_in_launch = heads_in_launch;
  q.single_tiles = single ? 1 : 0;
  q.n_q_tiles = (p.q_len + (q.single_tiles ? kTileM : 2 * kTileM) - 1) / (q.single_tiles ? kTileM : 2 * kTileM);
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
  auto kernel = q.probe != nullptr ? (q.fp32_p ? attn_fwd_sm100_kernel<HD, true, true>
                                                : attn_fwd_sm100_kernel<HD, true, false>)
                                   : (q.fp32_p ? attn_fwd_sm100_kernel<HD, false, true>
                                               : attn_fwd_sm100_kernel<HD, false, false>);
  kernel<<<grid, kThreads, Smem<HD>::kBytes, stream>>>(tq, tk, tv, to, q);
  return cudaGetLastError();
}

cudaError_t launch_attn_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const AttnFwdParams& p, int heads_in_launch, int batch,
                            cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (p.head_dim == 64) return launch_hd<64>(tq, tk, tv, p, heads_in_launch, batch, dev, stream);
  if (p.head_dim == 128) return launch_hd<128>(tq, tk, tv, p, heads_in_launch, batch, dev, stream);
  return launch_attn_wide(tq, tk, tv, p, heads_in_launch, batch, dev, stream);
}

}  // namespace ax
