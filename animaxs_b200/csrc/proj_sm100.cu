// proj_sm100.cu -- the GEMMs on either side of DiT attention, with their
// elementwise steps fused into the epilogue (B200, sm_100a).
//
// The reference runs, per attention branch (DiTBlockExecutor.swift:1097-1131,
// 1223-1236): LinearExecutor.encode (fp16 x fp16 -> fp16 projection,
// LinearExecutor.swift:79-) for q, k and v, then rms_rope_split_half /
// rmsnorm_heads_half on q and k (AnimaKernels.metal:660-729); after attention
// the out-projection, then gate_add_half_f32 (AnimaKernels.metal:624-634:
// residual[i] += float(branch[i]) * gate[i % N], fp32 residual and gate).
// Here each of those is one kernel: out = x w^T (x [m, k] and w [n, k] fp16,
// K-major; fp32 accumulation in TMEM) with the epilogue
//   kProjStore    out fp16 = fp16(acc)
//   kProjQkvNorm  columns [0, q_cols) / [q_cols, q_cols + k_cols) are q / k
//                 heads of 128: y = fp16(acc), then RMSNorm with fp32
//                 statistics rsqrt(mean(y^2) + eps) and a shared [128]
//                 weight, then the split-half RoPE of pairs (p, p + 64) from
//                 [token][64][2][2] blocks [cos, -sin, sin, cos] (re-laid out
//                 pair-major by rope_pairs_kernel first); the remaining
//                 columns (v) are stored as fp16(acc)
//   kProjGateAdd  residual fp32 += float(fp16(acc)) * gate[row / tokens][col],
//                 written with TMA reduce-add (no read of the residual by the SMs)
// A 128-column half of an output tile is exactly one head, so the norm and
// the rotation need nothing beyond the thread's own row.
//
// CTA pairs.  A 128 x 256 tile per SM needs ~96 B/clk of operands from L2 at
// full tensor rate, above what L2 delivers (~53 B/clk/SM measured), so two
// CTAs of a cluster run as one tcgen05 CTA pair (cta_group::2) on 256 x 256
// tiles: the pair leader issues M = 256, N = 256 MMAs whose A rows (x) come
// from both CTAs and whose B (w) is split along N, so each CTA loads its own
// 128 rows of x and half of the tile's w rows -- 32 KiB per K-slice of 64
// instead of 48 for the same work.  The copies of both CTAs complete on the
// leader's barriers (armed by the leader for both halves); MMA completions are
// committed to both CTAs' barriers.
//
// Persistent: each pair walks 256 x 256 output tiles (row-major over the tile
// grid).  Twelve warps per CTA: warp 0 TMA producer (6-stage ring), warp 1
// TMEM owner and, in the leader, MMA issuer (4 MMAs per stage), warps 4-11
// epilogue of the CTA's 128 rows (two threads per row = TMEM lane, each holding
// half of every head's columns).  Two 256-column TMEM accumulators alternate,
// so a tile's epilogue runs while the next tile accumulates; the epilogue
// warps of both CTAs release an accumulator on the leader's barrier.  Outputs
// leave through a 32 KiB shared-memory stage in the tensor-store layout (TMA
// stores / reduce-adds; rows and columns past the matrix are clipped by the
// tensor map).
#include <atomic>

#include "flash_common.cuh"
#include "kernels.h"

namespace ax {
namespace {

constexpr int kBM = 128;   // rows per CTA (256 per pair)
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 6;
constexpr int kThreads = 384;       // warpgroup 0: TMA warp, MMA warp (+2 idle); warpgroups 1-2: epilogue
constexpr int kEpiThreads = 256;
// Register split (setmaxnreg): the kernel launches at the compiler's per-thread
// count N (ptxas: 168); the epilogue warpgroups raise theirs to AX_EPI_REGS and
// warpgroup 0 lowers its to AX_PROJ_OTHER_REGS.  256*AX_EPI_REGS +
// 128*AX_PROJ_OTHER_REGS must not exceed 384*N, or the raise would wait
// forever: build.py checks this against the ptxas report.
#define AX_EPI_REGS 208
#define AX_PROJ_OTHER_REGS 56
constexpr uint32_t kABytes = kBM * kBK * 2;        // 16 KiB: this CTA's 128 rows of x
constexpr uint32_t kBBytes = (kBN / 2) * kBK * 2;  // 16 KiB: this CTA's half of the tile's w rows
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kOut = kStages * kStageBytes;  // 192 KiB
constexpr uint32_t kOutBytes = 32768;             // output stage
constexpr uint32_t kBar = kOut + kOutBytes;
constexpr uint32_t kXss = kBar + 256;             // [2][128] fp32 row sums of squares
constexpr uint32_t kSmemBytes = kXss + 1024 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds the 227 KiB opt-in");

enum : int {
  kBarFull = 0,                      // +stage
  kBarEmpty = kBarFull + kStages,    // +stage
  kBarAccFull = kBarEmpty + kStages, // +accumulator
  kBarAccEmpty = kBarAccFull + 2,    // +accumulator, leader: 16 arrivals (epilogue warps of both CTAs)
  kBarDone = kBarAccEmpty + 2,
  kNumBars
};
constexpr uint32_t kSlotTmem = kNumBars * 8;
constexpr uint32_t kSlotAbort = kSlotTmem + 4;
static_assert(kSlotAbort + 4 <= 256, "barrier block overflows its 256 bytes");
constexpr uint32_t kIdesc = idesc_f16_f32(2 * kBM, kBN, false);  // pair MMA: M 256, N 256
constexpr uint32_t kEpiBar = 1;   // named barrier of the 8 epilogue warps

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

__global__ void __launch_bounds__(kThreads, 1)
    proj_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_out, const ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + kBar;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + kBar + kSlotTmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kBar + kSlotAbort);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_blocks = (p.k + kBK - 1) / kBK;
  // Cluster (2, 1, 1): rank 0 leads the pair; rank c holds rows [128c, 128c + 128)
  // of every 256-row tile and w rows [128c, 128c + 128) of its 256 columns.
  const int cid = static_cast<int>(cluster_ctarank());
  const int pair = static_cast<int>(blockIdx.x) >> 1;
  const int pairs = static_cast<int>(gridDim.x) >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(BAR(i), (i >= kBarAccEmpty && i < kBarAccEmpty + 2) ? 16u : 1u);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc2(bar0 + kSlotTmem, 512);
    tmem_relinquish2();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_out);
  }
  // Both CTAs' barriers exist (and TMEM is allocated) before any copy or
  // arrival targets the leader's.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(AX_PROJ_OTHER_REGS));
  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.tiles; t += pairs) {
        const int m0 = (t / p.tiles_n) * 2 * kBM, n0 = (t % p.tiles_n) * kBN;
        for (int kb = 0; kb < k_blocks; ++kb, ++g) {
          const uint32_t st = g % kStages;
          if (!(ok = mbar_wait(BAR(kBarEmpty + st), ((g / kStages) & 1u) ^ 1u, abort_flag, p.status))) break;
          const uint32_t sa = base + st * kStageBytes;
          const uint32_t full = mapa_shared(BAR(kBarFull + st), 0);
          if (cid == 0) mbar_arrive_expect_tx(BAR(kBarFull + st), 2 * kStageBytes);
          tma_load_2d_pair(sa, &tm_a, full, kb * kBK, m0 + cid * kBM);
          tma_load_2d_pair(sa + kABytes, &tm_b, full, kb * kBK, n0 + cid * (kBN / 2));
        }
      }
      // The copies complete on the leader's barriers.  Normally every one was
      // consumed by an MMA that retired before Done; after an abort, give the
      // ones still in flight time to land before the CTA may exit.
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 100000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    uint32_t g = 0;
    bool ok = true;
    int it = 0;
    for (int t = pair; cid == 0 && ok && t < p.tiles; t += pairs, ++it) {
      const uint32_t acc = it & 1;
      // The epilogue has drained this accumulator (its previous use, two tiles ago).
      if (!(ok = mbar_wait_warp(BAR(kBarAccEmpty + acc), ((it >> 1) & 1u) ^ 1u, abort_flag, p.status))) break;
      tc_fence_after();
      const uint32_t d = tmem + acc * kBN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const uint32_t st = g % kStages;
        if (!(ok = mbar_wait_warp(BAR(kBarFull + st), (g / kStages) & 1u, abort_flag, p.status))) break;
        tc_fence_after();
        const uint32_t sa = base + st * kStageBytes;
        const uint64_t a0 = sw128_desc(sa, 16, 1024), b0 = sw128_desc(sa + kABytes, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma2_f16_ss_warp(d, a0 + static_cast<uint64_t>(kk * 2), b0 + static_cast<uint64_t>(kk * 2), kIdesc,
                            (kb > 0 || kk > 0) ? 1u : 0u);
        tc_commit2_mc_warp(BAR(kBarEmpty + st), 3);
      }
      if (!ok) break;
      tc_commit2_mc_warp(BAR(kBarAccFull + acc), 3);
    }
    // Every MMA of the pair retires before either CTA releases TMEM or exits.
    if (cid == 0) tc_commit2_mc_warp(BAR(kBarDone), 3);
    mbar_wait_drain(BAR(kBarDone), 0);
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(AX_EPI_REGS));
    // ------------------------------------------------------------ epilogue --
    // Eight warps (4-11): warp w reads TMEM lanes [32(w%4), 32(w%4) + 32) (thread =
    // output row); `half` splits every 128-column head so that each thread
    // holds complete rotation pairs: columns [32 half, 32 half + 32) and
    // [64 + 32 half, 64 + 32 half + 32).  The two threads of a row exchange
    // only their sums of squares.
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;               // 0: warps 4-7, 1: warps 8-11
    const int r = quarter * 32 + lane;              // row within the tile
    const int et = threadIdx.x - 128;               // 0..255 over the epilogue warps
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool leader = (et == 0);                  // issues the tensor stores
    const uint32_t sOut = base + kOut;
    volatile float* xss = reinterpret_cast<volatile float*>(gbase + kXss);  // [2][128] sums of squares
    const uint32_t acc_empty0 = mapa_shared(BAR(kBarAccEmpty), 0);  // the leader's
    bool ok = true;
    int it = 0;
    for (int t = pair; t < p.tiles; t += pairs, ++it) {
      const uint32_t acc = it & 1;
      const int m0 = (t / p.tiles_n) * 2 * kBM + cid * kBM, n0 = (t % p.tiles_n) * kBN;
      const int row = m0 + r;
      bool got = ok && mbar_wait(BAR(kBarAccFull + acc), (it >> 1) & 1u, abort_flag, p.status);
      got = __all_sync(0xffffffffu, got);
      ok = got;
      tc_fence_after();
      // This thread's 32 rotation blocks (cos, sin), shared by the tile's two heads.
      float cs[32], sn[32];
      const bool rope_tile = p.mode == kProjQkvNorm && p.rope != nullptr && n0 < p.q_cols + p.k_cols;
      if (rope_tile && row < p.m) {
        // Pair-major (cos, sin) table: a warp's 32 consecutive rows read 256
        // contiguous bytes per pair.
        const float2* tab = reinterpret_cast<const float2*>(p.rope) +
                            static_cast<long long>(half * 32) * p.tokens + row % p.tokens;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 cv = __ldg(tab + static_cast<long long>(i) * p.tokens);
          cs[i] = cv.x;
          sn[i] = cv.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) cs[i] = sn[i] = 0.f;
      }
      for (int h = 0; h < kBN / 128; ++h) {
        const int c0 = n0 + h * 128;                // first column of this head
        float x[64];                                // [0,32): cols 32 half + i; [32,64): cols 64 + 32 half + i
        if (got) {
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + acc * kBN + h * 128 + q2 * 64 + half * 32, v);
            tmem_ld_wait(v);
#pragma unroll
            for (int i = 0; i < 32; ++i) x[q2 * 32 + i] = round_f16(__uint_as_float(v[i]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) x[i] = 0.f;
        }
        if (h == kBN / 128 - 1) {
          // Both heads are in registers: the accumulator may take the next tile.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * acc);
        }
        if (p.mode == kProjGateAdd) {
          // fp32 through the stage in two 64-column rounds, each two 32-column
          // boxes (128 B rows, 128-byte swizzle) added into the residual by TMA;
          // in round q2 this thread holds box `half` (columns q2*64 + 32 half + [0,32)).
          const int img = row / p.tokens;
          const float* gate = p.gate + static_cast<long long>(img) * p.gate_stride;
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int cb = q2 * 64 + half * 32;     // first column (in the head) of this thread's block
            named_bar_sync(kEpiBar, kEpiThreads);   // the previous round's reduce has read the stage
#pragma unroll
            for (int u = 0; u < 8; ++u) {           // 16-byte unit u of the thread's 32 columns
              float gv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                gv[e] = (row < p.m && c0 + cb + 4 * u + e < p.n) ? __ldg(gate + c0 + cb + 4 * u + e) : 0.f;
              const uint32_t addr = sOut + half * 16384 + r * 128 + (((u ^ (r & 7))) << 4);
              st_shared_v4(addr, __float_as_uint(x[q2 * 32 + 4 * u] * gv[0]),
                           __float_as_uint(x[q2 * 32 + 4 * u + 1] * gv[1]),
                           __float_as_uint(x[q2 * 32 + 4 * u + 2] * gv[2]),
                           __float_as_uint(x[q2 * 32 + 4 * u + 3] * gv[3]));
            }
            fence_proxy_async_smem();
            named_bar_sync(kEpiBar, kEpiThreads);
            if (leader && got) {
              for (int bx = 0; bx < 2; ++bx)
                if (c0 + q2 * 64 + bx * 32 < p.n)
                  tma_reduce_add_2d(&tm_out, sOut + bx * 16384, c0 + q2 * 64 + bx * 32, m0);
              tma_store_commit();
              tma_store_wait_read();
            }
          }
          continue;
        }
        bool head_q = false, head_k = false;
        if (p.mode == kProjQkvNorm) {
          head_q = c0 < p.q_cols;
          head_k = !head_q && c0 < p.q_cols + p.k_cols;
        }
        if (head_q || head_k) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) ss = fmaf(x[32 + i], x[32 + i], fmaf(x[i], x[i], ss));
          xss[half * 128 + r] = ss;
          named_bar_sync(kEpiBar, kEpiThreads);
          ss += xss[(half ^ 1) * 128 + r];
          const float inv = rsqrtf(ss * (1.0f / 128) + p.eps);
          const __half* w = head_q ? p.q_w : p.k_w;
          if (w != nullptr) {
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2)
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(w + q2 * 64 + half * 32 + i));
                x[q2 * 32 + i] *= inv * wf.x;
                x[q2 * 32 + i + 1] *= inv * wf.y;
              }
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) x[i] *= inv;
          }
          if (rope_tile) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float a = x[i], b = x[32 + i];
              x[i] = cs[i] * a - sn[i] * b;
              x[32 + i] = sn[i] * a + cs[i] * b;
            }
          }
        } else {
          named_bar_sync(kEpiBar, kEpiThreads);  // the previous head's store has read the stage
        }
        // Stage the head as fp16 in the store layout: two 64-column panels of
        // 128 rows x 128 B, 16-byte unit u of row r at unit u ^ (r % 8); this
        // thread's columns are units [4 half, 4 half + 4) of both panels.  (For
        // a normalised head the exchange barrier above ordered the previous
        // head's store before these writes; the exchange slot is rewritten only
        // after the next barrier.)
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2)
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int uu = half * 4 + u;
            const float* xv = x + q2 * 32 + 8 * u;
            st_shared_v4(sOut + q2 * 16384 + r * 128 + (((uu ^ (r & 7))) << 4),
                         pack_half2(xv[0], xv[1]), pack_half2(xv[2], xv[3]), pack_half2(xv[4], xv[5]),
                         pack_half2(xv[6], xv[7]));
          }
        fence_proxy_async_smem();
        named_bar_sync(kEpiBar, kEpiThreads);
        if (leader && got) {
          for (int pn = 0; pn < 2; ++pn)
            if (c0 + pn * 64 < p.n) tma_store_2d(&tm_out, sOut + pn * 16384, c0 + pn * 64, m0);
          tma_store_commit();
          tma_store_wait_read();
        }
      }
    }
    if (leader) tma_store_wait_all();
  }

  // Neither CTA of the pair releases TMEM while the other may still use it.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, 512);
  }
#undef BAR
}

// [rows][64][2][2] rotation blocks [cos, -sin, sin, cos] -> pair-major
// [64][rows] (cos, sin), the layout the epilogue reads.
__global__ void rope_pairs_kernel(const float4* __restrict__ in, float2* __restrict__ out, int rows) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(rows) * 64) return;
  const int pair = static_cast<int>(i / rows), row = static_cast<int>(i % rows);
  const float4 blk = __ldg(in + static_cast<long long>(row) * 64 + pair);
  out[i] = make_float2(blk.x, blk.z);
}

}  // namespace

cudaError_t launch_rope_pairs(const float* table, void* out, int rows, cudaStream_t stream) {
  const long long n = static_cast<long long>(rows) * 64;
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  rope_pairs_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const float4*>(table),
                                                 static_cast<float2*>(out), rows);
  return cudaGetLastError();
}

cudaError_t launch_proj(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tout,
                        const ProjParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load(std::memory_order_acquire) & bit) == 0) {
    e = cudaFuncSetAttribute(proj_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
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
  if (p.tiles <= 0) return cudaSuccess;
  const int pairs = p.tiles < sms / 2 ? p.tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, proj_sm100_kernel, ta, tb, tout, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int proj_kernel_attributes(int* regs, int* max_threads, int* smem_static, int* smem_dynamic_max) {
  cudaFuncAttributes a{};
  if (cudaFuncGetAttributes(&a, proj_sm100_kernel) != cudaSuccess) return -1;
  *regs = a.numRegs;
  *max_threads = a.maxThreadsPerBlock;
  *smem_static = static_cast<int>(a.sharedSizeBytes);
  *smem_dynamic_max = a.maxDynamicSharedSizeBytes;
  return 0;
}

}  // namespace ax
