// noalloc.cu -- animaxs_attn_forward_noalloc: the fused attention call for
// callers that must not allocate device memory.
//
// Some callers cannot let a library call cudaMalloc: an application that
// reserves the whole device budget at start-up (weights, caches) and treats any
// later allocation as a failure; a host runtime whose own allocator has to own
// every device allocation; a latency-critical loop where an allocation (which
// can synchronise the device and take milliseconds) is not acceptable.  For
// them this entry point runs the same prologue + flash-attention kernels as
// animaxs_attn_forward, but the prologue's normalised q/k copies live in a
// fixed, file-scope device array instead of context-owned cudaMalloc'd scratch.
//
// Limits and sharing:
//  - The array is kNoAllocScratchBytes (32 MiB) on every GPU that loads the
//    library, held until the process exits.  A call whose normalised q/k need
//    more (animaxs_attn_scratch_bytes) is rejected with
//    ANIMAXS_ERR_SCRATCH_LIMIT before anything is launched.
//  - Every call on a device shares the one array and it keeps the previous
//    call's contents.  Nothing in it has to start at zero: the prologue
//    overwrites every byte the attention kernel later reads.  Calls that
//    overlap on the GPU (different streams, or different host threads) race on
//    the array; serialise them.
//  - In host code the array's name is not a device address.  The device
//    address is looked up once per device with cudaGetSymbolAddress, with that
//    device current, on the first call made on it; make that first call before
//    any stream capture.  The address is kept for the life of the process: after
//    cudaDeviceReset (or any teardown of the device's primary context) it is
//    stale, so do not use this entry point across a device reset.
//  - No context is involved, so there is no last-error text.  A device-side
//    wait that expires sets a second file-scope word (looked up like the
//    array), which animaxs_attn_noalloc_status reads and clears.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "../../include/animaxs_attn.h"
#include "api_internal.h"
#include "kernels.h"

namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t{32} << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Timeout bit of the kernels' bounded waits for calls made here.
static __device__ unsigned int g_noalloc_status;

constexpr int kMaxDevices = 64;

struct Symbols {
  void* scratch;
  unsigned int* status;
};

// Device addresses of g_noalloc_scratch / g_noalloc_status on `dev` (which
// must be current), looked up on the first call made on that device.
int symbol_addresses(int dev, Symbols* out) {
  static std::mutex mu;
  static Symbols addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return ANIMAXS_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev].scratch == nullptr) {
    void* p = nullptr;
    void* st = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess || p == nullptr || st == nullptr) {
      cudaGetLastError();
      return ANIMAXS_ERR_CUDA;
    }
    addr[dev] = Symbols{p, static_cast<unsigned int*>(st)};
  }
  *out = addr[dev];
  return ANIMAXS_OK;
}

}  // namespace

extern "C" int animaxs_attn_forward_noalloc(const animaxs_attn_desc* d, const void* q,
                                            const void* k, const void* v, void* o,
                                            void* stream_) {
  AxRange range("animaxs_attn_forward_noalloc");
  int rc = ax_validate(nullptr, d, q, k, v, o);
  if (rc != ANIMAXS_OK) return rc;
  int64_t need = 0;
  animaxs_attn_scratch_bytes(d, &need);
  if (need > kNoAllocScratchBytes) return ANIMAXS_ERR_SCRATCH_LIMIT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ANIMAXS_ERR_NO_DEVICE;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
      major != 10 || minor != 0)
    return ANIMAXS_ERR_NO_DEVICE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Symbols sym{};
  rc = symbol_addresses(dev, &sym);
  if (rc != ANIMAXS_OK) return rc;

  const int64_t D = d->head_dim;
  const void* qa = q;
  const void* ka = k;
  int64_t q_st = d->q_tok_stride, q_sh = d->q_head_stride, q_sb = d->q_batch_stride;
  int64_t k_st = d->k_tok_stride, k_sh = d->k_head_stride, k_sb = d->k_batch_stride;
  if (d->qk_norm != ANIMAXS_QK_NONE) {
    // Layout as animaxs_attn_scratch_bytes counts it: q's copy (when q is
    // normalised here), then k's at the next 256-byte boundary.
    const bool q_here = d->qk_norm_targets != ANIMAXS_QK_NORM_K_ONLY;
    const int64_t q_bytes = q_here ? static_cast<int64_t>(d->batch) * d->q_len * d->heads * D * 2 : 0;
    __half* qn = static_cast<__half*>(sym.scratch);
    __half* kn = reinterpret_cast<__half*>(static_cast<char*>(sym.scratch) +
                                           ((q_bytes + 255) & ~static_cast<int64_t>(255)));
    ax::NormParams np{};
    np.head_dim = static_cast<int>(d->head_dim);
    np.eps = d->eps > 0.f ? d->eps : 1e-6f;
    np.rope = d->qk_norm == ANIMAXS_QK_RMS_ROPE ? d->rope_table : nullptr;
    ax::NormJob& jq = np.job[0];
    jq.in = static_cast<const __half*>(q);
    jq.out = qn;
    jq.in_tok = q_st;
    jq.in_head = q_sh;
    jq.in_batch = q_sb;
    jq.out_tok = static_cast<int64_t>(d->heads) * D;
    jq.out_head = D;
    jq.out_batch = static_cast<int64_t>(d->q_len) * d->heads * D;
    jq.tokens = d->q_len;
    jq.heads = d->heads;
    jq.batch = d->batch;
    jq.weight = static_cast<const __half*>(d->q_norm_weight);
    jq.rows = static_cast<int64_t>(d->batch) * d->q_len * d->heads;
    ax::NormJob& jk = np.job[1];
    jk.in = static_cast<const __half*>(k);
    jk.out = kn;
    jk.in_tok = k_st;
    jk.in_head = k_sh;
    jk.in_batch = k_sb;
    jk.out_tok = static_cast<int64_t>(d->kv_heads) * D;
    jk.out_head = D;
    jk.out_batch = static_cast<int64_t>(d->kv_len) * d->kv_heads * D;
    jk.tokens = d->kv_len;
    jk.heads = d->kv_heads;
    jk.batch = d->batch;
    jk.weight = static_cast<const __half*>(d->k_norm_weight);
    jk.rows = static_cast<int64_t>(d->batch) * d->kv_len * d->kv_heads;
    // The caller may hold an already normalised q or k (qk_norm_targets).
    const bool norm_q = d->qk_norm_targets != ANIMAXS_QK_NORM_K_ONLY;
    const bool norm_k = d->qk_norm_targets != ANIMAXS_QK_NORM_Q_ONLY;
    const ax::NormJob q_job = jq, k_job = jk;
    np.njobs = 0;
    if (norm_q) np.job[np.njobs++] = q_job;
    if (norm_k) np.job[np.njobs++] = k_job;
    np.status = sym.status;
    if (ax::launch_qk_norm(np, stream) != cudaSuccess) return ANIMAXS_ERR_CUDA;
    if (norm_q) {
      qa = qn;
      q_st = q_job.out_tok;
      q_sh = D;
      q_sb = q_job.out_batch;
    }
    if (norm_k) {
      ka = kn;
      k_st = k_job.out_tok;
      k_sh = D;
      k_sb = k_job.out_batch;
    }
  }

  CUtensorMap tq, tk, tv;
  rc = ax_make_tmap(nullptr, &tq, qa, d->head_dim, d->q_len, d->heads, d->batch, q_st, q_sh, q_sb);
  if (rc == ANIMAXS_OK)
    rc = ax_make_tmap(nullptr, &tk, ka, d->head_dim, d->kv_len, d->kv_heads, d->batch, k_st, k_sh, k_sb);
  if (rc == ANIMAXS_OK)
    rc = ax_make_tmap(nullptr, &tv, v, d->head_dim, d->kv_len, d->kv_heads, d->batch, d->v_tok_stride,
                      d->v_head_stride, d->v_batch_stride);
  if (rc != ANIMAXS_OK) return rc;

  ax::AttnFwdParams p{};
  p.head_dim = static_cast<int>(d->head_dim);
  p.q_len = d->q_len;
  p.kv_len = d->kv_len;
  p.heads_per_kv = d->heads / d->kv_heads;
  p.kv_valid = d->kv_valid_len > 0 ? d->kv_valid_len : d->kv_len;
  p.kv_valid_dev = d->kv_valid_lens;
  p.causal = d->causal ? 1 : 0;
  const int rows_per_cta = ax::attn_fwd_rows_per_cta();
  p.n_q_tiles = (d->q_len + rows_per_cta - 1) / rows_per_cta;
  p.head_offset = 0;
  p.o_head_base = 0;
  const float scale = d->scale > 0.f ? d->scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = static_cast<__half*>(o);
  p.o_tok = d->o_tok_stride;
  p.o_head = d->o_head_stride;
  p.o_batch = d->o_batch_stride;
  p.status = sym.status;
  p.fp32_p = d->numerics == ANIMAXS_NUMERICS_FP32_SCORES_AND_SOFTMAX ? 1 : 0;
  if (ax::launch_attn_fwd(tq, tk, tv, p, d->heads, d->batch, stream) != cudaSuccess)
    return ANIMAXS_ERR_CUDA;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_noalloc_status(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ANIMAXS_ERR_NO_DEVICE;
  Symbols sym{};
  int rc = symbol_addresses(dev, &sym);
  if (rc != ANIMAXS_OK) return rc;
  unsigned int status = 0;
  cudaError_t e = cudaMemcpy(&status, sym.status, sizeof(status), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && status != 0) e = cudaMemset(sym.status, 0, sizeof(status));
  if (e != cudaSuccess) return ANIMAXS_ERR_CUDA;
  if (status & ax::kStatusTimeoutBit) return ANIMAXS_ERR_TIMEOUT;
  return status != 0 ? ANIMAXS_ERR_CUDA : ANIMAXS_OK;
}
