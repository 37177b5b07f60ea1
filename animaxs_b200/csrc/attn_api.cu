// attn_api.cu -- the C ABI of libanimaxs_attn.so (declared in include/animaxs_attn.h).
//
// Host-side responsibilities: argument validation (mirroring
// AttentionExecutor.validate, AnimaXS/Runtime/Metal/AttentionExecutor.swift:778-825),
// context-owned scratch (the reference's BufferPool, MetalContext.swift:86-103),
// TMA tensor-map construction, kernel launches, the RoPE table builders
// (DitRoPE.swift:58-107, QwenEncoderMetal.swift:126-142) and the GQA rule (:222).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/animaxs_attn.h"
#include "api_internal.h"
#include "kernels.h"
#include "sm100_ptx.cuh"

using ax::AttnFwdParams;
using ax::NormJob;
using ax::NormParams;

// ------------------------------------------------------------------ context --
int ax_set_error(animaxs_attn_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx != nullptr) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

static int ok(animaxs_attn_ctx* ctx) {
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

int ax_cuda_fail(animaxs_attn_ctx* ctx, cudaError_t e, const char* what) {
  return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int ax_ensure_scratch(animaxs_attn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return ANIMAXS_OK;
  if (ctx->scratch != nullptr) {
    // The previous buffer may still be read by queued work on another stream.
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "scratch resize sync");
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  size_t grow = bytes + bytes / 8;
  grow = (grow + 4095) & ~static_cast<size_t>(4095);
  cudaError_t e = cudaMalloc(&ctx->scratch, grow);
  if (e != cudaSuccess) {
    ctx->scratch = nullptr;
    return ax_cuda_fail(ctx, e, "scratch allocation");
  }
  ctx->scratch_bytes = grow;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_abi_version(void) { return ANIMAXS_ATTN_ABI_VERSION; }

extern "C" int animaxs_attn_create(int device, animaxs_attn_ctx** out) {
  if (out == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return ANIMAXS_ERR_NO_DEVICE;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return ANIMAXS_ERR_NO_DEVICE;
  if (prop.major != 10 || prop.minor != 0) return ANIMAXS_ERR_NO_DEVICE;  // sm_100 only
  auto* ctx = new (std::nothrow) animaxs_attn_ctx();
  if (ctx == nullptr) return ANIMAXS_ERR_CUDA;
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  cudaError_t e = cudaMalloc(&ctx->d_status, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(unsigned int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    delete ctx;
    return ANIMAXS_ERR_CUDA;
  }
  *out = ctx;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_destroy(animaxs_attn_ctx* ctx) {
  if (ctx == nullptr) return ANIMAXS_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->staging) cudaFree(ctx->staging);
  if (ctx->d_status) cudaFree(ctx->d_status);
  for (cudaEvent_t e : ctx->events) cudaEventDestroy(e);
  cudaSetDevice(prev);
  delete ctx;
  return ANIMAXS_OK;
}

extern "C" const char* animaxs_attn_last_error(const animaxs_attn_ctx* ctx) {
  if (ctx == nullptr) return "null context";
  return ctx->last_error.c_str();
}

extern "C" int animaxs_attn_desc_init(animaxs_attn_desc* d, int batch, int heads, int kv_heads,
                                      int q_len, int kv_len, int head_dim) {
  if (d == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  std::memset(d, 0, sizeof(*d));
  d->batch = batch;
  d->heads = heads;
  d->kv_heads = kv_heads;
  d->q_len = q_len;
  d->kv_len = kv_len;
  d->head_dim = head_dim;
  const int64_t hd = head_dim;
  d->q_tok_stride = static_cast<int64_t>(heads) * hd;
  d->q_head_stride = hd;
  d->q_batch_stride = static_cast<int64_t>(q_len) * heads * hd;
  d->o_tok_stride = d->q_tok_stride;
  d->o_head_stride = hd;
  d->o_batch_stride = d->q_batch_stride;
  d->k_tok_stride = static_cast<int64_t>(kv_heads) * hd;
  d->k_head_stride = hd;
  d->k_batch_stride = static_cast<int64_t>(kv_len) * kv_heads * hd;
  d->v_tok_stride = d->k_tok_stride;
  d->v_head_stride = hd;
  d->v_batch_stride = d->k_batch_stride;
  d->eps = 1e-6f;
  return ANIMAXS_OK;
}

// ----------------------------------------------------------------- validate --
static const char* kShapeMsg = "invalid attention shape, offset, or causal dimensions";

// Largest element offset touched by a [batch][rows][heads][128] strided view,
// plus one row; false on overflow.
static bool view_extent(int64_t batch, int64_t rows, int64_t heads, int64_t dim, int64_t sb,
                        int64_t st, int64_t sh, int64_t* bytes) {
  __int128 last = static_cast<__int128>(batch - 1) * sb + static_cast<__int128>(rows - 1) * st +
                  static_cast<__int128>(heads - 1) * sh + dim;
  __int128 b = last * 2;
  if (b > static_cast<__int128>(INT64_MAX)) return false;
  *bytes = static_cast<int64_t>(b);
  return true;
}

int ax_validate(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d, const void* q, const void* k,
                const void* v, const void* o) {
  if (d == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "null descriptor");
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "attention buffers must not be null");
  if (d->batch <= 0 || d->heads <= 0 || d->q_len <= 0 || d->kv_len <= 0 || d->head_dim <= 0 ||
      d->kv_heads <= 0 || d->heads % d->kv_heads != 0 || (d->causal && d->q_len != d->kv_len))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "%s", kShapeMsg);
  const bool wide = d->head_dim == 256 || d->head_dim == 384;
  if (d->head_dim != 128 && d->head_dim != 64 && !wide)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "attention on B200 requires headDim 64, 128, 256 or 384 (got %d)", d->head_dim);
  if (d->kv_valid_len < 0 || d->kv_valid_len > d->kv_len)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "kv_valid_len %d outside [0, keyCount %d]", d->kv_valid_len, d->kv_len);
  if (!(d->scale >= 0.f) || !std::isfinite(d->scale))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "softmax scale must be finite and >= 0");
  if (!(d->eps >= 0.f) || !std::isfinite(d->eps))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "eps must be finite and >= 0");
  if (d->qk_norm < ANIMAXS_QK_NONE || d->qk_norm > ANIMAXS_QK_RMS_ROPE)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "unknown qk_norm mode %d", d->qk_norm);
  if (d->qk_norm_targets < ANIMAXS_QK_NORM_BOTH || d->qk_norm_targets > ANIMAXS_QK_NORM_K_ONLY)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "unknown qk_norm_targets %d",
                        d->qk_norm_targets);
  if (d->numerics < ANIMAXS_NUMERICS_LEGACY || d->numerics > ANIMAXS_NUMERICS_BF16_COMPUTE)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "unknown numerics %d", d->numerics);
  if (d->numerics == ANIMAXS_NUMERICS_BF16_COMPUTE)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "bf16Compute numerics emulates Apple5 BF16 rounding and is not built for B200");
  if (wide && d->numerics == ANIMAXS_NUMERICS_FP32_SCORES_AND_SOFTMAX)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "fp32ScoresAndSoftmax numerics requires headDim 64 or 128 (got %d)", d->head_dim);
  if (wide && d->qk_norm != ANIMAXS_QK_NONE)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "fused q/k normalisation requires headDim 128 or 64 (got %d)", d->head_dim);
  if (d->qk_norm == ANIMAXS_QK_RMS_ROPE) {
    if (d->rope_table == nullptr)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "qk_norm RMS_ROPE needs a rope table");
    const int need = d->q_len > d->kv_len ? d->q_len : d->kv_len;
    if (d->rope_rows < need)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                          "rope table has %d rows, the call needs %d", d->rope_rows, need);
    if (reinterpret_cast<uintptr_t>(d->rope_table) % 16 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "rope table must be 16-byte aligned");
  }
  for (const void* w : {d->q_norm_weight, d->k_norm_weight})
    if (w != nullptr && reinterpret_cast<uintptr_t>(w) % 16 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "norm weights must be 16-byte aligned");
  for (const void* ptr : {q, k, v, o})
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                          "attention requires 16-byte-aligned offsets and row stride");
  const int64_t strides[12] = {d->q_tok_stride, d->q_head_stride, d->q_batch_stride,
                               d->k_tok_stride, d->k_head_stride, d->k_batch_stride,
                               d->v_tok_stride, d->v_head_stride, d->v_batch_stride,
                               d->o_tok_stride, d->o_head_stride, d->o_batch_stride};
  for (int i = 0; i < 12; ++i) {
    if (strides[i] < 0 || strides[i] % 8 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                          "attention requires 16-byte-aligned offsets and row stride");
    if (strides[i] >= (static_cast<int64_t>(1) << 39))
      return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "attention byte size overflow");
  }
  // Dimensions longer than one element need a positive stride.
  const bool zero_stride = (d->q_len > 1 && d->q_tok_stride == 0) ||
                           (d->kv_len > 1 && (d->k_tok_stride == 0 || d->v_tok_stride == 0)) ||
                           (d->q_len > 1 && d->o_tok_stride == 0) ||
                           (d->heads > 1 && (d->q_head_stride == 0 || d->o_head_stride == 0)) ||
                           (d->kv_heads > 1 && (d->k_head_stride == 0 || d->v_head_stride == 0));
  if (zero_stride) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "%s", kShapeMsg);
  struct View {
    int64_t rows, heads, sb, st, sh, have;
  } views[4] = {
      {d->q_len, d->heads, d->q_batch_stride, d->q_tok_stride, d->q_head_stride, d->q_bytes},
      {d->kv_len, d->kv_heads, d->k_batch_stride, d->k_tok_stride, d->k_head_stride, d->k_bytes},
      {d->kv_len, d->kv_heads, d->v_batch_stride, d->v_tok_stride, d->v_head_stride, d->v_bytes},
      {d->q_len, d->heads, d->o_batch_stride, d->o_tok_stride, d->o_head_stride, d->o_bytes}};
  for (const View& w : views) {
    int64_t need = 0;
    if (!view_extent(d->batch, w.rows, w.heads, d->head_dim, w.sb, w.st, w.sh, &need))
      return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "attention byte size overflow");
    if (w.have > 0 && need > w.have)
      return ax_set_error(ctx, ANIMAXS_ERR_OOB, "attention buffer range is out of bounds");
  }
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_validate(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d,
                                     const void* q, const void* k, const void* v, const void* o) {
  int rc = ax_validate(ctx, d, q, k, v, o);
  if (rc == ANIMAXS_OK && ctx != nullptr) ctx->last_error.clear();
  return rc;
}

// -------------------------------------------------------------- tensor maps --
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [batch][heads][rows][dim] fp16 view (dim a multiple of 64); box = 64 columns x
// box_rows rows, 128B swizzle.
int ax_make_tmap(animaxs_attn_ctx* ctx, CUtensorMap* map, const void* base, int64_t dim, int64_t rows,
                 int64_t heads, int64_t batch, int64_t st, int64_t sh, int64_t sb, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  // A stride of a dimension of extent 1 is never used for addressing but must
  // still satisfy the encoder's rules; substitute a legal value.
  const int64_t fallback = dim * 2;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(rows > 1 ? st * 2 : fallback),
                           static_cast<cuuint64_t>(heads > 1 ? sh * 2 : fallback),
                           static_cast<cuuint64_t>(batch > 1 ? sb * 2 : fallback)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)",
                        static_cast<int>(r));
  return ANIMAXS_OK;
}

// ------------------------------------------------------------------ forward --
extern "C" int animaxs_attn_scratch_bytes(const animaxs_attn_desc* d, int64_t* bytes) {
  if (d == nullptr || bytes == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *bytes = 0;
  if (d->qk_norm == ANIMAXS_QK_NONE) return ANIMAXS_OK;
  // Only the copies the prologue writes: q unless the caller normalised it,
  // k unless the caller normalised it (qk_norm_targets); k follows q at a
  // 256-byte boundary.
  const bool norm_q = d->qk_norm_targets != ANIMAXS_QK_NORM_K_ONLY;
  const bool norm_k = d->qk_norm_targets != ANIMAXS_QK_NORM_Q_ONLY;
  const int64_t q = norm_q ? static_cast<int64_t>(d->batch) * d->q_len * d->heads * d->head_dim * 2 : 0;
  const int64_t k = norm_k ? static_cast<int64_t>(d->batch) * d->kv_len * d->kv_heads * d->head_dim * 2 : 0;
  *bytes = ((q + 255) & ~static_cast<int64_t>(255)) + k;
  return ANIMAXS_OK;
}

// Core of the forward path; `heads_begin/heads_count` select the query heads
// computed (the head-sharded path uses a sub-range), `o_override` lets the
// caller redirect the output.
int ax_forward_range(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d, const void* q,
                     const void* k, const void* v, void* o, int heads_begin, int heads_count,
                     const AxOutView* o_view, cudaStream_t stream, const AxPeers* peers) {
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  struct Restore {
    int dev, prev;
    ~Restore() {
      if (dev != prev) cudaSetDevice(prev);
    }
  } restore{ctx->device, prev};

  const int64_t D = d->head_dim;
  if (ctx->score_probe != nullptr && D != 64 && D != 128)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED, "the score probe supports headDim 64 and 128 (got %lld)",
                        static_cast<long long>(D));
  const void* qa = q;
  const void* ka = k;
  int64_t q_st = d->q_tok_stride, q_sh = d->q_head_stride, q_sb = d->q_batch_stride;
  int64_t k_st = d->k_tok_stride, k_sh = d->k_head_stride, k_sb = d->k_batch_stride;
  const int rows_per_cta = ax::attn_fwd_rows_per_cta();
  const int n_q_tiles = (d->q_len + rows_per_cta - 1) / rows_per_cta;

  if (d->qk_norm != ANIMAXS_QK_NONE) {
    const bool norm_q = d->qk_norm_targets != ANIMAXS_QK_NORM_K_ONLY;
    const bool norm_k = d->qk_norm_targets != ANIMAXS_QK_NORM_Q_ONLY;
    const int64_t q_bytes = static_cast<int64_t>(d->batch) * d->q_len * d->heads * D * 2;
    const int64_t k_bytes = static_cast<int64_t>(d->batch) * d->kv_len * d->kv_heads * D * 2;
    // Layout as animaxs_attn_scratch_bytes counts it: q's copy, then k's at
    // the next 256-byte boundary (each only when the prologue writes it).
    const int64_t k_off = ((norm_q ? q_bytes : 0) + 255) & ~static_cast<int64_t>(255);
    int rc = ax_ensure_scratch(ctx, static_cast<size_t>(k_off + (norm_k ? k_bytes : 0)));
    if (rc != ANIMAXS_OK) return rc;
    __half* qn = static_cast<__half*>(ctx->scratch);
    __half* kn = reinterpret_cast<__half*>(static_cast<char*>(ctx->scratch) + k_off);
    NormParams np{};
    np.head_dim = static_cast<int>(d->head_dim);
    np.eps = d->eps > 0.f ? d->eps : 1e-6f;
    np.rope = d->qk_norm == ANIMAXS_QK_RMS_ROPE ? d->rope_table : nullptr;
    // Only the query heads this call computes need normalising.
    NormJob& jq = np.job[0];
    jq.in = static_cast<const __half*>(q) + static_cast<int64_t>(heads_begin) * q_sh;
    jq.out = qn + static_cast<int64_t>(heads_begin) * D;
    jq.in_tok = q_st;
    jq.in_head = q_sh;
    jq.in_batch = q_sb;
    jq.out_tok = static_cast<int64_t>(d->heads) * D;
    jq.out_head = D;
    jq.out_batch = static_cast<int64_t>(d->q_len) * d->heads * D;
    jq.tokens = d->q_len;
    jq.heads = heads_count;
    jq.batch = d->batch;
    jq.weight = static_cast<const __half*>(d->q_norm_weight);
    jq.rows = static_cast<int64_t>(d->batch) * d->q_len * heads_count;
    const int group = d->heads / d->kv_heads;
    const int kv_begin = heads_begin / group;
    const int kv_count = (heads_begin + heads_count - 1) / group - kv_begin + 1;
    NormJob& jk = np.job[1];
    jk.in = static_cast<const __half*>(k) + static_cast<int64_t>(kv_begin) * k_sh;
    jk.out = kn + static_cast<int64_t>(kv_begin) * D;
    jk.in_tok = k_st;
    jk.in_head = k_sh;
    jk.in_batch = k_sb;
    jk.out_tok = static_cast<int64_t>(d->kv_heads) * D;
    jk.out_head = D;
    jk.out_batch = static_cast<int64_t>(d->kv_len) * d->kv_heads * D;
    jk.tokens = d->kv_len;
    jk.heads = kv_count;
    jk.batch = d->batch;
    jk.weight = static_cast<const __half*>(d->k_norm_weight);
    jk.rows = static_cast<int64_t>(d->batch) * d->kv_len * kv_count;
    // The caller may hold an already normalised q or k (qk_norm_targets).
    const NormJob q_job = jq, k_job = jk;
    np.njobs = 0;
    if (norm_q) np.job[np.njobs++] = q_job;
    if (norm_k) np.job[np.njobs++] = k_job;
    np.status = ctx->d_status;
    if (np.njobs > 0) {
      cudaError_t e = ax::launch_qk_norm(np, stream);
      if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "qk_norm launch");
    }
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
  int rc = ax_make_tmap(ctx, &tq, qa, d->head_dim, d->q_len, d->heads, d->batch, q_st, q_sh, q_sb);
  if (rc == ANIMAXS_OK)
    rc = ax_make_tmap(ctx, &tk, ka, d->head_dim, d->kv_len, d->kv_heads, d->batch, k_st, k_sh, k_sb);
  if (rc == ANIMAXS_OK)
    rc = ax_make_tmap(ctx, &tv, v, d->head_dim, d->kv_len, d->kv_heads, d->batch, d->v_tok_stride,
                      d->v_head_stride, d->v_batch_stride);
  if (rc != ANIMAXS_OK) return rc;

  AttnFwdParams p{};
  p.head_dim = static_cast<int>(d->head_dim);
  p.q_len = d->q_len;
  p.kv_len = d->kv_len;
  p.heads_per_kv = d->heads / d->kv_heads;
  p.kv_valid = d->kv_valid_len > 0 ? d->kv_valid_len : d->kv_len;
  p.kv_valid_dev = d->kv_valid_lens;
  p.causal = d->causal ? 1 : 0;
  p.n_q_tiles = n_q_tiles;
  p.head_offset = heads_begin;
  const float scale = d->scale > 0.f ? d->scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  if (o_view != nullptr) {
    p.o = static_cast<__half*>(o_view->ptr);
    p.o_tok = o_view->tok;
    p.o_head = o_view->head;
    p.o_batch = o_view->batch;
    p.o_head_base = o_view->head_base;
  } else {
    p.o = static_cast<__half*>(o);
    p.o_tok = d->o_tok_stride;
    p.o_head = d->o_head_stride;
    p.o_batch = d->o_batch_stride;
  }
  p.status = ctx->d_status;
  p.probe = ctx->score_probe;
  p.fp32_p = d->numerics == ANIMAXS_NUMERICS_FP32_SCORES_AND_SOFTMAX ? 1 : 0;
  if (peers != nullptr) {
    if (peers->n < 0 || peers->n > ax::kMaxPeers || (d->head_dim != 64 && d->head_dim != 128))
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "peer stores need head_dim 64 or 128 and <= 7 peers");
    p.n_peers = peers->n;
    for (int i = 0; i < peers->n; ++i) {
      p.peer_delta[i] = peers->delta[i];
      p.peer_arrive[i] = peers->arrive[i];
    }
    p.peer_go = peers->go;
    p.peer_go_value = peers->go_value;
  }
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
  if (ctx->timing) {
    while (ctx->events.size() < ctx->events_used + 2) {
      cudaEvent_t ev;
      cudaError_t ce = cudaEventCreate(&ev);
      if (ce != cudaSuccess) return ax_cuda_fail(ctx, ce, "timing event");
      ctx->events.push_back(ev);
    }
    ev_start = ctx->events[ctx->events_used];
    ev_stop = ctx->events[ctx->events_used + 1];
    cudaEventRecord(ev_start, stream);
  }
  cudaError_t e = ax::launch_attn_fwd(tq, tk, tv, p, heads_count, d->batch, stream);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "attention launch");
  if (ctx->timing) {
    cudaEventRecord(ev_stop, stream);
    ctx->events_used += 2;
  }
  ctx->query_tiles += static_cast<int64_t>(heads_count) * d->batch *
                      ((d->q_len + ax::kTileM - 1) / ax::kTileM);
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_forward(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d,
                                    const void* q, const void* k, const void* v, void* o,
                                    void* stream) {
  AxRange range("animaxs_attn_forward");
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int rc = ax_validate(ctx, d, q, k, v, o);
  if (rc != ANIMAXS_OK) return rc;
  rc = ax_forward_range(ctx, d, q, k, v, o, 0, d->heads, nullptr,
                        static_cast<cudaStream_t>(stream));
  return rc == ANIMAXS_OK ? ok(ctx) : rc;
}

extern "C" int animaxs_attn_synchronize(animaxs_attn_ctx* ctx, void* stream) {
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  unsigned int status = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&status, ctx->d_status, sizeof(status), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && status != 0) e = cudaMemset(ctx->d_status, 0, sizeof(status));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "synchronize");
  if (status & ax::kStatusTimeoutBit)
    return ax_set_error(ctx, ANIMAXS_ERR_TIMEOUT, "a bounded device-side wait expired");
  if (status != 0) return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "device status 0x%x", status);
  return ok(ctx);
}

// ------------------------------------------------------ failure detection --
namespace {
// One thread waits, through the kernels' bounded mbarrier wait, on a phase
// that nothing completes; after `limit_ns` it sets the timeout status bit and
// returns, as an aborting kernel does.
__global__ void selftest_wait_kernel(unsigned int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ax::mbar_init(ax::smem_u32(&bar), 1);
    abort_flag = 0;
    ax::mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) ax::mbar_wait_for(ax::smem_u32(&bar), 0, &abort_flag, status, limit_ns);
}
}  // namespace

extern "C" int animaxs_attn_selftest_wait_timeout(animaxs_attn_ctx* ctx, int64_t timeout_ns, void* stream) {
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (timeout_ns <= 0 || timeout_ns > 10'000'000'000LL)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "self-test timeout must be in (0, 10 s]");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      ctx->d_status, static_cast<unsigned long long>(timeout_ns));
  cudaError_t e = cudaGetLastError();
  cudaSetDevice(prev);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "self-test launch");
  return ok(ctx);
}

extern "C" int animaxs_attn_set_kernel_timing(animaxs_attn_ctx* ctx, int enable) {
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  ctx->timing = enable != 0;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_set_score_probe(animaxs_attn_ctx* ctx, unsigned int* stats) {
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (stats != nullptr && reinterpret_cast<uintptr_t>(stats) % 4 != 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "probe slot must be 4-byte aligned");
  ctx->score_probe = stats;
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_kernel_timing(animaxs_attn_ctx* ctx, int64_t* launches,
                                          double* total_ms, double* max_ms) {
  if (ctx == nullptr || launches == nullptr || total_ms == nullptr || max_ms == nullptr)
    return ANIMAXS_ERR_INVALID_ARG;
  *launches = 0;
  *total_ms = 0.0;
  *max_ms = 0.0;
  if (ctx->events_used == 0) return ok(ctx);
  cudaError_t e = cudaEventSynchronize(ctx->events[ctx->events_used - 1]);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "timing read");
  for (size_t i = 0; i + 1 < ctx->events_used; i += 2) {
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, ctx->events[i], ctx->events[i + 1]);
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "timing elapsed");
    *launches += 1;
    *total_ms += ms;
    if (ms > *max_ms) *max_ms = ms;
  }
  ctx->events_used = 0;
  return ok(ctx);
}

extern "C" int animaxs_attn_query_tiles(const animaxs_attn_ctx* ctx, int64_t* tiles) {
  if (ctx == nullptr || tiles == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *tiles = ctx->query_tiles;
  return ANIMAXS_OK;
}

// ------------------------------------------------------ standalone qk norms --
static int norm_standalone(animaxs_attn_ctx* ctx, const void* in, void* out, const void* weight,
                           const float* rope, int tokens, int heads, int head_dim,
                           int64_t row_stride, float eps, void* stream) {
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (in == nullptr || out == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "null buffer");
  if (tokens <= 0 || heads <= 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "invalid rms norm shape");
  if (head_dim != 128 && head_dim != 64)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED, "rms norm requires headDim 128 or 64");
  if (row_stride == 0) row_stride = static_cast<int64_t>(heads) * head_dim;
  if (row_stride < static_cast<int64_t>(heads) * head_dim || row_stride % 8 != 0 ||
      reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
      reinterpret_cast<uintptr_t>(weight) % 16 || reinterpret_cast<uintptr_t>(rope) % 16)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "rms norm requires 16-byte-aligned buffers and row stride");
  if (!(eps >= 0.f)) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "eps must be >= 0");
  NormParams np{};
  np.head_dim = head_dim;
  np.eps = eps > 0.f ? eps : 1e-6f;
  np.rope = rope;
  NormJob& j = np.job[0];
  j.in = static_cast<const __half*>(in);
  j.out = static_cast<__half*>(out);
  j.in_tok = j.out_tok = row_stride;
  j.in_head = j.out_head = head_dim;
  j.in_batch = j.out_batch = 0;
  j.tokens = tokens;
  j.heads = heads;
  j.batch = 1;
  j.weight = static_cast<const __half*>(weight);
  j.rows = static_cast<int64_t>(tokens) * heads;
  np.njobs = 1;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  np.status = ctx->d_status;
  cudaError_t e = ax::launch_qk_norm(np, static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "rms norm launch");
  return ok(ctx);
}

extern "C" int animaxs_rms_rope_split_half(animaxs_attn_ctx* ctx, const void* in, void* out,
                                           const void* weight, const float* rope_table,
                                           int tokens, int heads, int head_dim,
                                           int64_t row_stride, float eps, void* stream) {
  if (rope_table == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "rms_rope_split_half needs a rope table");
  return norm_standalone(ctx, in, out, weight, rope_table, tokens, heads, head_dim, row_stride,
                         eps, stream);
}

extern "C" int animaxs_rmsnorm_heads_half(animaxs_attn_ctx* ctx, const void* in, void* out,
                                          const void* weight, int tokens, int heads,
                                          int head_dim, int64_t row_stride, float eps,
                                          void* stream) {
  return norm_standalone(ctx, in, out, weight, nullptr, tokens, heads, head_dim, row_stride, eps,
                         stream);
}

// ------------------------------------------------------------- host helpers --
static void write_block(float* out, int64_t tok, int pairs, int f, float angle) {
  const float c = std::cos(angle), s = std::sin(angle);
  float* b = out + (tok * pairs + f) * 4;
  b[0] = c;
  b[1] = -s;
  b[2] = s;
  b[3] = c;
}

extern "C" int animaxs_rope3d_table(int T, int H, int W, float* out) {
  if (T <= 0 || H <= 0 || W <= 0 || out == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  constexpr int hd = 128, dim_h = hd / 6 * 2, dim_w = dim_h, dim_t = hd - 2 * dim_h;
  const float h_theta = static_cast<float>(10000.0 * std::pow(4.0, dim_h / (dim_h - 2.0)));
  const float w_theta = static_cast<float>(10000.0 * std::pow(4.0, dim_w / (dim_w - 2.0)));
  const float t_theta = static_cast<float>(10000.0 * std::pow(1.0, dim_t / (dim_t - 2.0)));
  float fh[dim_h / 2], fw[dim_w / 2], ft[dim_t / 2];
  for (int d = 0; d < dim_h / 2; ++d)
    fh[d] = 1.0f / std::pow(h_theta, static_cast<float>(2 * d) / static_cast<float>(dim_h));
  for (int d = 0; d < dim_w / 2; ++d)
    fw[d] = 1.0f / std::pow(w_theta, static_cast<float>(2 * d) / static_cast<float>(dim_w));
  for (int d = 0; d < dim_t / 2; ++d)
    ft[d] = 1.0f / std::pow(t_theta, static_cast<float>(2 * d) / static_cast<float>(dim_t));
  constexpr int pairs = hd / 2;
  int64_t tok = 0;
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h)
      for (int w = 0; w < W; ++w, ++tok) {
        int f = 0;
        for (int d = 0; d < dim_t / 2; ++d) write_block(out, tok, pairs, f++, static_cast<float>(t) * ft[d]);
        for (int d = 0; d < dim_h / 2; ++d) write_block(out, tok, pairs, f++, static_cast<float>(h) * fh[d]);
        for (int d = 0; d < dim_w / 2; ++d) write_block(out, tok, pairs, f++, static_cast<float>(w) * fw[d]);
      }
  return ANIMAXS_OK;
}

extern "C" int animaxs_rope1d_table(int seq_len, int head_dim, double theta, float* out) {
  if (seq_len <= 0 || head_dim <= 0 || head_dim % 2 || !(theta > 0) || out == nullptr)
    return ANIMAXS_ERR_INVALID_ARG;
  const int pairs = head_dim / 2;
  for (int p = 0; p < pairs; ++p) {
    const float inv = 1.0f / std::pow(static_cast<float>(theta),
                                      static_cast<float>(2 * p) / static_cast<float>(head_dim));
    for (int t = 0; t < seq_len; ++t) write_block(out, t, pairs, p, static_cast<float>(t) * inv);
  }
  return ANIMAXS_OK;
}

extern "C" int animaxs_gqa_kv_head(int query_head, int heads, int kv_heads) {
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || query_head < 0 ||
      query_head >= heads)
    return ANIMAXS_ERR_INVALID_ARG;
  return query_head / (heads / kv_heads);
}
