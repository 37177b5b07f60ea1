// cross_kv_cache.cu -- the DiT's cross-attention K/V cache (C ABI in
// include/animaxs_attn.h).
//
// Replaces the reference's CrossKVCache (AnimaXS/Runtime/Metal/
// DiTBlockExecutor.swift:19-43) and the block executor's use of it
// (:1105-1161): the cross-attention K and V of a block are projected from the
// LLM-adapter context, K is RMS-normalised, and both are kept for the other
// Euler steps of the generation, because the context does not change between
// steps.  The reference copies a hit back into its scratch buffers with a blit;
// here attention reads the cache in place (the descriptor carries its strides)
// with qk_norm_targets Q_ONLY, so a hit costs nothing.
//
// Layout: for each block, [batch][tokens][K (kv_heads x head_dim) | V (kv_heads
// x head_dim)] fp16 -- one row holds a token's K and V, which is what one
// fused projection of the context against the stacked [W_k; W_v] writes.
#include <cuda_runtime.h>

#include <new>
#include <vector>

#include "../../include/animaxs_attn.h"
#include "api_internal.h"
#include "kernels.h"

struct animaxs_cross_kv_cache {
  animaxs_attn_ctx* ctx = nullptr;
  int blocks = 0, batch = 0, tokens = 0, kv_heads = 0, head_dim = 0;
  char* mem = nullptr;
  bool owned = false;
  std::vector<unsigned char> ready;

  int64_t row() const { return 2LL * kv_heads * head_dim; }            // elements per token row
  int64_t batch_stride() const { return row() * tokens; }               // elements per image
  int64_t block_bytes() const { return batch_stride() * batch * 2; }
  __half* k(int b) const { return reinterpret_cast<__half*>(mem + b * block_bytes()); }
  __half* v(int b) const { return k(b) + static_cast<int64_t>(kv_heads) * head_dim; }
};

namespace {

int check_shape(int blocks, int batch, int tokens, int kv_heads, int head_dim) {
  if (blocks <= 0 || batch <= 0 || tokens <= 0 || kv_heads <= 0) return ANIMAXS_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return ANIMAXS_ERR_UNSUPPORTED;
  return ANIMAXS_OK;
}

int check_block(animaxs_cross_kv_cache* c, int block) {
  if (c == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (block < 0 || block >= c->blocks)
    return ax_set_error(c->ctx, ANIMAXS_ERR_INVALID_ARG, "cross-K/V cache block %d outside [0, %d)", block,
                        c->blocks);
  return ANIMAXS_OK;
}

struct DeviceScope {
  int prev = 0, dev = 0;
  explicit DeviceScope(int d) : dev(d) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    if (prev != dev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int animaxs_cross_kv_cache_bytes(int blocks, int batch, int tokens, int kv_heads, int head_dim,
                                            int64_t* bytes) {
  if (bytes == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  const int rc = check_shape(blocks, batch, tokens, kv_heads, head_dim);
  if (rc != ANIMAXS_OK) return rc;
  *bytes = static_cast<int64_t>(blocks) * batch * tokens * 2 * kv_heads * head_dim * 2;
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_create(animaxs_attn_ctx* ctx, int blocks, int batch, int tokens,
                                             int kv_heads, int head_dim, void* memory, int64_t memory_bytes,
                                             animaxs_cross_kv_cache** out) {
  if (ctx == nullptr || out == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *out = nullptr;
  int64_t need = 0;
  int rc = animaxs_cross_kv_cache_bytes(blocks, batch, tokens, kv_heads, head_dim, &need);
  if (rc != ANIMAXS_OK)
    return ax_set_error(ctx, rc, "invalid cross-K/V cache shape (head_dim 64 or 128, positive sizes)");
  if (memory != nullptr && (memory_bytes < need || reinterpret_cast<uintptr_t>(memory) % 256 != 0))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "cross-K/V cache memory must be 256-byte aligned and hold %lld bytes",
                        static_cast<long long>(need));
  auto* c = new (std::nothrow) animaxs_cross_kv_cache();
  if (c == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "host allocation failed");
  c->ctx = ctx;
  c->blocks = blocks;
  c->batch = batch;
  c->tokens = tokens;
  c->kv_heads = kv_heads;
  c->head_dim = head_dim;
  c->ready.assign(blocks, 0);
  if (memory != nullptr) {
    c->mem = static_cast<char*>(memory);
  } else {
    DeviceScope scope(ctx->device);
    const cudaError_t e = cudaMalloc(&c->mem, static_cast<size_t>(need));
    if (e != cudaSuccess) {
      delete c;
      return ax_cuda_fail(ctx, e, "cross-K/V cache allocation");
    }
    c->owned = true;
  }
  *out = c;
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_destroy(animaxs_cross_kv_cache* c) {
  if (c == nullptr) return ANIMAXS_OK;
  if (c->owned) {
    DeviceScope scope(c->ctx->device);
    cudaDeviceSynchronize();  // queued attention may still read the cache
    cudaFree(c->mem);
  }
  delete c;
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_fill(animaxs_cross_kv_cache* c, int block, const void* k,
                                           int64_t k_tok_stride, int64_t k_batch_stride, const void* v,
                                           int64_t v_tok_stride, int64_t v_batch_stride, int k_norm,
                                           const void* k_norm_weight, float eps, void* stream) {
  int rc = check_block(c, block);
  if (rc != ANIMAXS_OK) return rc;
  animaxs_attn_ctx* ctx = c->ctx;
  const int64_t hd = static_cast<int64_t>(c->kv_heads) * c->head_dim;
  if (k == nullptr || v == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "cross-K/V cache fill needs k and v");
  if (k_tok_stride < hd || v_tok_stride < hd || k_tok_stride % 8 || v_tok_stride % 8 ||
      (c->batch > 1 && (k_batch_stride < k_tok_stride * c->tokens || v_batch_stride < v_tok_stride * c->tokens)) ||
      reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16 ||
      reinterpret_cast<uintptr_t>(k_norm_weight) % 16)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "cross-K/V cache fill needs 16-byte-aligned k, v and weight and token strides "
                        ">= kv_heads * head_dim (multiples of 8)");
  if (k_norm != 0 && k_norm != 1) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "k_norm must be 0 or 1");
  if (!(eps >= 0.f)) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "eps must be >= 0");
  DeviceScope scope(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k_norm) {
    // K: the same RMSNorm kernel the attention prologue runs (qk_norm.cu),
    // so cached and uncached calls see the same normalised bits.
    ax::NormParams np{};
    np.head_dim = c->head_dim;
    np.eps = eps > 0.f ? eps : 1e-6f;
    np.rope = nullptr;
    np.njobs = 1;
    np.status = ctx->d_status;
    ax::NormJob& j = np.job[0];
    j.in = static_cast<const __half*>(k);
    j.out = c->k(block);
    j.in_tok = k_tok_stride;
    j.in_head = c->head_dim;
    j.in_batch = k_batch_stride;
    j.out_tok = c->row();
    j.out_head = c->head_dim;
    j.out_batch = c->batch_stride();
    j.tokens = c->tokens;
    j.heads = c->kv_heads;
    j.batch = c->batch;
    j.weight = static_cast<const __half*>(k_norm_weight);
    j.rows = static_cast<int64_t>(c->batch) * c->tokens * c->kv_heads;
    const cudaError_t e = ax::launch_qk_norm(np, s);
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "cross-K/V cache K normalisation");
  }
  for (int b = 0; b < c->batch; ++b) {
    cudaError_t e = cudaSuccess;
    if (!k_norm)
      e = cudaMemcpy2DAsync(c->k(block) + b * c->batch_stride(), c->row() * 2,
                            static_cast<const __half*>(k) + b * k_batch_stride, k_tok_stride * 2, hd * 2,
                            c->tokens, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(c->v(block) + b * c->batch_stride(), c->row() * 2,
                            static_cast<const __half*>(v) + b * v_batch_stride, v_tok_stride * 2, hd * 2,
                            c->tokens, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "cross-K/V cache copy");
  }
  c->ready[block] = 1;
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_project(animaxs_cross_kv_cache* c, int block, const void* context,
                                              int64_t context_stride, int context_dim, const void* w_kv,
                                              int64_t w_stride, const void* k_norm_weight, float eps,
                                              void* stream) {
  int rc = check_block(c, block);
  if (rc != ANIMAXS_OK) return rc;
  if (c->head_dim != 128)
    return ax_set_error(c->ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "cross-K/V cache projection normalises heads of 128 (got %d)", c->head_dim);
  // One GEMM: [batch*tokens, context_dim] x [W_k; W_v]^T -> the block's K|V
  // rows, RMSNorm on the K columns in the epilogue (the reference's linear K,
  // linear V, then rmsnorm_heads_half on K, DiTBlockExecutor.swift:1123-1150).
  animaxs_proj_desc d;
  animaxs_proj_desc_init(&d, c->batch * c->tokens, static_cast<int>(c->row()), context_dim,
                         ANIMAXS_PROJ_QKV_NORM);
  d.x_stride = context_stride;
  d.w_stride = w_stride;
  d.out_stride = c->row();
  d.tokens = c->tokens;
  d.qk_norm = ANIMAXS_QK_RMS;
  d.q_cols = 0;
  d.k_cols = c->kv_heads * c->head_dim;
  d.k_norm_weight = k_norm_weight;
  d.eps = eps;
  rc = animaxs_proj_forward(c->ctx, &d, context, w_kv, c->k(block), stream);
  if (rc != ANIMAXS_OK) return rc;
  c->ready[block] = 1;
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_block(const animaxs_cross_kv_cache* c, int block, void** k, void** v,
                                            int64_t* tok_stride, int64_t* batch_stride, int* ready) {
  if (c == nullptr || block < 0 || block >= c->blocks) return ANIMAXS_ERR_INVALID_ARG;
  if (k) *k = c->k(block);
  if (v) *v = c->v(block);
  if (tok_stride) *tok_stride = c->row();
  if (batch_stride) *batch_stride = c->batch_stride();
  if (ready) *ready = c->ready[block];
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_mark_ready(animaxs_cross_kv_cache* c, int block, int ready) {
  const int rc = check_block(c, block);
  if (rc != ANIMAXS_OK) return rc;
  c->ready[block] = ready ? 1 : 0;
  return ANIMAXS_OK;
}

extern "C" int animaxs_cross_kv_cache_reset(animaxs_cross_kv_cache* c) {
  if (c == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  c->ready.assign(c->blocks, 0);
  return ANIMAXS_OK;
}
