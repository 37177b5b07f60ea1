// proj_api.cu -- C ABI of the fused attention projections (include/animaxs_attn.h):
// validation, 2-D tensor maps, launch.  The kernel is proj_sm100.cu.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/animaxs_attn.h"
#include "api_internal.h"
#include "kernels.h"

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [rows][cols] row-major matrix with `stride` elements between rows; box
// box_cols x box_rows, 128-byte swizzle (box_cols * element size == 128).
int make_tmap_2d(animaxs_attn_ctx* ctx, CUtensorMap* map, const void* base, bool f32, int64_t cols,
                 int64_t rows, int64_t stride, int box_cols, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int64_t es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(rows > 1 ? stride * es : cols * es + (16 - cols * es % 16) % 16)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return ANIMAXS_OK;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int proj_validate(animaxs_attn_ctx* ctx, const animaxs_proj_desc* d, const void* x, const void* w,
                  const void* out) {
  if (d == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "null descriptor");
  if (x == nullptr || w == nullptr || out == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "projection buffers must not be null");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0 || d->tokens <= 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "invalid projection shape");
  if (d->epilogue < ANIMAXS_PROJ_STORE || d->epilogue > ANIMAXS_PROJ_GATE_ADD)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "unknown projection epilogue %d", d->epilogue);
  const bool f32_out = d->epilogue == ANIMAXS_PROJ_GATE_ADD;
  // W8/W4 codes are decoded into an aligned fp16 copy first: only an fp16
  // weight is read by the GEMM's tensor map (w_stride is then unused).
  const bool fp16_w = d->w_storage == ANIMAXS_WEIGHT_FP16;
  if (d->k % 8 != 0 || d->x_stride < d->k || d->x_stride % 8 != 0 ||
      (fp16_w && (d->w_stride < d->k || d->w_stride % 8 != 0 || !aligned16(w))) || d->out_stride < d->n ||
      d->out_stride % (f32_out ? 4 : 8) != 0 || !aligned16(x) || !aligned16(out))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "projection requires 16-byte-aligned buffers and row strides, k a multiple of 8");
  if (d->x_stride >= (int64_t{1} << 38) || (fp16_w && d->w_stride >= (int64_t{1} << 38)) ||
      d->out_stride >= (int64_t{1} << 38))
    return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "projection byte size overflow");
  if (!(d->eps >= 0.f) || !std::isfinite(d->eps))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "eps must be finite and >= 0");
  if (d->epilogue == ANIMAXS_PROJ_QKV_NORM) {
    if (d->qk_norm != ANIMAXS_QK_RMS && d->qk_norm != ANIMAXS_QK_RMS_ROPE)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "QKV_NORM needs qk_norm RMS or RMS_ROPE");
    if (d->q_cols < 0 || d->k_cols < 0 || d->q_cols % 128 != 0 || d->k_cols % 128 != 0 ||
        static_cast<int64_t>(d->q_cols) + d->k_cols > d->n || d->n % 128 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                          "QKV_NORM normalises heads of 128: q_cols, k_cols and n must be multiples of 128");
    if (d->qk_norm == ANIMAXS_QK_RMS_ROPE &&
        (d->rope_table == nullptr || d->rope_rows < d->tokens || !aligned16(d->rope_table)))
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                          "RMS_ROPE needs a 16-byte-aligned rope table with >= tokens rows");
    for (const void* wt : {d->q_norm_weight, d->k_norm_weight})
      if (wt != nullptr && !aligned16(wt))
        return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "norm weights must be 16-byte aligned");
  }
  if (d->epilogue == ANIMAXS_PROJ_GATE_ADD) {
    if (d->gate == nullptr || d->gate_stride < d->n)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "GATE_ADD needs a gate with gate_stride >= n");
  }
  if (d->w_storage != ANIMAXS_WEIGHT_FP16) {
    if (d->w_storage != ANIMAXS_WEIGHT_W8 && d->w_storage != ANIMAXS_WEIGHT_W4)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "unknown weight storage %d", d->w_storage);
    const int64_t need = d->w_storage == ANIMAXS_WEIGHT_W4 ? (int64_t{d->k} + 1) / 2 : d->k;
    if (d->w_scale == nullptr || d->w_zero == nullptr || d->w_packed_stride < need ||
        reinterpret_cast<uintptr_t>(d->w_scale) % 2 != 0 || reinterpret_cast<uintptr_t>(d->w_zero) % 2 != 0)
      return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                          "W8/W4 weights need fp16 scale and zero and w_packed_stride >= %lld bytes",
                          static_cast<long long>(need));
    if (d->w_packed_stride >= (int64_t{1} << 40) ||
        static_cast<int64_t>(d->n) * d->k >= (int64_t{1} << 40))
      return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "projection byte size overflow");
  }
  return ANIMAXS_OK;
}

int dequant_validate(animaxs_attn_ctx* ctx, int bits, const void* packed, const void* scale, const void* zero,
                     const void* out, int rows, int k, int64_t packed_stride, int64_t out_stride) {
  if (bits != 4 && bits != 8) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "bits must be 4 or 8");
  if (packed == nullptr || scale == nullptr || zero == nullptr || out == nullptr)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "dequant buffers must not be null");
  if (rows <= 0 || k <= 0) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "invalid dequant shape");
  const int64_t need = bits == 4 ? (int64_t{k} + 1) / 2 : k;
  if (packed_stride < need || out_stride < k)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG,
                        "packed_stride must be >= %lld bytes and out_stride >= k", static_cast<long long>(need));
  if (reinterpret_cast<uintptr_t>(scale) % 2 != 0 || reinterpret_cast<uintptr_t>(zero) % 2 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 2 != 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "scale, zero and out must be 2-byte aligned");
  if (packed_stride >= (int64_t{1} << 40) || out_stride >= (int64_t{1} << 40))
    return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "dequant byte size overflow");
  return ANIMAXS_OK;
}

}  // namespace

extern "C" int animaxs_proj_desc_init(animaxs_proj_desc* d, int m, int n, int k, int epilogue) {
  if (d == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  std::memset(d, 0, sizeof(*d));
  d->m = m;
  d->n = n;
  d->k = k;
  d->x_stride = k;
  d->w_stride = k;
  d->out_stride = n;
  d->epilogue = epilogue;
  d->tokens = m;
  d->gate_stride = n;
  d->eps = 1e-6f;
  return ANIMAXS_OK;
}

extern "C" int animaxs_proj_validate(animaxs_attn_ctx* ctx, const animaxs_proj_desc* d, const void* x,
                                     const void* w, const void* out) {
  const int rc = proj_validate(ctx, d, x, w, out);
  if (rc == ANIMAXS_OK && ctx != nullptr) ctx->last_error.clear();
  return rc;
}

extern "C" int animaxs_dequant_to_half(animaxs_attn_ctx* ctx, int bits, const void* packed, const void* scale,
                                       const void* zero, void* out, int rows, int k, int64_t packed_stride,
                                       int64_t out_stride, void* stream) {
  AxRange range("animaxs_dequant_to_half");
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int rc = dequant_validate(ctx, bits, packed, scale, zero, out, rows, k, packed_stride, out_stride);
  if (rc != ANIMAXS_OK) return rc;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  cudaError_t e = ax::launch_dequant(bits, packed, scale, zero, out, rows, k, packed_stride, out_stride,
                                     ctx->num_sms, static_cast<cudaStream_t>(stream));
  if (prev != ctx->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "weight decode");
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" int animaxs_proj_forward(animaxs_attn_ctx* ctx, const animaxs_proj_desc* d, const void* x,
                                    const void* w, void* out, void* stream) {
  AxRange range("animaxs_proj_forward");
  if (ctx == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int rc = proj_validate(ctx, d, x, w, out);
  if (rc != ANIMAXS_OK) return rc;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  struct Restore {
    int dev, prev;
    ~Restore() {
      if (dev != prev) cudaSetDevice(prev);
    }
  } restore{ctx->device, prev};

  const bool f32_out = d->epilogue == ANIMAXS_PROJ_GATE_ADD;
  const bool rope = d->epilogue == ANIMAXS_PROJ_QKV_NORM && d->qk_norm == ANIMAXS_QK_RMS_ROPE;
  const bool quant = d->w_storage != ANIMAXS_WEIGHT_FP16;
  // Context scratch: the pair-major RoPE table, then the decoded fp16 weight.
  const size_t rope_bytes = rope ? (static_cast<size_t>(d->tokens) * 64 * 8 + 255) / 256 * 256 : 0;
  const size_t wdec_bytes = quant ? static_cast<size_t>(d->n) * d->k * 2 : 0;
  if (rope || quant) {
    rc = ax_ensure_scratch(ctx, rope_bytes + wdec_bytes);
    if (rc != ANIMAXS_OK) return rc;
  }
  const void* wmat = w;
  int64_t wstride = d->w_stride;
  if (quant) {
    // Decode the W8/W4 weight into fp16 (ordered before the GEMM on the same
    // stream), as the reference's dequantize-then-GEMM path.
    void* wdec = static_cast<char*>(ctx->scratch) + rope_bytes;
    cudaError_t e = ax::launch_dequant(d->w_storage == ANIMAXS_WEIGHT_W4 ? 4 : 8, w, d->w_scale, d->w_zero, wdec,
                                       d->n, d->k, d->w_packed_stride, d->k, ctx->num_sms,
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "weight decode");
    wmat = wdec;
    wstride = d->k;
  }
  CUtensorMap ta, tb, tout;
  rc = make_tmap_2d(ctx, &ta, x, false, d->k, d->m, d->x_stride, 64, 128);
  if (rc == ANIMAXS_OK) rc = make_tmap_2d(ctx, &tb, wmat, false, d->k, d->n, wstride, 64, 128);
  if (rc == ANIMAXS_OK)
    rc = f32_out ? make_tmap_2d(ctx, &tout, out, true, d->n, d->m, d->out_stride, 32, 128)
                 : make_tmap_2d(ctx, &tout, out, false, d->n, d->m, d->out_stride, 64, 128);
  if (rc != ANIMAXS_OK) return rc;

  ax::ProjParams p{};
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.tokens = d->tokens;
  p.mode = d->epilogue == ANIMAXS_PROJ_QKV_NORM ? ax::kProjQkvNorm
           : f32_out                            ? ax::kProjGateAdd
                                                : ax::kProjStore;
  p.q_cols = d->q_cols;
  p.k_cols = d->k_cols;
  p.q_w = static_cast<const __half*>(d->q_norm_weight);
  p.k_w = static_cast<const __half*>(d->k_norm_weight);
  p.rope = nullptr;
  if (rope) {
    // The epilogue reads the table pair-major: re-lay the `tokens` rows it uses
    // out into context scratch (ordered before the GEMM on the same stream).
    cudaError_t e = ax::launch_rope_pairs(d->rope_table, ctx->scratch, d->tokens, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "rope table re-layout");
    p.rope = static_cast<const float*>(ctx->scratch);
  }
  p.eps = d->eps > 0.f ? d->eps : 1e-6f;
  p.gate = d->gate;
  p.gate_stride = d->gate_stride;
  p.tiles_n = (d->n + 255) / 256;
  const long long tiles = static_cast<long long>((d->m + 255) / 256) * p.tiles_n;  // 256 x 256 (a CTA pair)
  if (tiles > 0x7fffffffLL) return ax_set_error(ctx, ANIMAXS_ERR_OVERFLOW, "projection too large");
  p.tiles = static_cast<int>(tiles);
  p.status = ctx->d_status;
  // Kernel timing (animaxs_attn_set_kernel_timing) brackets this launch too.
  cudaEvent_t ev_stop = nullptr;
  if (ctx->timing) {
    while (ctx->events.size() < ctx->events_used + 2) {
      cudaEvent_t ev;
      cudaError_t ce = cudaEventCreate(&ev);
      if (ce != cudaSuccess) return ax_cuda_fail(ctx, ce, "timing event");
      ctx->events.push_back(ev);
    }
    cudaEventRecord(ctx->events[ctx->events_used], static_cast<cudaStream_t>(stream));
    ev_stop = ctx->events[ctx->events_used + 1];
  }
  cudaError_t e = ax::launch_proj(ta, tb, tout, p, static_cast<cudaStream_t>(stream));
  if (ev_stop != nullptr && e == cudaSuccess) {
    cudaEventRecord(ev_stop, static_cast<cudaStream_t>(stream));
    ctx->events_used += 2;
  }
  if (e != cudaSuccess) {
    int regs = 0, threads = 0, ss = 0, sd = 0;
    ax::proj_kernel_attributes(&regs, &threads, &ss, &sd);
    return ax_set_error(ctx, ANIMAXS_ERR_CUDA,
                        "projection launch: %s (kernel: %d registers, max %d threads, %d B static + %d B "
                        "dynamic shared memory allowed)",
                        cudaGetErrorString(e), regs, threads, ss, sd);
  }
  ctx->last_error.clear();
  return ANIMAXS_OK;
}
