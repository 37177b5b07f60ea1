/*
 * animaxs_attn.h -- C ABI of libanimaxs_attn.so, the B200 (sm_100a) build of
 * the AnimaXS attention hot path.
 *
 * The reference exposes this path as the Swift class `AttentionExecutor`
 * (AnimaXS/Runtime/Metal/AttentionExecutor.swift:77-848), the Metal kernels it
 * and its callers encode (AnimaXS/Shaders/AnimaKernels.metal: rmsnorm_heads_half
 * :660-689, rms_rope_split_half :696-729, attention_softmax_rows :1051-1100,
 * dit_flash_attention_h128_q4_k32 :2193-2318), the RoPE table builders
 * (AnimaXS/Runtime/Text/DitRoPE.swift:58-107,
 * AnimaXS/Runtime/Metal/QwenEncoderMetal.swift:126-142) and the GQA rule
 * (AttentionExecutor.swift:222).  Each declaration below names the reference
 * interface it replaces.  A Swift caller binds this header through a module
 * map (`module CAnimaxsAttn { header "animaxs_attn.h" link "animaxs_attn" }`).
 *
 * Conventions
 *  - Plain C: pointers, sizes and a descriptor struct; no CUDA or C++ types.
 *    `stream` arguments are a `cudaStream_t` passed as `void*` (NULL = the
 *    legacy default stream).
 *  - Every call returns an `animaxs_status`; nothing aborts.  The message of
 *    the last failure on a context is returned by animaxs_attn_last_error().
 *  - Device buffers are fp16 (IEEE half) unless stated; every device pointer
 *    must be 16-byte aligned and every stride a multiple of 8 elements, which
 *    the Tensor Memory Accelerator requires (the reference requires 16-byte
 *    aligned offsets and row stride on its strided path, :799-805).
 *  - Work is enqueued on `stream` and is asynchronous, like the reference's
 *    `encode(commandBuffer:...)`.  A context is NOT reentrant: it owns scratch
 *    memory, exactly like the reference executor's BufferPool (:69-70).  Use one
 *    context per stream / host thread.
 */
#ifndef ANIMAXS_ATTN_H
#define ANIMAXS_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 2: animaxs_proj_desc gained the weight-storage fields (w_storage, w_scale,
 * w_zero, w_packed_stride); the peer-group and dequant entry points.
 * 3: animaxs_attn_desc gained `numerics`; the cross-K/V cache, weight
 * streamer and no-alloc status entry points. */
#define ANIMAXS_ATTN_ABI_VERSION 3

/* Status codes.  The reference throws AnimapkError.validation(String) for every
 * argument problem (AttentionExecutor.swift:778-825) and surfaces GPU errors as
 * `completed.error` (:771); here they are distinct negative codes. */
typedef enum animaxs_status {
  ANIMAXS_OK = 0,
  ANIMAXS_ERR_INVALID_ARG = -1, /* bad shape / offset / causal dims (:784-789) */
  ANIMAXS_ERR_UNSUPPORTED = -2, /* valid request this build does not run (:157,:174,:687) */
  ANIMAXS_ERR_OOB = -3,         /* "attention buffer range is out of bounds" (:817-823) */
  ANIMAXS_ERR_CUDA = -4,        /* CUDA runtime / launch failure */
  ANIMAXS_ERR_TIMEOUT = -5,     /* a bounded device-side wait expired */
  ANIMAXS_ERR_NO_DEVICE = -6,   /* no sm_100 device */
  ANIMAXS_ERR_NCCL = -7,        /* NCCL unavailable or a collective failed */
  ANIMAXS_ERR_OVERFLOW = -8,    /* "attention byte size overflow" (:830-838) */
  ANIMAXS_ERR_SCRATCH_LIMIT = -9 /* call needs more than animaxs_attn_forward_noalloc's fixed scratch */
} animaxs_status;

/* q/k normalisation fused in front of the attention.
 *  NONE     - q and k are used as given (AttentionExecutor.encode semantics).
 *  RMS      - per-(token, head) RMSNorm over head_dim with a shared weight;
 *             DiT cross-attention (rmsnorm_heads_half, AnimaKernels.metal:660-689,
 *             called at DiTBlockExecutor.swift:1608-1626).
 *  RMS_ROPE - RMSNorm then split-half RoPE (pairs p, p+head_dim/2) from a
 *             [rows, head_dim/2, 2, 2] fp32 table; DiT self-attention and Qwen
 *             (rms_rope_split_half, AnimaKernels.metal:696-729, called at
 *             DiTBlockExecutor.swift:1586-1606 and QwenEncoderMetal.swift:329-350). */
typedef enum animaxs_qk_norm {
  ANIMAXS_QK_NONE = 0,
  ANIMAXS_QK_RMS = 1,
  ANIMAXS_QK_RMS_ROPE = 2
} animaxs_qk_norm;

/* Which of q and k the qk_norm mode is applied to.  Q_ONLY serves callers that
 * keep k already normalised, such as the cross-K/V cache (CrossKVCache,
 * DiTBlockExecutor.swift:19-43; cached post-RMSNorm K reused across steps at
 * :1105-1161): normalise K once with animaxs_rmsnorm_heads_half, then pass it
 * with Q_ONLY.  0 (BOTH) is the zero-initialised default. */
typedef enum animaxs_qk_norm_targets {
  ANIMAXS_QK_NORM_BOTH = 0,
  ANIMAXS_QK_NORM_Q_ONLY = 1,
  ANIMAXS_QK_NORM_K_ONLY = 2
} animaxs_qk_norm_targets;

/* Arithmetic of the attention (`numerics:` of AttentionExecutor.init,
 * AttentionExecutor.swift:97-110).
 *  LEGACY  - fp32 scores (fp16 q.k products summed in fp32) and fp32 softmax
 *            statistics; the probabilities are rounded to fp16 for the P x V
 *            product (the reference's legacy path also rounds the scores).
 *  FP32_SCORES_AND_SOFTMAX - the reference's diagnostic mode (encodeFP32,
 *            AttentionExecutor.swift:325-405; kernels attention_qk_f16_to_f32,
 *            attention_softmax_rows_f32, attention_pv_f32_f16_to_f16,
 *            AnimaKernels.metal:1105-1185): fp32 scores, fp32 softmax and
 *            fp32 probabilities times fp16 V with fp32 accumulation.  Here P
 *            enters the tensor-core product as two fp16 terms, P_hi = fp16(P)
 *            and P_lo = fp16(P - P_hi), which together carry ~22 significant
 *            bits, and exp2 is evaluated on the SFU only.  About 1.3x the time
 *            of LEGACY.  Head dims 64 and 128.
 *  BF16_COMPUTE - an Apple5 bf16 rounding emulation: ANIMAXS_ERR_UNSUPPORTED. */
typedef enum animaxs_numerics {
  ANIMAXS_NUMERICS_LEGACY = 0,
  ANIMAXS_NUMERICS_FP32_SCORES_AND_SOFTMAX = 1,
  ANIMAXS_NUMERICS_BF16_COMPUTE = 2
} animaxs_numerics;

/* One attention call.  Replaces the argument list of
 * AttentionExecutor.encode(commandBuffer:query:queryOffset:key:...:heads:
 * queryCount:keyCount:headDim:keyValueHeads:causal:probe:layout:)
 * (AttentionExecutor.swift:122-133).  All strides are in fp16 ELEMENTS.
 * Token-major DiT tensors ([rows, heads*128]): tok_stride = heads*128,
 * head_stride = 128.  Head-major tensors ([heads, rows, 128], the Qwen layout):
 * tok_stride = 128, head_stride = rows*128. */
typedef struct animaxs_attn_desc {
  int32_t batch;        /* independent sequences (>= 1) */
  int32_t heads;        /* query heads, `heads:` */
  int32_t kv_heads;     /* `keyValueHeads:`; query head h reads kv head h / (heads/kv_heads) */
  int32_t q_len;        /* `queryCount:` */
  int32_t kv_len;       /* `keyCount:` */
  int32_t head_dim;     /* `headDim:`; this build runs 128 (DiT, Qwen), 64 (LLM adapter,
                           LLMAdapterMetal.swift:9-10,394-397), 384 (VAE middle attention,
                           VAEDecoder.swift:398-404: heads 1) and 256; others -> UNSUPPORTED.
                           qk_norm other than NONE needs 128 or 64. */
  int64_t q_tok_stride, q_head_stride, q_batch_stride;
  int64_t k_tok_stride, k_head_stride, k_batch_stride;
  int64_t v_tok_stride, v_head_stride, v_batch_stride;
  int64_t o_tok_stride, o_head_stride, o_batch_stride;
  int32_t causal;       /* `causal:`; requires q_len == kv_len (:787); key j visible to row i iff j <= i */
  int32_t kv_valid_len; /* key padding: keys >= kv_valid_len are masked for every batch;
                           0 means kv_len (no padding, the reference's semantics) */
  const int32_t* kv_valid_lens; /* optional DEVICE int32[batch]; overrides kv_valid_len per batch */
  float scale;          /* softmax scale; 0 means 1/sqrt(head_dim) (:139) */
  int32_t qk_norm;      /* animaxs_qk_norm */
  float eps;            /* RMSNorm epsilon; 0 means 1e-6 */
  const void* q_norm_weight; /* DEVICE fp16[head_dim] shared by all heads, or NULL for ones */
  const void* k_norm_weight; /* DEVICE fp16[head_dim], or NULL for ones */
  const float* rope_table;   /* DEVICE fp32[rope_rows][head_dim/2][2][2] blocks [cos,-sin,sin,cos];
                                row = token index; RMS_ROPE only */
  int32_t rope_rows;         /* rows in rope_table; must be >= max(q_len, kv_len) */
  int32_t qk_norm_targets;   /* animaxs_qk_norm_targets; 0 = q and k */
  /* Optional extents (bytes from the pointer passed to the call) used for the
   * reference's range validation (:808-823); 0 = not checked. */
  int64_t q_bytes, k_bytes, v_bytes, o_bytes;
  int32_t numerics;          /* animaxs_numerics; 0 = LEGACY */
} animaxs_attn_desc;

typedef struct animaxs_attn_ctx animaxs_attn_ctx;

/* ABI version of the loaded library (ANIMAXS_ATTN_ABI_VERSION). */
int animaxs_attn_abi_version(void);

/* Create / destroy an executor context on `device`.  Replaces
 * AttentionExecutor.init(context:tileRows:numerics:monitor:layout:attentionBackend:)
 * (AttentionExecutor.swift:97-110); the context owns its scratch like the
 * reference's BufferPool.  Fails with ANIMAXS_ERR_NO_DEVICE when `device` is
 * not an sm_100 GPU (there is no CPU fallback). */
int animaxs_attn_create(int device, animaxs_attn_ctx** out);
int animaxs_attn_destroy(animaxs_attn_ctx* ctx);

/* Message describing the most recent failure on `ctx` ("" after success). */
const char* animaxs_attn_last_error(const animaxs_attn_ctx* ctx);

/* Fill `desc` with defaults for a packed token-major call
 * ([batch, len, heads*128] q/o, [batch, len, kv_heads*128] k/v). */
int animaxs_attn_desc_init(animaxs_attn_desc* desc, int batch, int heads, int kv_heads,
                           int q_len, int kv_len, int head_dim);

/* Validate `desc` exactly as animaxs_attn_forward does, without a GPU.
 * Mirrors AttentionExecutor.validate (AttentionExecutor.swift:778-825). */
int animaxs_attn_validate(animaxs_attn_ctx* ctx, const animaxs_attn_desc* desc,
                          const void* q, const void* k, const void* v, const void* o);

/* Fused attention: (optional q/k RMSNorm [+ split-half RoPE]) -> softmax(q k^T * scale
 * + masks) v, fp32 accumulation, fp16 output.  Replaces AttentionExecutor.encode
 * (AttentionExecutor.swift:122-302) together with the rms/rope encodes its
 * callers issue in front of it (DiTBlockExecutor.swift:1139-1172,
 * QwenEncoderMetal.swift:264-279).  Asynchronous on `stream`. */
int animaxs_attn_forward(animaxs_attn_ctx* ctx, const animaxs_attn_desc* desc,
                         const void* q, const void* k, const void* v, void* o, void* stream);

/* Wait for the work enqueued on `stream` and report device-side failures
 * (a bounded wait that expired -> ANIMAXS_ERR_TIMEOUT; a CUDA error ->
 * ANIMAXS_ERR_CUDA).  Replaces the completion half of
 * AttentionExecutor.execute(...) async throws (AttentionExecutor.swift:751-776),
 * which awaits the command buffer and rethrows `completed.error`. */
int animaxs_attn_synchronize(animaxs_attn_ctx* ctx, void* stream);

/* Scratch bytes the fused q/k normalisation of a call with `desc` needs when
 * it runs as a prologue: the normalised copy of q (unless qk_norm_targets is
 * K_ONLY) and, at the next 256-byte boundary, of k (unless Q_ONLY); 0 for
 * qk_norm NONE; animaxs_attn_forward's context scratch and
 * animaxs_attn_forward_noalloc's fixed array hold exactly this.  Replaces
 * maximumScoreScratchBytes(keyCount:queryCount:) (AttentionExecutor.swift:112-120);
 * the flash kernel itself needs no score scratch. */
int animaxs_attn_scratch_bytes(const animaxs_attn_desc* desc, int64_t* bytes);


/* Number of (head, 128-row query tile) units executed on this context since
 * creation; the counter the reference keeps with
 * MetricsCollector.recordAttentionQueryTile (GenerationMetrics.swift:490-510). */
int animaxs_attn_query_tiles(const animaxs_attn_ctx* ctx, int64_t* tiles);

/* Opt-in GPU timing of the flash-attention kernel: when enabled, every
 * animaxs_attn_forward on this context brackets the attention kernel (not the
 * q/k prologue) with a pair of CUDA events on the caller's stream.
 * animaxs_attn_kernel_timing waits for the recorded events, returns the
 * launch count, the summed and the largest per-launch time in milliseconds,
 * and clears the record.  Counterpart of the reference's GPU stage timers
 * (MetricsCollector, GenerationMetrics.swift:325-610, fed from
 * command.gpuStartTime/gpuEndTime, DiTBlockExecutor.swift:265-270). */
int animaxs_attn_set_kernel_timing(animaxs_attn_ctx* ctx, int enable);
int animaxs_attn_kernel_timing(animaxs_attn_ctx* ctx, int64_t* launches, double* total_ms,
                               double* max_ms);

/* Numerical health of the attention scores: the reference's score probes
 * (NumericalMonitor .selfScores / .crossScores, bound by encode(probe:) to
 * attention_softmax_rows_probe, AttentionExecutor.swift:148,266 and
 * AnimaKernels.metal:1738-1830).  While `stats` is set, every forward call on
 * this context folds the health of its scaled scores (scale * q.k over the
 * unmasked keys) into the probe slot `stats`, DEVICE uint32[4] with the
 * reference's layout (NumericalMonitor.swift:17-119):
 *   [0] |= flags    ANIMAXS_PROBE_* below
 *   [1]  = max of the float bits of |score| over the finite scores
 *   [2]  = min key index of a flagged score (initialise to 0xFFFFFFFF)
 *   [3]    unused
 * The words are updated with device atomics in stream order; NULL turns the
 * probe off.  Head dims 64 and 128 (the DiT and adapter calls); set with head
 * dim 256 or 384 a forward call returns ANIMAXS_ERR_UNSUPPORTED.  The
 * reference's scores are fp16 (a score beyond 65504 is stored as Inf there);
 * here they are fp32, so such a score raises ANIMAXS_PROBE_HALF_OVERFLOW and
 * keeps its magnitude. */
#define ANIMAXS_PROBE_NAN 1u
#define ANIMAXS_PROBE_POS_INF 2u
#define ANIMAXS_PROBE_NEG_INF 4u
#define ANIMAXS_PROBE_HALF_OVERFLOW 8u
int animaxs_attn_set_score_probe(animaxs_attn_ctx* ctx, unsigned int* stats);

/* Standalone per-(token, head) RMSNorm + split-half RoPE, fp16 in/out
 * ([tokens, heads, head_dim] rows, `row_stride` elements apart per token),
 * in place allowed.  Replaces kernel rms_rope_split_half
 * (AnimaKernels.metal:696-729) at head_dim 128 and rms_rope_adapter64
 * (AnimaKernels.metal:733-763) at head_dim 64.  `rope_table` is DEVICE fp32
 * [tokens][head_dim/2][2][2]; `weight` DEVICE fp16[head_dim] or NULL. */
int animaxs_rms_rope_split_half(animaxs_attn_ctx* ctx, const void* in, void* out,
                                const void* weight, const float* rope_table,
                                int tokens, int heads, int head_dim, int64_t row_stride,
                                float eps, void* stream);

/* Standalone per-(token, head) RMSNorm without RoPE.  Replaces kernel
 * rmsnorm_heads_half (AnimaKernels.metal:660-689). */
int animaxs_rmsnorm_heads_half(animaxs_attn_ctx* ctx, const void* in, void* out,
                               const void* weight, int tokens, int heads, int head_dim,
                               int64_t row_stride, float eps, void* stream);

/* ---- Cross-attention K/V cache ---------------------------------------------
 * Replaces CrossKVCache (DiTBlockExecutor.swift:19-43) and its use by the DiT
 * block (:1105-1161): the cross-attention K and V of every block depend only
 * on the LLM-adapter context, so they are projected (and K RMS-normalised)
 * once per generation and reused by the other Euler steps.  A cache holds
 * `blocks` blocks of [batch][tokens][K | V] fp16 rows: a token's row is its
 * kv_heads x head_dim K values followed by its kv_heads x head_dim V values
 * (token stride 2 x kv_heads x head_dim elements).  Attention reads a block in
 * place: pass the pointers and strides from animaxs_cross_kv_cache_block as k
 * and v with qk_norm RMS and qk_norm_targets Q_ONLY (the reference blits a hit
 * back into its scratch instead).  Like the reference's cache it belongs to
 * one generation; animaxs_cross_kv_cache_reset starts the next.  Not
 * reentrant; work is enqueued on `stream`. */
typedef struct animaxs_cross_kv_cache animaxs_cross_kv_cache;

/* Device bytes of a cache (CrossKVCache.blockStride x blockCount). */
int animaxs_cross_kv_cache_bytes(int blocks, int batch, int tokens, int kv_heads, int head_dim,
                                 int64_t* bytes);

/* A cache on ctx's device (head_dim 64 or 128).  `memory` (256-byte aligned,
 * >= animaxs_cross_kv_cache_bytes) is used if given, else the cache allocates
 * its own (CrossKVCache.init, :30-36); the cache keeps `ctx` for errors and launches. */
int animaxs_cross_kv_cache_create(animaxs_attn_ctx* ctx, int blocks, int batch, int tokens, int kv_heads,
                                  int head_dim, void* memory, int64_t memory_bytes,
                                  animaxs_cross_kv_cache** out);
int animaxs_cross_kv_cache_destroy(animaxs_cross_kv_cache* cache);

/* Store block `block` from projected K and V ([batch][tokens][kv_heads x
 * head_dim] fp16, token / batch strides in elements).  With k_norm = 1, K is
 * RMS-normalised with `k_norm_weight` (fp16[head_dim] or NULL) by the same
 * kernel as the attention prologue, so attention on the cached block equals
 * the uncached fused call bit for bit; k_norm = 0 stores K as given.  Marks
 * the block ready (the miss path of :1123-1160: project, RMSNorm K, store). */
int animaxs_cross_kv_cache_fill(animaxs_cross_kv_cache* cache, int block, const void* k, int64_t k_tok_stride,
                                int64_t k_batch_stride, const void* v, int64_t v_tok_stride,
                                int64_t v_batch_stride, int k_norm, const void* k_norm_weight, float eps,
                                void* stream);

/* Store block `block` straight from the adapter context: one fused projection
 * of `context` ([batch x tokens][context_dim] fp16, rows context_stride
 * elements apart) against `w_kv` ([2 x kv_heads x 128][context_dim]: the
 * cross W_k rows, then the cross W_v rows; rows w_stride apart), the
 * projection rounded to fp16 and the K columns RMS-normalised in the
 * epilogue (animaxs_proj_forward with ANIMAXS_PROJ_QKV_NORM).  head_dim 128.
 * Marks the block ready. */
int animaxs_cross_kv_cache_project(animaxs_cross_kv_cache* cache, int block, const void* context,
                                   int64_t context_stride, int context_dim, const void* w_kv, int64_t w_stride,
                                   const void* k_norm_weight, float eps, void* stream);

/* Block `block`'s K and V device pointers, token and batch strides (elements)
 * and whether it is ready (CrossKVCache.kOffset / vOffset / isReady, :38-41). */
int animaxs_cross_kv_cache_block(const animaxs_cross_kv_cache* cache, int block, void** k, void** v,
                                 int64_t* tok_stride, int64_t* batch_stride, int* ready);
/* CrossKVCache.markReady (:42) for a block the caller filled itself; reset
 * marks every block not ready. */
int animaxs_cross_kv_cache_mark_ready(animaxs_cross_kv_cache* cache, int block, int ready);
int animaxs_cross_kv_cache_reset(animaxs_cross_kv_cache* cache);

/* ---- Weight streaming --------------------------------------------------------
 * Replaces WeightStreamer (WeightStreamer.swift:84-213): bounded device memory
 * of 1 to 4 slots of `capacity` bytes, each loaded with one execution range of
 * a weight pack (the W8/W4 codes, scales and zeros of a block, as the
 * reference's .animapk ranges) from host memory, and never overwritten while
 * queued work still reads it.  The reference copies with the CPU and
 * ping-pongs two slots so that block n+1's copy overlaps block n's GPU work
 * (DiTBlockExecutor.swift:222-260); here a load is an asynchronous
 * host-to-device copy on the caller's stream (use a copy stream to overlap),
 * and the ordering is kept on the GPU with events:
 *  - load: copies `bytes` from host `src` into `slot` on `stream` and records
 *    the slot's "loaded" event; if the slot was marked in flight, the copy
 *    first waits (on the GPU) for that mark, so in-flight readers always see
 *    the old contents.  Ranges larger than the slot are refused ("execution
 *    range does not fit the weight slot").
 *  - wait_loaded: `consumer_stream` waits (on the GPU) for the slot's last load.
 *  - mark_in_flight: records that work queued on `consumer_stream` reads the
 *    slot (markInFlight); complete clears the mark when the caller knows that
 *    work has finished (complete).
 *  - register_host: pins a host range (cudaHostRegister, read-only), e.g. the
 *    mapped pack file, so its loads run as DMA at PCIe speed; undone at destroy.
 * The slots hold whatever the caller loads; animaxs_proj_forward reads W8/W4
 * weights straight from a slot (w, w_scale, w_zero point into it). */
typedef struct animaxs_weight_streamer animaxs_weight_streamer;
int animaxs_weight_streamer_create(animaxs_attn_ctx* ctx, int64_t capacity, int slots,
                                   animaxs_weight_streamer** out);
int animaxs_weight_streamer_destroy(animaxs_weight_streamer* streamer);
int animaxs_weight_streamer_register_host(animaxs_weight_streamer* streamer, void* base, int64_t bytes);
int animaxs_weight_streamer_load(animaxs_weight_streamer* streamer, int slot, const void* src, int64_t bytes,
                                 int64_t logical_index, void* stream);
/* Device address of `slot` (256-byte aligned), NULL for a bad slot. */
void* animaxs_weight_streamer_slot(const animaxs_weight_streamer* streamer, int slot);
int animaxs_weight_streamer_wait_loaded(animaxs_weight_streamer* streamer, int slot, void* consumer_stream);
int animaxs_weight_streamer_mark_in_flight(animaxs_weight_streamer* streamer, int slot, void* consumer_stream);
int animaxs_weight_streamer_complete(animaxs_weight_streamer* streamer, int slot);
/* The logical index of the slot's last load (-1: none) and whether it is
 * marked in flight (loadedLogicalIndexes / inFlightSlotSet). */
int animaxs_weight_streamer_state(animaxs_weight_streamer* streamer, int slot, int64_t* logical_index,
                                  int* in_flight);

/* Host helpers (no GPU).  DiT 3-D RoPE table [T*H*W][64][2][2] fp32 with the
 * t/h/w = 44/42/42 dim split, theta_hw = 10000*4^(42/40), theta_t = 1e4.
 * Replaces DitRoPE.generate(T:H:W:) (DitRoPE.swift:58-107).  `out` holds
 * T*H*W*256 floats. */
int animaxs_rope3d_table(int T, int H, int W, float* out);

/* 1-D NeoX RoPE table [seq_len][head_dim/2][2][2] fp32, inv_freq =
 * theta^(-2p/head_dim).  Replaces QwenEncoderMetal.makeRope(tokens:)
 * (QwenEncoderMetal.swift:126-142: head_dim 128, theta 1e6) and
 * LLMAdapterMetal.makeRope(tokens:key:) (LLMAdapterMetal.swift:162-178:
 * head_dim 64, theta 1e4). */
int animaxs_rope1d_table(int seq_len, int head_dim, double theta, float* out);

/* GQA head map: kv head read by query head `query_head`
 * (AttentionExecutor.swift:222; GqaHeadMappingTests.swift:17-21).
 * Returns < 0 (ANIMAXS_ERR_INVALID_ARG) if heads is not a multiple of kv_heads. */
int animaxs_gqa_kv_head(int query_head, int heads, int kv_heads);

/* Allocation-free variant of animaxs_attn_forward.  No counterpart exists in
 * the reference; it is for callers that must not have device memory allocated
 * behind their back -- an application that reserves the device's memory up
 * front, a host runtime whose allocator owns every device allocation, or a
 * latency-critical loop in which an allocation (which may synchronise the
 * device) is unacceptable.  It runs the same kernels, but the normalised q/k
 * copies of the fused prologue live in one fixed 32 MiB device array that
 * every GPU loading the library holds until the process exits; it takes no
 * context and allocates nothing.  Works on the CURRENT device.
 *  - A call needing more than 32 MiB of normalised q/k (see
 *    animaxs_attn_scratch_bytes) fails with ANIMAXS_ERR_SCRATCH_LIMIT, e.g. the
 *    16384-token self-attention; qk_norm = NONE needs none.
 *  - All calls on a device share the array and it keeps the last call's
 *    contents (every byte read is rewritten first); calls that overlap on the
 *    GPU race on it, so serialise them.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress); make that call before any stream capture.  The
 *    address is kept for the life of the process, so it goes stale after
 *    cudaDeviceReset: do not use this entry point across a device reset.
 *  - Returns status codes only (no last-error text).  A bounded device-side
 *    wait that expires is recorded in a fixed device word of the current
 *    device, read with animaxs_attn_noalloc_status. */
int animaxs_attn_forward_noalloc(const animaxs_attn_desc* desc, const void* q, const void* k,
                                 const void* v, void* o, void* stream);

/* Read and clear the current device's status word of
 * animaxs_attn_forward_noalloc: ANIMAXS_ERR_TIMEOUT when a bounded
 * device-side wait of one of its calls expired since the last read, else
 * ANIMAXS_OK.  Synchronise the streams of the calls it should cover first.
 * Allocates nothing. */
int animaxs_attn_noalloc_status(void);

/* Failure-detection self-test: enqueue one kernel whose only thread waits,
 * through the same bounded device-side wait every kernel here uses, on a
 * barrier phase that nothing completes; after `timeout_ns` (<= 10 s) it sets
 * the context's status word and returns, exactly as a kernel whose wait ran
 * out does.  The next animaxs_attn_synchronize on the stream then returns
 * ANIMAXS_ERR_TIMEOUT (and clears the status); the context stays usable.
 * Nothing faults or hangs.  Counterpart of the reference's numerical-failure
 * detection surfacing a GPU error through `completed.error`
 * (AttentionExecutor.swift:771). */
int animaxs_attn_selftest_wait_timeout(animaxs_attn_ctx* ctx, int64_t timeout_ns, void* stream);

/* ---- Fused attention projections ------------------------------------------
 * The GEMMs on either side of DiT attention, each with its elementwise step
 * fused into the epilogue (one kernel per call).  The reference encodes them
 * separately: LinearExecutor.encode (LinearExecutor.swift:79-) for q, k, v
 * (DiTBlockExecutor.swift:1097-1131), then rms_rope_split_half /
 * rmsnorm_heads_half on q and k (AnimaKernels.metal:660-729); after attention
 * the out-projection and gate_add_half_f32 (DiTBlockExecutor.swift:1223-1236,
 * AnimaKernels.metal:624-634).  x [m][k] and w [n][k] are fp16 (w is the
 * reference's [out][in] weight); accumulation is fp32 and the projection is
 * rounded to fp16 before any epilogue math, as the reference's fp16 output. */
typedef enum animaxs_proj_epilogue {
  ANIMAXS_PROJ_STORE = 0,    /* out fp16 [m][out_stride] = fp16(x w^T) */
  ANIMAXS_PROJ_QKV_NORM = 1, /* as STORE; q and k heads then RMS-normalised (+ RoPE), v stored as is:
                                a fused q|k|v projection ready for animaxs_attn_forward with
                                qk_norm = NONE (strided views of `out`) */
  ANIMAXS_PROJ_GATE_ADD = 2  /* residual fp32 [m][out_stride] += float(fp16(x w^T)) * gate[row/tokens][col]
                                (gate_add_half_f32; `out` is the residual) */
} animaxs_proj_epilogue;

/* Weight storage of a projection (the reference's QuantizedLinearWeightBuffers,
 * LinearExecutor.swift:12-40 and :460-520): fp16, or W8 / W4 codes with a
 * per-row, per-64-column fp16 scale and zero, decoded as
 * half(float(q) * float(scale) + float(zero)) (AnimaKernels.metal:19-67). */
typedef enum animaxs_weight_storage {
  ANIMAXS_WEIGHT_FP16 = 0,
  ANIMAXS_WEIGHT_W8 = 1,  /* one byte per value */
  ANIMAXS_WEIGHT_W4 = 2   /* two values per byte, even column in the low nibble */
} animaxs_weight_storage;

typedef struct animaxs_proj_desc {
  int32_t m;                 /* rows = images x tokens (`inputRows:`) */
  int32_t n;                 /* output features (rows of w) */
  int32_t k;                 /* input features, a multiple of 8 */
  int64_t x_stride;          /* elements between rows of x (>= k, multiple of 8) */
  int64_t w_stride;          /* elements between rows of w (>= k, multiple of 8) */
  int64_t out_stride;        /* elements between rows of out (>= n; multiple of 8 fp16 / 4 fp32) */
  int32_t epilogue;          /* animaxs_proj_epilogue */
  int32_t tokens;            /* rows per image: RoPE row = row % tokens, gate row = row / tokens */
  int32_t qk_norm;           /* QKV_NORM: ANIMAXS_QK_RMS or ANIMAXS_QK_RMS_ROPE */
  int32_t q_cols;            /* QKV_NORM: columns [0, q_cols) are q heads of 128 */
  int32_t k_cols;            /* QKV_NORM: columns [q_cols, q_cols + k_cols) are k heads of 128 */
  int32_t rope_rows;         /* rows of rope_table (>= tokens) */
  const void* q_norm_weight; /* DEVICE fp16[128] shared by all q heads, or NULL for ones */
  const void* k_norm_weight; /* DEVICE fp16[128], or NULL for ones */
  const float* rope_table;   /* DEVICE fp32[rope_rows][64][2][2] blocks [cos,-sin,sin,cos] */
  float eps;                 /* RMSNorm epsilon; 0 means 1e-6 */
  int32_t w_storage;         /* animaxs_weight_storage of `w` */
  const float* gate;         /* GATE_ADD: DEVICE fp32 [m / tokens][gate_stride] */
  int64_t gate_stride;       /* elements between images' gate rows (>= n) */
  const void* w_scale;       /* W8/W4: DEVICE fp16 [n][ceil(k / 64)] */
  const void* w_zero;        /* W8/W4: DEVICE fp16 [n][ceil(k / 64)] */
  int64_t w_packed_stride;   /* W8/W4: bytes between packed rows of `w` (>= k or ceil(k / 2)) */
} animaxs_proj_desc;

/* Dense defaults: fp16 weights, strides = k / k / n, tokens = m, eps 1e-6.
 * With W8/W4 weights the call first decodes them into context scratch
 * (n * k * 2 bytes, as the reference's dequantized-MPS path), then runs the
 * same GEMM. */
int animaxs_proj_desc_init(animaxs_proj_desc* desc, int m, int n, int k, int epilogue);
/* Validate exactly as animaxs_proj_forward does, without a GPU. */
int animaxs_proj_validate(animaxs_attn_ctx* ctx, const animaxs_proj_desc* desc, const void* x,
                          const void* w, const void* out);
/* Enqueue the fused projection on `stream` (bracketed by CUDA events, like
 * the attention kernel, while animaxs_attn_set_kernel_timing is on). */
int animaxs_proj_forward(animaxs_attn_ctx* ctx, const animaxs_proj_desc* desc, const void* x,
                         const void* w, void* out, void* stream);

/* Decode W8 (bits 8) or W4 (bits 4) codes `packed` [rows][packed_stride bytes]
 * with fp16 `scale` / `zero` [rows][ceil(k / 64)] into fp16 `out`
 * [rows][out_stride elements]: out = half(float(q) * float(scale) + float(zero)),
 * rounded once after the multiply and once after the add.  Replaces
 * dequant_w8_to_half / dequant_w4_to_half (AnimaKernels.metal:19-67). */
int animaxs_dequant_to_half(animaxs_attn_ctx* ctx, int bits, const void* packed, const void* scale,
                            const void* zero, void* out, int rows, int k, int64_t packed_stride,
                            int64_t out_stride, void* stream);

/* ---- Multi-GPU: heads sharded across ranks + one NCCL all-gather ----------
 * No counterpart exists in the reference (a single-device app); this serves
 * the 16K-token DiT configuration.  NCCL is loaded at run time (dlopen of
 * libnccl.so.2), so the library has no link-time NCCL dependency. */
typedef struct animaxs_comm animaxs_comm;

/* 128-byte NCCL unique id produced on rank 0 and shared by the caller. */
int animaxs_comm_unique_id(void* id128);
int animaxs_comm_create(animaxs_attn_ctx* ctx, int world, int rank, const void* id128,
                        animaxs_comm** out);
int animaxs_comm_destroy(animaxs_comm* comm);

/* Rank `rank` of `world` computes query heads [rank*heads/world, (rank+1)*heads/world)
 * of `desc` (q/k/v/o pointers are the FULL tensors, identical on every rank),
 * then one ncclAllGather assembles every rank's heads into `o`, so every rank
 * ends with the complete output.  heads must be a multiple of world; head_dim
 * 128 or 64. */
int animaxs_attn_forward_head_sharded(animaxs_attn_ctx* ctx, animaxs_comm* comm,
                                      const animaxs_attn_desc* desc, const void* q,
                                      const void* k, const void* v, void* o, void* stream);

/* ---- Multi-GPU, fused: heads sharded, the gather done by the attention kernel
 * Same split of the heads as animaxs_attn_forward_head_sharded, without NCCL:
 * every rank's output buffer is mapped into every other rank's process (CUDA
 * IPC over NVLink / NVSwitch), the attention kernel stores each finished output
 * tile into every rank's buffer, and a one-block handshake before and after
 * (bounded waits on system-scope flags) orders the calls.
 *
 * Setup, on every rank: animaxs_peer_group_create allocates this rank's output
 * buffer (output_bytes, plus the flags) and returns its 64-byte IPC handle; the
 * caller exchanges the handles (any side channel, rank order); then
 * animaxs_peer_group_connect maps the peers' buffers.  Every call passes
 * o = animaxs_peer_group_output(group) with the same descriptor on all ranks,
 * in the same order (like a collective); the output stays valid until this
 * rank's next call.  A peer that does not arrive within ANIMAXS_WAIT_TIMEOUT
 * (2 s) makes animaxs_attn_synchronize report ANIMAXS_ERR_TIMEOUT; the group
 * must then be destroyed and recreated.  A call whose opening handshake timed
 * out stores nothing into any peer (a peer that was not seen ready may still
 * be reading its previous output) and adds no arrivals, so the peers' own
 * closing waits report the failure as well.
 * Teardown: every rank must be past its last call -- synchronised, and then a
 * barrier across the ranks -- before any rank calls animaxs_peer_group_destroy,
 * because destroy frees this rank's buffer, into which a slower peer may still
 * be storing. */
typedef struct animaxs_peer_group animaxs_peer_group;

int animaxs_peer_group_create(animaxs_attn_ctx* ctx, int world, int rank, int64_t output_bytes,
                              animaxs_peer_group** out, void* ipc_handle64);
int animaxs_peer_group_connect(animaxs_peer_group* group, const void* handles64 /* world x 64 B */);
void* animaxs_peer_group_output(animaxs_peer_group* group);
int animaxs_peer_group_destroy(animaxs_peer_group* group);
int animaxs_attn_forward_head_sharded_peer(animaxs_attn_ctx* ctx, animaxs_peer_group* group,
                                           const animaxs_attn_desc* desc, const void* q,
                                           const void* k, const void* v, void* o, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ANIMAXS_ATTN_H */
