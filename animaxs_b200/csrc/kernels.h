// kernels.h -- host-side launch interface of the CUDA kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ax {

// Parameters of the flash-attention kernels (attn_fwd_sm100.cu, attn_wide_sm100.cu).  q/k/v arrive
// through TMA tensor maps over [batch][head][token][head_dim] fp16 views (any
// strides); the output leaves through TMA tensor stores from a shared-memory
// stage (the launchers build its tensor map from `o` and the strides below).
struct AttnFwdParams {
  int head_dim;          // 64 or 128 (attn_fwd_sm100.cu), 256 or 384 (attn_wide_sm100.cu)
  int q_len;
  int kv_len;
  int heads_per_kv;      // heads / kv_heads (GQA group size)
  int kv_valid;          // keys >= kv_valid masked (already clamped to [1, kv_len])
  const int* kv_valid_dev;  // optional per-batch override (device)
  int causal;
  int n_q_tiles;         // query tiles per head: pairs or single 128-row tiles (head dims 64 / 128,
                         // chosen by launch_attn_fwd), 128-row tiles (wide)
  int single_tiles;      // set by launch_attn_fwd (head dims 64 / 128): items are single 128-row tiles
  int head_offset;       // first query head handled by this launch
  int heads_in_launch;   // set by launch_attn_fwd: query heads of this launch
  int n_items;           // set by launch_attn_fwd: n_q_tiles * heads_in_launch * batch
  int n_split;           // set by the wide launcher: CTAs (one cluster) sharing a query tile's keys
  int o_head_base;       // output head index = h - o_head_base
  float scale_log2;      // softmax scale * log2(e)
  __half* o;
  long long o_tok, o_head, o_batch;  // output strides (elements)
  unsigned int* status;  // device status word (bit 0: a bounded wait timed out)
  unsigned int* probe;   // score-health slot uint32[4] (animaxs_attn_set_score_probe) or nullptr
  int fp32_p;            // FP32_SCORES_AND_SOFTMAX: P x V from fp32 P (hi + lo fp16 terms)
  // Fused head-sharded gather (head dims 64 / 128; n_peers = 0 otherwise): the
  // epilogue also stores every output tile at the same offset in each peer's
  // output (peer GPU memory mapped into this process), and each CTA that
  // finished without a timeout adds its item count to every peer's arrival
  // word for this rank.
  int n_peers;
  long long peer_delta[7];           // bytes from `o` to the peer's copy of it
  unsigned int* peer_arrive[7];      // the peer's arrival word for this rank
  // The peer stores and arrivals happen only if *peer_go == peer_go_value:
  // the handshake before the call writes it when every peer was ready.
  const unsigned int* peer_go;
  unsigned int peer_go_value;
};

constexpr int kMaxPeers = 7;  // 8 GPUs per node

constexpr unsigned int kStatusTimeoutBit = 1u;  // a bounded device wait expired

constexpr int kTileM = 128;   // query rows per CTA
constexpr int kTileN = 128;   // keys per K/V tile
constexpr int kHeadDim = 128;   // DiT / Qwen; the LLM adapter runs 64

// One normalisation job: a [batch][tokens][heads][head_dim] fp16 tensor with strides.
struct NormJob {
  const __half* in;
  __half* out;
  long long in_tok, in_head, in_batch;
  long long out_tok, out_head, out_batch;
  int tokens, heads, batch;
  const __half* weight;  // shared [128] weight or nullptr (ones)
  long long rows;        // batch * tokens * heads
};

struct NormParams {
  NormJob job[2];
  int njobs;
  int head_dim;          // 64 or 128
  float eps;
  const float* rope;     // [tokens][head_dim/2][2][2] or nullptr (no rotation)
  unsigned int* status;  // device status word (nullable)

};

cudaError_t launch_attn_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const AttnFwdParams& p, int heads_in_launch, int batch,
                            cudaStream_t stream);

// Head dim 64 / 128, one query tile per item with three score buffers in TMEM
// (attn_s3_sm100.cu; called by launch_attn_fwd).
cudaError_t launch_attn_s3(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const AttnFwdParams& p, int heads_in_launch, int batch, int dev, int sms,
                           cudaStream_t stream);

// Head dims 256 / 384 (called by launch_attn_fwd).
cudaError_t launch_attn_wide(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnFwdParams& p, int heads_in_launch, int batch, int dev,
                             cudaStream_t stream);

int attn_fwd_rows_per_cta();  // query rows of a paired work item (head dims 64 / 128)
// Work items launch_attn_fwd deals for head dims 64 / 128 (pairs of query
// tiles, or single tiles when pairs would leave more than half of `sms` idle,
// or, for a launch with peer stores, any of them idle).
long long attn_fwd_work_items(int q_len, int heads_in_launch, int batch, int sms, bool peers);

cudaError_t launch_qk_norm(NormParams p, cudaStream_t stream);

// Peer handshake of the fused head-sharded path (peer_sync.cu): one block adds
// `add` to each peer's word `signal[i]` (release, system scope), then waits
// until every own word `wait[i]` (i != rank) has reached `target` (acquire,
// system scope; bounded by timeout_ns, after which kStatusTimeoutBit is set)
// and, if no wait gave up, writes `go_value` to `go`.
struct PeerSyncParams {
  unsigned int* signal[8];   // peers' words for this rank (mapped here); nullptr: no signal
  unsigned int add;
  const unsigned int* wait;  // this rank's [world] words
  unsigned int target;
  int world, rank;
  unsigned long long timeout_ns;
  unsigned int* status;
  unsigned int* go;          // set to go_value when every wait succeeded (nullptr: not written)
  unsigned int go_value;
};
cudaError_t launch_peer_sync(const PeerSyncParams& p, cudaStream_t stream);

// Fused attention projections (proj_sm100.cu): out = x w^T over fp16 operands
// with fp32 accumulation, then one of three epilogues.
enum ProjMode : int {
  kProjStore = 0,    // out fp16 = fp16(acc)
  kProjQkvNorm = 1,  // q / k column ranges: per-128-column-head RMSNorm (+ split-half RoPE)
  kProjGateAdd = 2,  // residual fp32 += float(fp16(acc)) * gate[row / tokens][col]
};
struct ProjParams {
  int m, n, k;
  int tokens;               // rows per image (RoPE row = row % tokens, gate row = row / tokens)
  int mode;                 // ProjMode
  int q_cols, k_cols;       // kProjQkvNorm: [0, q_cols) q heads, [q_cols, q_cols + k_cols) k heads
  const __half* q_w;        // kProjQkvNorm: shared [128] norm weights, or nullptr (ones)
  const __half* k_w;
  const float* rope;        // pair-major [64][tokens] (cos, sin) float2 (launch_rope_pairs), or nullptr
  float eps;
  const float* gate;        // kProjGateAdd: [images][gate_stride] fp32
  long long gate_stride;
  int tiles_n;              // ceil(n / 256)
  int tiles;                // ceil(m / 256) * tiles_n (256 x 256 tiles, one per CTA pair)
  unsigned int* status;
};
cudaError_t launch_proj(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tout,
                        const ProjParams& p, cudaStream_t stream);
int proj_kernel_attributes(int* regs, int* max_threads, int* smem_static, int* smem_dynamic_max);
// [rows][64][2][2] table blocks -> [64][rows] (cos, sin) pairs in `out` (rows*512 bytes).
cudaError_t launch_rope_pairs(const float* table, void* out, int rows, cudaStream_t stream);

// W8 (bits 8) / W4 (bits 4) codes + fp16 scale/zero per row and 64 columns ->
// fp16 [rows][out_stride] (dequant_sm100.cu).
cudaError_t launch_dequant(int bits, const void* packed, const void* scale, const void* zero, void* out,
                           int rows, int k, int64_t packed_stride, int64_t out_stride, int sms,
                           cudaStream_t stream);

}  // namespace ax
