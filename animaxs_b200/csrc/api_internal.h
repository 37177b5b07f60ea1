// api_internal.h -- context layout and helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/animaxs_attn.h"
#include <nvtx3/nvToolsExt.h>

// NVTX range around a C ABI call (header-only NVTX v3: a no-op unless a
// profiler injects itself), so a capture can attribute kernels to the call.
struct AxRange {
  explicit AxRange(const char* name) { nvtxRangePushA(name); }
  ~AxRange() { nvtxRangePop(); }
  AxRange(const AxRange&) = delete;
  AxRange& operator=(const AxRange&) = delete;
};

struct animaxs_attn_ctx {
  int device = 0;
  int num_sms = 0;
  void* scratch = nullptr;        // normalised q/k copies (grown on demand)
  size_t scratch_bytes = 0;
  void* staging = nullptr;        // head-sharded path: per-rank slice + gather buffer
  size_t staging_bytes = 0;
  unsigned int* d_status = nullptr;  // device status word written by kernels
  int64_t query_tiles = 0;
  bool timing = false;                        // bracket each attention kernel with events
  unsigned int* score_probe = nullptr;        // device uint32[4] probe slot, or nullptr
  std::vector<cudaEvent_t> events;            // pool: pairs (start, stop)
  size_t events_used = 0;                     // events recorded since the last read
  std::string last_error;
};

// Output redirection for the head-sharded path: query head h is written at
// ptr + (h - head_base) * head.
struct AxOutView {
  void* ptr;
  int64_t tok, head, batch;
  int head_base;
};

int ax_set_error(animaxs_attn_ctx* ctx, int code, const char* fmt, ...);
int ax_cuda_fail(animaxs_attn_ctx* ctx, cudaError_t e, const char* what);
int ax_ensure_scratch(animaxs_attn_ctx* ctx, size_t bytes);  // context scratch of at least `bytes`
int ax_validate(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d, const void* q, const void* k,
                const void* v, const void* o);
int ax_make_tmap(animaxs_attn_ctx* ctx, CUtensorMap* map, const void* base, int64_t dim, int64_t rows,
                 int64_t heads, int64_t batch, int64_t st, int64_t sh, int64_t sb, int box_rows = 128);
// Peers of a fused head-sharded call: the epilogue stores every output tile
// also at o + delta[i] and the CTAs count their items on arrive[i].
struct AxPeers {
  int n;
  long long delta[7];
  unsigned int* arrive[7];
  const unsigned int* go;  // the stores and arrivals happen only if *go == go_value
  unsigned int go_value;
};
int ax_forward_range(animaxs_attn_ctx* ctx, const animaxs_attn_desc* d, const void* q,
                     const void* k, const void* v, void* o, int heads_begin, int heads_count,
                     const AxOutView* o_view, cudaStream_t stream, const AxPeers* peers = nullptr);
