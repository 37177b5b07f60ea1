// call_bench.cu -- what one animaxs_attn_forward call costs without Python.
//
// Built by build.py as animaxs_b200/_build/call_bench (linked against
// libanimaxs_attn.so) and run by bench.py for its small-configuration figures.
// For each shape it enqueues `reps` calls through the C ABI on one stream and
// reports, per call:
//   host_us   - host time to enqueue the call (std::chrono around the loop),
//   eager_us  - device time of the eagerly enqueued loop (CUDA events), which
//               includes any gap the host leaves between launches,
//   graph_us  - device time of the same calls replayed from a CUDA graph,
//               i.e. the kernels back to back.
// Inputs are cudaMalloc'd and filled with small values, and the RoPE table is
// a 1-D table of the right size; the timing does not depend on either.
// Prints one JSON object.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../include/animaxs_attn.h"

namespace {

__global__ void fill_kernel(__half* p, size_t n, unsigned seed) {
  for (size_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    unsigned h = static_cast<unsigned>(i) * 2654435761u ^ seed;
    h ^= h >> 13;
    p[i] = __float2half(static_cast<float>(h & 0xFFFF) / 65536.0f - 0.5f);
  }
}

struct Shape {
  const char* name;
  int batch, heads, kv_heads, q_len, kv_len, causal, kv_valid, qk_norm, rope_rows, layers;
};

#define CHECK(x)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (x);                                                                 \
    if (e_ != cudaSuccess) {                                                              \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                       \
      std::exit(2);                                                                       \
    }                                                                                     \
  } while (0)

}  // namespace

int main(int argc, char** argv) {
  const int reps = argc > 1 ? std::atoi(argv[1]) : 200;
  // Configurations 1, 2 (masked), 3 (one layer; `layers` consecutive calls,
  // each with its own q/k/v, make the 28-layer prefill) of the workload.
  const Shape shapes[] = {
      {"config1_dit_self_1024", 1, 16, 16, 1024, 1024, 0, 0, ANIMAXS_QK_RMS_ROPE, 1024, 1},
      {"config2_dit_cross_4096x512", 1, 16, 16, 4096, 512, 0, 128, ANIMAXS_QK_RMS, 0, 1},
      {"config3_qwen_layer", 1, 16, 8, 512, 512, 1, 300, ANIMAXS_QK_RMS_ROPE, 512, 28},
  };
  animaxs_attn_ctx* ctx = nullptr;
  if (animaxs_attn_create(0, &ctx) != ANIMAXS_OK) {
    std::fprintf(stderr, "no sm_100 device\n");
    return 2;
  }
  cudaStream_t s;
  CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  std::printf("{\"reps\": %d", reps);
  for (const Shape& sh : shapes) {
    const size_t nq = static_cast<size_t>(sh.batch) * sh.q_len * sh.heads * 128;
    const size_t nk = static_cast<size_t>(sh.batch) * sh.kv_len * sh.kv_heads * 128;
    std::vector<__half*> q(sh.layers), k(sh.layers), v(sh.layers);
    __half* o = nullptr;
    float* rope = nullptr;
    for (int l = 0; l < sh.layers; ++l) {
      CHECK(cudaMalloc(&q[l], nq * 2));
      CHECK(cudaMalloc(&k[l], nk * 2));
      CHECK(cudaMalloc(&v[l], nk * 2));
      fill_kernel<<<256, 256, 0, s>>>(q[l], nq, 1u + 3 * l);
      fill_kernel<<<256, 256, 0, s>>>(k[l], nk, 2u + 3 * l);
      fill_kernel<<<256, 256, 0, s>>>(v[l], nk, 3u + 3 * l);
    }
    CHECK(cudaMalloc(&o, nq * 2));
    if (sh.rope_rows > 0) {
      std::vector<float> host(static_cast<size_t>(sh.rope_rows) * 256);
      animaxs_rope1d_table(sh.rope_rows, 128, 1.0e6, host.data());
      CHECK(cudaMalloc(&rope, host.size() * 4));
      CHECK(cudaMemcpy(rope, host.data(), host.size() * 4, cudaMemcpyHostToDevice));
    }
    animaxs_attn_desc d;
    animaxs_attn_desc_init(&d, sh.batch, sh.heads, sh.kv_heads, sh.q_len, sh.kv_len, 128);
    d.causal = sh.causal;
    d.kv_valid_len = sh.kv_valid;
    d.qk_norm = sh.qk_norm;
    d.rope_table = rope;
    d.rope_rows = sh.rope_rows;
    auto one = [&](int i) {
      const int l = i % sh.layers;
      const int rc = animaxs_attn_forward(ctx, &d, q[l], k[l], v[l], o, s);
      if (rc != ANIMAXS_OK) {
        std::fprintf(stderr, "%s: %s\n", sh.name, animaxs_attn_last_error(ctx));
        std::exit(3);
      }
    };
    for (int i = 0; i < 20; ++i) one(i);
    CHECK(cudaStreamSynchronize(s));
    cudaEvent_t e0, e1;
    CHECK(cudaEventCreate(&e0));
    CHECK(cudaEventCreate(&e1));
    CHECK(cudaEventRecord(e0, s));
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < reps; ++i) one(i);
    const auto t1 = std::chrono::steady_clock::now();
    CHECK(cudaEventRecord(e1, s));
    CHECK(cudaEventSynchronize(e1));
    float eager_ms = 0.f;
    CHECK(cudaEventElapsedTime(&eager_ms, e0, e1));
    const double host_us = std::chrono::duration<double, std::micro>(t1 - t0).count() / reps;
    // The same calls captured once and replayed.
    cudaGraph_t g;
    cudaGraphExec_t ge;
    CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    for (int i = 0; i < reps; ++i) one(i);
    CHECK(cudaStreamEndCapture(s, &g));
    CHECK(cudaGraphInstantiate(&ge, g, 0));
    CHECK(cudaGraphLaunch(ge, s));
    CHECK(cudaStreamSynchronize(s));
    float graph_ms = 1e30f;
    for (int r = 0; r < 3; ++r) {
      CHECK(cudaEventRecord(e0, s));
      CHECK(cudaGraphLaunch(ge, s));
      CHECK(cudaEventRecord(e1, s));
      CHECK(cudaEventSynchronize(e1));
      float ms = 0.f;
      CHECK(cudaEventElapsedTime(&ms, e0, e1));
      graph_ms = std::fmin(graph_ms, ms);
    }
    std::printf(", \"%s\": {\"host_us\": %.3f, \"eager_us\": %.3f, \"graph_us\": %.3f, \"calls_per_item\": %d}",
                sh.name, host_us, eager_ms * 1e3 / reps, graph_ms * 1e3 / reps, sh.layers);
    CHECK(cudaGraphExecDestroy(ge));
    CHECK(cudaGraphDestroy(g));
    CHECK(cudaEventDestroy(e0));
    CHECK(cudaEventDestroy(e1));
    for (int l = 0; l < sh.layers; ++l) {
      cudaFree(q[l]);
      cudaFree(k[l]);
      cudaFree(v[l]);
    }
    cudaFree(o);
    if (rope) cudaFree(rope);
  }
  std::printf("}\n");
  CHECK(cudaStreamDestroy(s));
  animaxs_attn_destroy(ctx);
  return 0;
}
