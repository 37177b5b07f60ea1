// weight_streamer.cu -- bounded device memory for weights streamed from host
// memory (C ABI in include/animaxs_attn.h).
//
// Replaces the reference's WeightStreamer (AnimaXS/Runtime/Metal/
// WeightStreamer.swift:84-213): 1 to 4 device slots of `capacity` bytes; a
// load copies one execution range of a weight pack (host memory, e.g. the
// mapped .animapk file) into a slot, and a slot that queued work still reads
// is never overwritten.  The reference copies with the CPU (memcpy into a
// shared buffer) and ping-pongs two slots so that block n+1's copy overlaps
// block n's command buffer (DiTBlockExecutor.swift:222-260); it refuses a load
// into a slot whose command buffer is still in flight (markInFlight /
// complete).
//
// B200 form:
//  - a load is an asynchronous host-to-device copy on the caller's stream (a
//    copy stream, so that it overlaps the kernels of the previous block); host
//    memory that is pinned or registered (animaxs_weight_streamer_register_host,
//    cudaHostRegister of the pack mapping) moves by DMA at PCIe speed;
//  - after a load the streamer records an event; a consumer stream waits for
//    it on the GPU (animaxs_weight_streamer_wait_loaded), not on the host;
//  - mark_in_flight records an event on the consumer stream; a later load into
//    that slot makes its copy stream wait for the event on the GPU, so the slot
//    is never overwritten while that work may read it, and the host never
//    blocks.  complete clears the mark when the caller knows the work is done.
#include <cuda_runtime.h>

#include <mutex>
#include <new>

#include "../../include/animaxs_attn.h"
#include "api_internal.h"

namespace {

constexpr int kMaxSlots = 4;

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

struct animaxs_weight_streamer {
  animaxs_attn_ctx* ctx = nullptr;
  int64_t capacity = 0, stride = 0;
  int slots = 0;
  char* mem = nullptr;
  cudaEvent_t loaded[kMaxSlots] = {};
  cudaEvent_t in_flight_ev[kMaxSlots] = {};
  bool in_flight[kMaxSlots] = {};
  bool has_load[kMaxSlots] = {};
  int64_t logical[kMaxSlots] = {-1, -1, -1, -1};
  void* registered[8] = {};
  int n_registered = 0;
  std::mutex mu;
};

namespace {

int slot_check(animaxs_weight_streamer* w, int slot) {
  if (w == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (slot < 0 || slot >= w->slots)
    return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "weight slot %d out of range", slot);
  return ANIMAXS_OK;
}

}  // namespace

extern "C" int animaxs_weight_streamer_create(animaxs_attn_ctx* ctx, int64_t capacity, int slots,
                                              animaxs_weight_streamer** out) {
  if (ctx == nullptr || out == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *out = nullptr;
  if (capacity <= 0) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "weight ring capacity must be positive");
  if (slots <= 0 || slots > kMaxSlots)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "weight slot count must be in 1...4");
  auto* w = new (std::nothrow) animaxs_weight_streamer();
  if (w == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_CUDA, "host allocation failed");
  w->ctx = ctx;
  w->capacity = capacity;
  w->stride = (capacity + 255) / 256 * 256;  // every slot 256-byte aligned
  w->slots = slots;
  DeviceScope scope(ctx->device);
  cudaError_t e = cudaMalloc(&w->mem, static_cast<size_t>(w->stride * slots));
  for (int s = 0; e == cudaSuccess && s < slots; ++s) {
    e = cudaEventCreateWithFlags(&w->loaded[s], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w->in_flight_ev[s], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    animaxs_weight_streamer_destroy(w);
    return ax_cuda_fail(ctx, e, "failed to allocate weight slot");
  }
  *out = w;
  ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_destroy(animaxs_weight_streamer* w) {
  if (w == nullptr) return ANIMAXS_OK;
  {
    DeviceScope scope(w->ctx->device);
    cudaDeviceSynchronize();  // queued copies and readers of the slots
    for (int s = 0; s < kMaxSlots; ++s) {
      if (w->loaded[s]) cudaEventDestroy(w->loaded[s]);
      if (w->in_flight_ev[s]) cudaEventDestroy(w->in_flight_ev[s]);
    }
    for (int i = 0; i < w->n_registered; ++i) cudaHostUnregister(w->registered[i]);
    if (w->mem) cudaFree(w->mem);
  }
  delete w;
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_register_host(animaxs_weight_streamer* w, void* base, int64_t bytes) {
  if (w == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (base == nullptr || bytes <= 0)
    return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "host range to register must be non-empty");
  std::lock_guard<std::mutex> lock(w->mu);
  if (w->n_registered == 8)
    return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "at most 8 host ranges can be registered");
  DeviceScope scope(w->ctx->device);
  const cudaError_t e = cudaHostRegister(base, static_cast<size_t>(bytes), cudaHostRegisterReadOnly);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return ax_cuda_fail(w->ctx, e, "host range registration");
  }
  w->registered[w->n_registered++] = base;
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_load(animaxs_weight_streamer* w, int slot, const void* src,
                                            int64_t bytes, int64_t logical_index, void* stream) {
  int rc = slot_check(w, slot);
  if (rc != ANIMAXS_OK) return rc;
  if (src == nullptr || bytes <= 0)
    return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "execution range has no mapped bytes");
  if (bytes > w->capacity)
    return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "execution range does not fit the weight slot");
  std::lock_guard<std::mutex> lock(w->mu);
  DeviceScope scope(w->ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (w->in_flight[slot]) {
    // The slot's readers were queued before this copy: order it after them.
    e = cudaStreamWaitEvent(s, w->in_flight_ev[slot], 0);
    w->in_flight[slot] = false;
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w->mem + slot * w->stride, src, static_cast<size_t>(bytes), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaEventRecord(w->loaded[slot], s);
  if (e != cudaSuccess) return ax_cuda_fail(w->ctx, e, "weight slot load");
  w->has_load[slot] = true;
  w->logical[slot] = logical_index;
  w->ctx->last_error.clear();
  return ANIMAXS_OK;
}

extern "C" void* animaxs_weight_streamer_slot(const animaxs_weight_streamer* w, int slot) {
  if (w == nullptr || slot < 0 || slot >= w->slots) return nullptr;
  return w->mem + slot * w->stride;
}

extern "C" int animaxs_weight_streamer_wait_loaded(animaxs_weight_streamer* w, int slot, void* consumer_stream) {
  int rc = slot_check(w, slot);
  if (rc != ANIMAXS_OK) return rc;
  std::lock_guard<std::mutex> lock(w->mu);
  if (!w->has_load[slot]) return ax_set_error(w->ctx, ANIMAXS_ERR_INVALID_ARG, "weight slot %d holds no range", slot);
  DeviceScope scope(w->ctx->device);
  const cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(consumer_stream), w->loaded[slot], 0);
  if (e != cudaSuccess) return ax_cuda_fail(w->ctx, e, "weight slot wait");
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_mark_in_flight(animaxs_weight_streamer* w, int slot, void* consumer_stream) {
  int rc = slot_check(w, slot);
  if (rc != ANIMAXS_OK) return rc;
  std::lock_guard<std::mutex> lock(w->mu);
  DeviceScope scope(w->ctx->device);
  const cudaError_t e = cudaEventRecord(w->in_flight_ev[slot], static_cast<cudaStream_t>(consumer_stream));
  if (e != cudaSuccess) return ax_cuda_fail(w->ctx, e, "weight slot in-flight mark");
  w->in_flight[slot] = true;
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_complete(animaxs_weight_streamer* w, int slot) {
  int rc = slot_check(w, slot);
  if (rc != ANIMAXS_OK) return rc;
  std::lock_guard<std::mutex> lock(w->mu);
  w->in_flight[slot] = false;
  return ANIMAXS_OK;
}

extern "C" int animaxs_weight_streamer_state(animaxs_weight_streamer* w, int slot, int64_t* logical_index,
                                             int* in_flight) {
  int rc = slot_check(w, slot);
  if (rc != ANIMAXS_OK) return rc;
  std::lock_guard<std::mutex> lock(w->mu);
  if (logical_index) *logical_index = w->logical[slot];
  if (in_flight) *in_flight = w->in_flight[slot] ? 1 : 0;
  return ANIMAXS_OK;
}
