// peer_sharded.cu -- heads sharded across the GPUs of one node with the
// all-gather fused into the attention kernel (include/animaxs_attn.h,
// animaxs_peer_group_* and animaxs_attn_forward_head_sharded_peer).
//
// The reference is a single-device app and has no counterpart; this serves
// the 16K-token DiT configuration without NCCL.  Every rank owns one output
// buffer, allocated here so that it is a whole cudaMalloc allocation and
// exportable through CUDA IPC; each rank maps every other rank's buffer.  A
// call on rank r:
//   1. peer_sync: add 1 to every peer's "ready" word for r, wait until every
//      peer's "ready" word here reached the call number (each peer has
//      reached this call in its stream, so it is done with the previous
//      output), bounded; only if every peer was ready, write the call number
//      to this rank's "go" word;
//   2. the attention kernel for heads [r*H/W, (r+1)*H/W): its epilogue stores
//      each output tile locally (TMA) and, if the "go" word holds this call's
//      number, at the same offset in every peer's buffer (NVLink stores), and
//      every CTA then adds its item count to every peer's "arrive" word for r
//      (release, system scope);
//   3. peer_sync: wait until every peer's "arrive" word here reached
//      call number x items per rank, bounded.
// After step 3 the local buffer holds every rank's heads.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "api_internal.h"
#include "kernels.h"

#ifndef ANIMAXS_WAIT_TIMEOUT_NS
#define ANIMAXS_WAIT_TIMEOUT_NS 2000000000ull  // 2 s, as the kernels' own waits
#endif

namespace {

constexpr int kMaxWorld = 8;
constexpr int64_t kFlagBytes = 256;  // ready [0, 8), arrive [8, 16), go [16] (uint32)
constexpr int kReady = 0;
constexpr int kArrive = 8;
constexpr int kGo = 16;  // written by this rank's ready handshake only

}  // namespace

struct animaxs_peer_group {
  animaxs_attn_ctx* ctx = nullptr;
  int world = 0, rank = 0, device = 0;
  int64_t out_bytes = 0;     // usable output bytes
  int64_t flags_off = 0;     // flags follow the output (256-byte aligned)
  char* local = nullptr;     // this rank's allocation
  char* base[kMaxWorld] = {};  // every rank's allocation as mapped here ([rank] = local)
  bool connected = false;
  unsigned int calls = 0;
};

namespace {

// cuMemGetAddressRange through the runtime's driver entry point (no link-time
// libcuda dependency): the size of the allocation a (mapped) pointer lies in.
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

unsigned int* flags_of(const animaxs_peer_group* g, int r) {
  return reinterpret_cast<unsigned int*>(g->base[r] + g->flags_off);
}

struct DeviceGuard {
  int prev = 0, dev = 0;
  explicit DeviceGuard(int d) : dev(d) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev != dev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int animaxs_peer_group_create(animaxs_attn_ctx* ctx, int world, int rank, int64_t output_bytes,
                                         animaxs_peer_group** out, void* ipc_handle64) {
  if (ctx == nullptr || out == nullptr || ipc_handle64 == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *out = nullptr;
  if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "peer group needs 2 <= world <= 8 and 0 <= rank < world");
  if (output_bytes <= 0 || output_bytes >= (int64_t{1} << 40))
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "invalid peer output size");
  DeviceGuard guard(ctx->device);
  auto* g = new animaxs_peer_group;
  g->ctx = ctx;
  g->world = world;
  g->rank = rank;
  g->device = ctx->device;
  g->out_bytes = output_bytes;
  g->flags_off = (output_bytes + 255) / 256 * 256;
  void* mem = nullptr;
  cudaError_t e = cudaMalloc(&mem, static_cast<size_t>(g->flags_off + kFlagBytes));
  if (e == cudaSuccess) e = cudaMemset(mem, 0, static_cast<size_t>(g->flags_off + kFlagBytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can signal
  cudaIpcMemHandle_t h{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, mem);
  if (e != cudaSuccess) {
    if (mem) cudaFree(mem);
    delete g;
    return ax_cuda_fail(ctx, e, "peer buffer");
  }
  g->local = static_cast<char*>(mem);
  g->base[rank] = g->local;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  std::memcpy(ipc_handle64, &h, 64);
  *out = g;
  return ANIMAXS_OK;
}

extern "C" int animaxs_peer_group_connect(animaxs_peer_group* g, const void* handles64) {
  if (g == nullptr || handles64 == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  if (g->connected) return ax_set_error(g->ctx, ANIMAXS_ERR_INVALID_ARG, "peer group already connected");
  DeviceGuard guard(g->device);
  AddressRangeFn range = address_range_fn();
  if (range == nullptr)
    return ax_set_error(g->ctx, ANIMAXS_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
  const auto* hs = static_cast<const unsigned char*>(handles64);
  auto unmap = [&]() {
    for (int q = 0; q < g->world; ++q)
      if (q != g->rank && g->base[q] != nullptr) {
        cudaIpcCloseMemHandle(g->base[q]);
        g->base[q] = nullptr;
      }
  };
  const size_t want = static_cast<size_t>(g->flags_off + kFlagBytes);
  for (int r = 0; r < g->world; ++r) {
    if (r == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + 64 * r, 64);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      unmap();
      return ax_cuda_fail(g->ctx, e, "mapping a peer's output (cudaIpcOpenMemHandle)");
    }
    g->base[r] = static_cast<char*>(p);
    // Every rank's buffer must have this rank's layout: the kernels store
    // into a peer at this rank's offsets.
    CUdeviceptr b = 0;
    size_t size = 0;
    if (range(&b, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS ||
        b != reinterpret_cast<CUdeviceptr>(p) || size < want) {
      unmap();
      return ax_set_error(g->ctx, ANIMAXS_ERR_INVALID_ARG,
                          "rank %d's peer buffer is not %zu bytes like this rank's (all ranks must pass the same "
                          "output_bytes)",
                          r, want);
    }
  }
  g->connected = true;
  return ANIMAXS_OK;
}

extern "C" void* animaxs_peer_group_output(animaxs_peer_group* g) { return g ? g->local : nullptr; }

extern "C" int animaxs_peer_group_destroy(animaxs_peer_group* g) {
  if (g == nullptr) return ANIMAXS_OK;
  {
    DeviceGuard guard(g->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < g->world; ++r)
      if (r != g->rank && g->base[r] != nullptr) cudaIpcCloseMemHandle(g->base[r]);
    if (g->local) cudaFree(g->local);
  }
  delete g;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_forward_head_sharded_peer(animaxs_attn_ctx* ctx, animaxs_peer_group* g,
                                                      const animaxs_attn_desc* d, const void* q, const void* k,
                                                      const void* v, void* o, void* stream_) {
  AxRange range("animaxs_attn_forward_head_sharded_peer");
  if (ctx == nullptr || g == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int rc = ax_validate(ctx, d, q, k, v, o);
  if (rc != ANIMAXS_OK) return rc;
  if (!g->connected) return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "peer group is not connected");
  if (g->ctx != ctx || g->device != ctx->device)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "peer group belongs to another context");
  if (o != g->local)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "o must be the peer group's output buffer");
  const int world = g->world, rank = g->rank;
  if (d->heads % world != 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "heads (%d) must be a multiple of world (%d)", d->heads,
                        world);
  if (d->head_dim != 64 && d->head_dim != 128)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "head-sharded attention requires headDim 128 or 64 (got %d)", d->head_dim);
  // The output view must lie inside the buffer every rank mapped.
  const int64_t last = (static_cast<int64_t>(d->batch) - 1) * d->o_batch_stride +
                       (static_cast<int64_t>(d->heads) - 1) * d->o_head_stride +
                       (static_cast<int64_t>(d->q_len) - 1) * d->o_tok_stride + d->head_dim;
  if (d->o_batch_stride < 0 || d->o_head_stride < 0 || d->o_tok_stride < 0 || last * 2 > g->out_bytes)
    return ax_set_error(ctx, ANIMAXS_ERR_OOB, "output view exceeds the peer group's %lld-byte buffer",
                        static_cast<long long>(g->out_bytes));
  const int hr = d->heads / world;
  const int h0 = rank * hr;
  const unsigned int items =
      static_cast<unsigned int>(ax::attn_fwd_work_items(d->q_len, hr, d->batch, ctx->num_sms, true));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceGuard guard(ctx->device);

  const unsigned int call = ++g->calls;
  ax::PeerSyncParams ready{};
  for (int r = 0; r < world; ++r)
    ready.signal[r] = r == rank ? nullptr : flags_of(g, r) + kReady + rank;
  ready.add = 1;
  ready.wait = flags_of(g, rank) + kReady;
  ready.target = call;
  ready.world = world;
  ready.rank = rank;
  ready.timeout_ns = ANIMAXS_WAIT_TIMEOUT_NS;
  ready.status = ctx->d_status;
  ready.go = flags_of(g, rank) + kGo;
  ready.go_value = call;
  cudaError_t e = ax::launch_peer_sync(ready, stream);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "peer handshake launch");

  AxPeers peers{};
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    peers.delta[peers.n] = static_cast<long long>(g->base[r] - g->local);
    peers.arrive[peers.n] = flags_of(g, r) + kArrive + rank;
    ++peers.n;
  }
  // A peer that was not ready (the handshake gave up) may still be reading its
  // previous output: then the kernel stores nothing into any peer and adds no
  // arrivals, so the peers' closing waits report the failure too.
  peers.go = flags_of(g, rank) + kGo;
  peers.go_value = call;
  rc = ax_forward_range(ctx, d, q, k, v, o, h0, hr, nullptr, stream, &peers);
  if (rc != ANIMAXS_OK) return rc;

  ax::PeerSyncParams arrive{};
  arrive.add = 0;
  arrive.wait = flags_of(g, rank) + kArrive;
  arrive.target = call * items;  // words only grow; compared wrap-safe
  arrive.world = world;
  arrive.rank = rank;
  arrive.timeout_ns = ANIMAXS_WAIT_TIMEOUT_NS;
  arrive.status = ctx->d_status;
  e = ax::launch_peer_sync(arrive, stream);
  if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "peer handshake launch");
  ctx->last_error.clear();
  return ANIMAXS_OK;
}
