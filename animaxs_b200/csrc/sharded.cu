// sharded.cu -- heads sharded across the GPUs of one node + one NCCL all-gather.
//
// The reference is a single-device app and has no counterpart; this serves the
// 16K-token DiT configuration: rank r computes query heads
// [r*H/W, (r+1)*H/W) for every query row (each rank holds the full K/V of its
// heads), and one ncclAllGather over NVLink assembles the output on every rank.
//
// NCCL is dlopen()ed (libnccl.so.2) so the library has no link-time NCCL
// dependency and uses whichever NCCL the host process already loaded (e.g.
// PyTorch's).  Communicators are created non-blocking and every NCCL wait is
// bounded by a wall-clock deadline, after which the communicator is aborted and
// ANIMAXS_ERR_TIMEOUT is returned (a rank that never joins cannot hang a caller).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "api_internal.h"
#include "kernels.h"

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char* n : names) {
      api.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
      if (api.handle) break;
    }
    if (!api.handle) return;
#define AX_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(api.handle, name))
    AX_SYM(getUniqueId, "ncclGetUniqueId");
    AX_SYM(commInitRankConfig, "ncclCommInitRankConfig");
    AX_SYM(allGather, "ncclAllGather");
    AX_SYM(commDestroy, "ncclCommDestroy");
    AX_SYM(commAbort, "ncclCommAbort");
    AX_SYM(commGetAsyncError, "ncclCommGetAsyncError");
    AX_SYM(getErrorString, "ncclGetErrorString");
#undef AX_SYM
    api.ok = api.getUniqueId && api.commInitRankConfig && api.allGather && api.commDestroy &&
             api.commAbort && api.commGetAsyncError && api.getErrorString;
  });
  return api.ok ? &api : nullptr;
}

double timeout_seconds() {
  const char* s = std::getenv("ANIMAXS_NCCL_TIMEOUT_S");
  const double v = s ? std::atof(s) : 0.0;
  return v > 0 ? v : 120.0;
}

// Poll a non-blocking communicator until its pending operation settles.
ncclResult_t settle(NcclApi* api, ncclComm_t comm, double seconds) {
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::duration_cast<std::chrono::steady_clock::duration>(
                            std::chrono::duration<double>(seconds));
  ncclResult_t st = ncclInProgress;
  while (true) {
    if (api->commGetAsyncError(comm, &st) != ncclSuccess) return ncclSystemError;
    if (st != ncclInProgress) return st;
    if (std::chrono::steady_clock::now() > deadline) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// gather[r][b][s][hl][D] -> o[b*ob + s*ot + (r*hr + hl)*oh], 16 B per thread;
// a head row is D/8 = 1 << chunk_shift chunks of 16 B.
__global__ void permute_heads_kernel(const uint4* __restrict__ gather, __half* __restrict__ o,
                                     long long total16, int world, int batch, int q_len, int hr,
                                     long long ot, long long oh, long long ob, int chunk_shift) {
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total16) return;
  const int c16 = static_cast<int>(i & ((1 << chunk_shift) - 1));
  long long r = i >> chunk_shift;
  const int hl = static_cast<int>(r % hr);
  r /= hr;
  const int s = static_cast<int>(r % q_len);
  r /= q_len;
  const int b = static_cast<int>(r % batch);
  const int rank = static_cast<int>(r / batch);
  __half* dst = o + static_cast<long long>(b) * ob + static_cast<long long>(s) * ot +
                static_cast<long long>(rank * hr + hl) * oh + c16 * 8;
  *reinterpret_cast<uint4*>(dst) = gather[i];
}

}  // namespace

struct animaxs_comm {
  ncclComm_t comm = nullptr;
  int world = 1;
  int rank = 0;
  int device = 0;
};

extern "C" int animaxs_comm_unique_id(void* id128) {
  if (id128 == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  NcclApi* api = nccl();
  if (api == nullptr) return ANIMAXS_ERR_NCCL;
  ncclUniqueId id;
  if (api->getUniqueId(&id) != ncclSuccess) return ANIMAXS_ERR_NCCL;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id128, &id, sizeof(id));
  return ANIMAXS_OK;
}

extern "C" int animaxs_comm_create(animaxs_attn_ctx* ctx, int world, int rank, const void* id128,
                                   animaxs_comm** out) {
  if (ctx == nullptr || out == nullptr || id128 == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "invalid world %d / rank %d", world, rank);
  NcclApi* api = nccl();
  if (api == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_NCCL, "libnccl.so.2 not loadable");
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof(id));
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = api->commInitRankConfig(&comm, world, id, rank, &cfg);
  if (r == ncclInProgress || r == ncclSuccess) r = settle(api, comm, timeout_seconds());
  cudaSetDevice(prev);
  if (r != ncclSuccess) {
    if (comm) api->commAbort(comm);
    if (r == ncclInProgress)
      return ax_set_error(ctx, ANIMAXS_ERR_TIMEOUT, "NCCL communicator init timed out");
    return ax_set_error(ctx, ANIMAXS_ERR_NCCL, "NCCL init failed: %s", api->getErrorString(r));
  }
  auto* c = new animaxs_comm();
  c->comm = comm;
  c->world = world;
  c->rank = rank;
  c->device = ctx->device;
  *out = c;
  return ANIMAXS_OK;
}

extern "C" int animaxs_comm_destroy(animaxs_comm* c) {
  if (c == nullptr) return ANIMAXS_OK;
  NcclApi* api = nccl();
  if (api && c->comm) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    ncclResult_t r = api->commDestroy(c->comm);
    if (r == ncclInProgress) r = settle(api, c->comm, timeout_seconds());
    if (r != ncclSuccess) api->commAbort(c->comm);
    cudaSetDevice(prev);
  }
  delete c;
  return ANIMAXS_OK;
}

extern "C" int animaxs_attn_forward_head_sharded(animaxs_attn_ctx* ctx, animaxs_comm* comm,
                                                 const animaxs_attn_desc* d, const void* q,
                                                 const void* k, const void* v, void* o,
                                                 void* stream_) {
  AxRange range("animaxs_attn_forward_head_sharded");
  if (ctx == nullptr || comm == nullptr) return ANIMAXS_ERR_INVALID_ARG;
  int rc = ax_validate(ctx, d, q, k, v, o);
  if (rc != ANIMAXS_OK) return rc;
  if (comm->device != ctx->device)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "communicator is on another device");
  const int world = comm->world, rank = comm->rank;
  if (d->heads % world != 0)
    return ax_set_error(ctx, ANIMAXS_ERR_INVALID_ARG, "heads (%d) must be a multiple of world (%d)",
                        d->heads, world);
  if (d->head_dim != 64 && d->head_dim != 128)
    return ax_set_error(ctx, ANIMAXS_ERR_UNSUPPORTED,
                        "head-sharded attention requires headDim 128 or 64 (got %d)", d->head_dim);
  const int hr = d->heads / world;  // every rank reads the full K/V, so any GQA grouping works
  NcclApi* api = nccl();
  if (api == nullptr) return ax_set_error(ctx, ANIMAXS_ERR_NCCL, "libnccl.so.2 not loadable");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int h0 = rank * hr;
  const int64_t D = d->head_dim;
  const size_t slice = static_cast<size_t>(d->batch) * d->q_len * hr * D;  // elements

  const bool in_place = d->batch == 1 && d->o_tok_stride == D && d->o_head_stride == d->q_len * D;
  __half* gather = nullptr;
  AxOutView view{};
  if (in_place) {
    // Head-major output: every rank's heads are one contiguous slice of o.
    view = AxOutView{o, d->o_tok_stride, d->o_head_stride, d->o_batch_stride, 0};
  } else {
    const size_t need = slice * world * sizeof(__half);
    if (need > ctx->staging_bytes) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(ctx->device);
      if (ctx->staging) {
        cudaDeviceSynchronize();
        cudaFree(ctx->staging);
        ctx->staging = nullptr;
        ctx->staging_bytes = 0;
      }
      cudaError_t e = cudaMalloc(&ctx->staging, need);
      cudaSetDevice(prev);
      if (e != cudaSuccess) return ax_cuda_fail(ctx, e, "staging allocation");
      ctx->staging_bytes = need;
    }
    gather = static_cast<__half*>(ctx->staging);
    view = AxOutView{gather + rank * slice, hr * D, D, static_cast<int64_t>(d->q_len) * hr * D, h0};
  }
  rc = ax_forward_range(ctx, d, q, k, v, o, h0, hr, &view, stream);
  if (rc != ANIMAXS_OK) return rc;

  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  const void* send = in_place ? static_cast<const void*>(static_cast<__half*>(o) + h0 * d->q_len * D)
                              : static_cast<const void*>(gather + rank * slice);
  void* recv = in_place ? o : static_cast<void*>(gather);
  ncclResult_t r = api->allGather(send, recv, slice, ncclFloat16, comm->comm, stream);
  if (r == ncclInProgress) r = settle(api, comm->comm, timeout_seconds());
  if (r != ncclSuccess) {
    cudaSetDevice(prev);
    if (r == ncclInProgress) {
      api->commAbort(comm->comm);
      comm->comm = nullptr;
      return ax_set_error(ctx, ANIMAXS_ERR_TIMEOUT, "NCCL all-gather enqueue timed out");
    }
    return ax_set_error(ctx, ANIMAXS_ERR_NCCL, "ncclAllGather: %s", api->getErrorString(r));
  }
  if (!in_place) {
    const long long total16 = static_cast<long long>(slice) * world / 8;
    const unsigned blocks = static_cast<unsigned>((total16 + 255) / 256);
    permute_heads_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(gather),
                                                     static_cast<__half*>(o), total16, world,
                                                     d->batch, d->q_len, hr, d->o_tok_stride,
                                                     d->o_head_stride, d->o_batch_stride,
                                                     D == 64 ? 3 : 4);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      cudaSetDevice(prev);
      return ax_cuda_fail(ctx, e, "permute launch");
    }
  }
  cudaSetDevice(prev);
  ctx->last_error.clear();
  return ANIMAXS_OK;
}
