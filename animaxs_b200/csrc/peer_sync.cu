// peer_sync.cu -- the cross-GPU handshake of the fused head-sharded path
// (animaxs_attn_forward_head_sharded_peer in sharded.cu).
//
// One block: thread 0 adds `add` to each peer's word for this rank (a release
// at system scope, so everything this GPU wrote before, in stream order, is
// visible to a peer that acquires the word), then thread i (< world, != rank)
// waits with acquire loads until this rank's word i reaches `target`.  The
// words only grow; "reached" is a wrap-safe signed difference.  Every wait is
// bounded by `timeout_ns` of %globaltimer, after which the status word gets
// the timeout bit and the kernel returns: a peer that never arrives cannot
// hang this GPU.  When every wait succeeded it writes the call's "go" value,
// without which the attention kernel that follows stores nothing into a peer.
#include <cuda_runtime.h>

#include "kernels.h"
#include "sm100_ptx.cuh"

namespace ax {
namespace {

__global__ void __launch_bounds__(32) peer_sync_kernel(const PeerSyncParams p) {
  const int i = static_cast<int>(threadIdx.x);
  if (i == 0 && p.add != 0) {
    __threadfence_system();
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank && p.signal[r] != nullptr) red_add_release_sys(p.signal[r], p.add);
  }
  bool ok = true;
  if (i < p.world && i != p.rank) {
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int>(ld_acquire_sys(p.wait + i) - p.target) < 0) {
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        atomicOr(p.status, kStatusTimeoutBit);
        ok = false;
        break;
      }
      __nanosleep(200);
    }
  }
  // Only a handshake that every peer completed lets the next kernel in the
  // stream write into the peers (it compares the word with this call's value).
  if (__all_sync(0xffffffffu, ok) && i == 0 && p.go != nullptr) *p.go = p.go_value;
  __syncwarp();
}

}  // namespace

cudaError_t launch_peer_sync(const PeerSyncParams& p, cudaStream_t stream) {
  peer_sync_kernel<<<1, 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ax
