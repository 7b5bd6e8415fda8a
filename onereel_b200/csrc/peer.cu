// Device-side barrier over peer memory, for the K/V exchange that reads other GPUs' buffers directly.
//
// The reference moves K/V between ranks with NCCL send/recv (src/onereel/parallel/comm.py:126-201 HaloExchange).
// Here every rank keeps its own K/V rows in a symmetric buffer (mapped into every peer's address space over NVLink)
// and the ranks that need them pull them with the pack kernel (TMA bulk loads from the peer's memory, no multicast).
// Before a pull, the owner's rows must have landed: orl_peer_barrier is that synchronisation. Each rank has a signal
// pad of `world` ints in symmetric memory; a call with epoch e writes e into slot `rank` of every rank's pad (a system-
// scope release store over NVLink), then waits until every slot of its own pad holds at least e (acquire loads).
// Epochs only grow, so pads never need resetting. The wait is bounded: after timeout_ns it ORs kErrPeerTimeout into
// err_dev and returns (a rank that left or never arrived ends the step with an error, not a hang).
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"
#include "ptx.cuh"

namespace orl {

constexpr int kMaxPeers = 16;

struct PeerPads {
  int* pad[kMaxPeers];   // pad[p]: rank p's signal pad (peer addresses, valid in this process)
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(PeerPads pads, int world, int rank, int epoch,
                                                          unsigned long long timeout_ns, int* err) {
  const int p = threadIdx.x;
  if (p < world) st_release_sys(pads.pad[p] + rank, epoch);
  __syncwarp();
  if (p < world) {
    const int* mine = pads.pad[rank] + p;
    const unsigned long long t0 = global_ns();
    // wrap-safe: epochs compared by their difference in two's complement
    while (static_cast<int>(static_cast<unsigned>(ld_acquire_sys(mine)) - static_cast<unsigned>(epoch)) < 0) {
      if (global_ns() - t0 > timeout_ns) {
        atomicOr(err, kErrPeerTimeout);
        break;
      }
    }
  }
}

}  // namespace orl

using namespace orl;

extern "C" int orl_peer_barrier(int* const* pads, int world, int rank, int epoch, unsigned long long timeout_ns,
                                int* err_dev, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (pads == nullptr || err_dev == nullptr || world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return ORL_ERR_ARG;
  if (timeout_ns == 0 || timeout_ns > kWaitLimitNs * 10) return ORL_ERR_ARG;
  PeerPads pp{};
  for (int p = 0; p < world; ++p) {
    if (pads[p] == nullptr || (reinterpret_cast<uintptr_t>(pads[p]) & 3u)) return ORL_ERR_ARG;
    pp.pad[p] = pads[p];
  }
  peer_barrier_kernel<<<1, 32, 0, stream>>>(pp, world, rank, epoch, timeout_ns, err_dev);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
