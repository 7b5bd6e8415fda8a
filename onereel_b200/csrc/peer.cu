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
//
// orl_peer_gather is the all-to-all of the Ulysses path over the same peer mappings (the reference's a2a_heads /
// a2a_tokens, parallel/comm.py:276-295, are NCCL all_to_all_single calls around transposed copies): every rank pulls,
// from every peer p, `rows` row segments of seg_bytes (its heads of p's tokens, or its tokens of p's heads) straight
// into their final place — no transposed staging copy on either side.
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

constexpr int kGatherPlanes = 3;
constexpr int kGatherUnroll = 4;

struct GatherArgs {
  const uint8_t* src[kGatherPlanes][kMaxPeers];   // per plane, peer p's buffer
  uint8_t* dst[kGatherPlanes];
};

// vector g of plane `pl`: segment s = g / vps (peer p = s / rows, row i = s % rows), 16-byte vector v = g % vps;
// reads src[pl][p] + src_row0 + i * src_stride + 16 v, writes dst[pl] + p * dst_pstride + i * dst_stride + 16 v
__global__ void __launch_bounds__(256) peer_gather_kernel(const __grid_constant__ GatherArgs a, int planes, unsigned per_plane, unsigned rows,
                                                          unsigned vps, long long src_row0, long long src_stride,
                                                          long long dst_pstride, long long dst_stride) {
  const unsigned total = per_plane * static_cast<unsigned>(planes);
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned g0 = blockIdx.x * blockDim.x + threadIdx.x; g0 < total; g0 += stride * kGatherUnroll) {
    uint4 val[kGatherUnroll];
    uint4* dp[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const unsigned g = g0 + u * stride;
      dp[u] = nullptr;
      if (g < total && g >= g0) {                          // (g >= g0: no wrap past 2^32)
        const unsigned pl = g / per_plane, rem = g - pl * per_plane;
        const unsigned sgi = rem / vps, v = rem - sgi * vps;
        const unsigned p = sgi / rows, i = sgi - p * rows;
        const uint4* sp = reinterpret_cast<const uint4*>(a.src[pl][p] + src_row0 + i * src_stride) + v;
        dp[u] = reinterpret_cast<uint4*>(a.dst[pl] + p * dst_pstride + i * dst_stride) + v;
        val[u] = __ldcs(sp);
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u)
      if (dp[u] != nullptr) *dp[u] = val[u];
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

extern "C" int orl_peer_gather(const void* const* src, void* const* dst, int planes, int n_peers, long long rows,
                               long long seg_bytes, long long src_row0, long long src_stride, long long dst_pstride,
                               long long dst_stride, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (src == nullptr || dst == nullptr || planes < 1 || planes > kGatherPlanes || n_peers < 1 || n_peers > kMaxPeers ||
      rows < 0 || seg_bytes < 0 || src_row0 < 0 || src_stride < 0 || dst_pstride < 0 || dst_stride < 0)
    return ORL_ERR_ARG;
  if (((seg_bytes | src_row0 | src_stride | dst_pstride | dst_stride) & 15) != 0) return ORL_ERR_ALIGN;
  if (rows == 0 || seg_bytes == 0) return ORL_OK;
  const long long vps = seg_bytes / 16;
  const long long per_plane = static_cast<long long>(n_peers) * rows * vps;
  if (per_plane * planes >= (1ll << 31)) return ORL_ERR_CAPACITY;
  GatherArgs a{};
  for (int pl = 0; pl < planes; ++pl) {
    a.dst[pl] = static_cast<uint8_t*>(dst[pl]);
    if (a.dst[pl] == nullptr || (reinterpret_cast<uintptr_t>(a.dst[pl]) & 15u)) return ORL_ERR_ALIGN;
    for (int p = 0; p < n_peers; ++p) {
      a.src[pl][p] = static_cast<const uint8_t*>(src[pl * n_peers + p]);
      if (a.src[pl][p] == nullptr || (reinterpret_cast<uintptr_t>(a.src[pl][p]) & 15u)) return ORL_ERR_ALIGN;
    }
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (per_plane * planes + 256 * kGatherUnroll - 1) / (256 * kGatherUnroll);
  const int blocks = static_cast<int>(want < sms * 8ll ? (want > 0 ? want : 1) : sms * 8ll);
  peer_gather_kernel<<<blocks, 256, 0, stream>>>(a, planes, static_cast<unsigned>(per_plane),
                                                 static_cast<unsigned>(rows), static_cast<unsigned>(vps), src_row0,
                                                 src_stride, dst_pstride, dst_stride);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
