// Gather/pack kernel and LSE merge.
//
// orl_pack executes a prepared run table: every run copies one contiguous byte range (a run of rows) from a source
// base to a destination base. It replaces the torch.cat copies that assemble each packed segment of the reference
// (src/onereel/attention.py:60-61, 69; src/onereel/models/hunyuan15.py:164, 168, 225; parallel/comm.py:200) and the
// scatter of outputs back to token rows (hunyuan15.py:231-235; wan.py:117-118). All runs of a plane (e.g. K, then V
// sharing the same table) are one flat space of 16-byte vectors cut into tiles of kPackTile vectors; a block takes
// tiles in a grid-stride loop, finds the run of the tile's first vector once (binary search over the runs' vector
// prefix, uniform across the block), and each thread then copies kPackUnroll vectors of the tile, consecutive
// threads on consecutive 16-byte vectors (coalesced), all loads issued before the stores. A thread's run index only
// moves forward inside a tile (runs are at least one 16-byte vector, usually whole rows of kilobytes).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"

namespace orl {

constexpr int kPackThreads = 256;
constexpr int kPackUnroll = 8;
constexpr int kPackTile = kPackThreads * kPackUnroll;   // 2048 vectors = 32 KiB per tile
constexpr int kMaxSlots = 8;
constexpr int kMaxPlanes = 3;

struct PackBases {
  const uint8_t* src[kMaxPlanes * kMaxSlots];
  uint8_t* dst[kMaxPlanes * kMaxSlots];
};

// last run whose vec0 <= v (runs sorted by vec0, runs[0].vec0 == 0)
__device__ __forceinline__ int find_run(const CopyRun* __restrict__ runs, int n_runs, long long v) {
  int lo = 0, hi = n_runs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(&runs[mid].vec0) <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(const CopyRun* __restrict__ runs, int n_runs,
                                                            long long total_vecs, long long tiles_per_plane,
                                                            int n_planes, int n_slots, PackBases bases,
                                                            const int32_t* __restrict__ seg_len, int n_seg,
                                                            int32_t* __restrict__ cu_out) {
  if (cu_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    int32_t acc = 0;
    cu_out[0] = 0;
    for (int i = 0; i < n_seg; ++i) {
      acc += seg_len[i];
      cu_out[i + 1] = acc;
    }
  }
  const long long n_tiles = tiles_per_plane * n_planes;
  for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int plane = static_cast<int>(tile / tiles_per_plane);
    const long long t0 = (tile - plane * tiles_per_plane) * kPackTile;
    int r = find_run(runs, n_runs, t0);              // same address on every thread: a broadcast load
    long long next = r + 1 < n_runs ? __ldg(&runs[r + 1].vec0) : total_vecs;
    uint4 val[kPackUnroll];
    uint4* dst[kPackUnroll];
#pragma unroll
    for (int u = 0; u < kPackUnroll; ++u) {
      const long long v = t0 + threadIdx.x + u * kPackThreads;
      dst[u] = nullptr;
      if (v < total_vecs) {
        while (v >= next) {                          // the thread's run moves forward only
          ++r;
          next = r + 1 < n_runs ? __ldg(&runs[r + 1].vec0) : total_vecs;
        }
        const long long off = (v - __ldg(&runs[r].vec0)) * 16;
        const int ss = __ldg(&runs[r].src_slot), ds = __ldg(&runs[r].dst_slot);
        const uint4* src =
            reinterpret_cast<const uint4*>(bases.src[plane * n_slots + ss] + __ldg(&runs[r].src_off) + off);
        dst[u] = reinterpret_cast<uint4*>(bases.dst[plane * n_slots + ds] + __ldg(&runs[r].dst_off) + off);
        val[u] = __ldcs(src);                        // source rows are read once: streaming load
      }
    }
#pragma unroll
    for (int u = 0; u < kPackUnroll; ++u)
      if (dst[u] != nullptr) *dst[u] = val[u];
  }
}

// Merge weights of two partial results by their log-sum-exp (m = max(l1, l2), 0 when both are -inf):
// a = w1 / (w1 + w2), b = w2 / (w1 + w2) with w_i = exp(l_i - m), and the merged lse m + log(w1 + w2).
__device__ __forceinline__ float merge_weights(float l1, float l2, float& a, float& b) {
  float m = fmaxf(l1, l2);
  if (isinf(m)) m = 0.f;
  const float w1 = __expf(l1 - m), w2 = __expf(l2 - m);
  const float den = w1 + w2;
  a = w1 / den;
  b = w2 / den;
  return m + __logf(den);
}

// lanes of the thread's (row, head) group: `per` consecutive lanes (per a power of two <= 32, groups warp-aligned)
__device__ __forceinline__ unsigned group_mask(int per) {
  const unsigned lane = threadIdx.x & 31u;
  return per >= 32 ? 0xffffffffu : (((1u << per) - 1u) << (lane & ~static_cast<unsigned>(per - 1)));
}

// o1 = (o1 * w1 + o2 * w2) / (w1 + w2) and lse1 = merged lse, in place (hunyuan15.py:274-276). One thread per
// 8 elements (16 bytes) of a (row, head); the head_dim / 8 threads of a (row, head) are consecutive lanes of one
// warp, which read the two lse values before the group's first lane overwrites lse1.
__global__ void lse_merge_kernel(__nv_bfloat16* __restrict__ o1, float* __restrict__ lse1,
                                 const __nv_bfloat16* __restrict__ o2, const float* __restrict__ lse2, long long n,
                                 long long ld1, long long ld2, int heads, int head_dim) {
  const int per = head_dim >> 3;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n * heads * per) return;
  const long long rh = idx / per;
  const int c = static_cast<int>(idx - rh * per);
  const long long row = rh / heads;
  const int h = static_cast<int>(rh - row * heads);
  float a, b;
  const float lse = merge_weights(lse1[h * ld1 + row], lse2[h * ld2 + row], a, b);
  uint4* p1 = reinterpret_cast<uint4*>(o1 + rh * head_dim) + c;
  const uint4 x = *p1, y = __ldg(reinterpret_cast<const uint4*>(o2 + rh * head_dim) + c);
  const uint32_t* xw = &x.x;
  const uint32_t* yw = &y.x;
  uint4 r;
  uint32_t* rw = &r.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 xf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[i]));
    const float2 yf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yw[i]));
    const __nv_bfloat162 o = __floats2bfloat162_rn(xf.x * a + yf.x * b, xf.y * a + yf.y * b);
    rw[i] = *reinterpret_cast<const uint32_t*>(&o);
  }
  *p1 = r;
  __syncwarp(group_mask(per));
  if (c == 0) lse1[h * ld1 + row] = lse;
}

// fp32 accumulator version (parallel/ring.py:63-70 `_merge`): acc (fp32, in/out) with lse_acc merged with a bf16
// partial result and its lse; one thread per 8 elements as above.
__global__ void lse_merge_acc_kernel(float* __restrict__ acc, float* __restrict__ lse_acc,
                                     const __nv_bfloat16* __restrict__ part, const float* __restrict__ lse_part,
                                     long long n, long long ld1, long long ld2, int heads, int head_dim) {
  const int per = head_dim >> 3;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n * heads * per) return;
  const long long rh = idx / per;
  const int c = static_cast<int>(idx - rh * per);
  const long long row = rh / heads;
  const int h = static_cast<int>(rh - row * heads);
  float a, b;
  const float lse = merge_weights(lse_acc[h * ld1 + row], lse_part[h * ld2 + row], a, b);
  float4* p1 = reinterpret_cast<float4*>(acc + rh * head_dim) + 2 * c;
  const uint4 y = __ldg(reinterpret_cast<const uint4*>(part + rh * head_dim) + c);
  const uint32_t* yw = &y.x;
  float4 x0 = p1[0], x1 = p1[1];
  const float2 y0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yw[0]));
  const float2 y1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yw[1]));
  const float2 y2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yw[2]));
  const float2 y3 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yw[3]));
  x0 = make_float4(x0.x * a + y0.x * b, x0.y * a + y0.y * b, x0.z * a + y1.x * b, x0.w * a + y1.y * b);
  x1 = make_float4(x1.x * a + y2.x * b, x1.y * a + y2.y * b, x1.z * a + y3.x * b, x1.w * a + y3.y * b);
  p1[0] = x0;
  p1[1] = x1;
  __syncwarp(group_mask(per));
  if (c == 0) lse_acc[h * ld1 + row] = lse;
}

}  // namespace orl

using namespace orl;

// the merge kernels give a (row, head) head_dim / 8 lanes of one warp: a power of two from 1 to 32
static bool merge_head_dim_ok(int head_dim) {
  const int per = head_dim / 8;
  return head_dim > 0 && head_dim % 8 == 0 && per <= 32 && (per & (per - 1)) == 0;
}

extern "C" long long orl_pack_prepare(orl_copy_run* runs, const int64_t* nbytes, int n_runs) {
  if (n_runs < 0 || (n_runs > 0 && (runs == nullptr || nbytes == nullptr))) return ORL_ERR_ARG;
  long long acc = 0;
  for (int i = 0; i < n_runs; ++i) {
    if (nbytes[i] < 0 || (nbytes[i] & 15) || (runs[i].src_off & 15) || (runs[i].dst_off & 15) || runs[i].src_off < 0 ||
        runs[i].dst_off < 0)
      return ORL_ERR_ALIGN;
    if (runs[i].src_slot < 0 || runs[i].src_slot >= kMaxSlots || runs[i].dst_slot < 0 ||
        runs[i].dst_slot >= kMaxSlots)
      return ORL_ERR_ARG;
    runs[i].vec0 = acc;
    acc += nbytes[i] / 16;
  }
  return acc;
}

extern "C" int orl_pack(const orl_copy_run* runs_dev, int n_runs, long long total_vecs, int n_planes, int n_slots,
                        const void* const* src_bases, void* const* dst_bases, const int32_t* seg_len_dev, int n_seg,
                        int32_t* cu_out_dev, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (n_planes < 1 || n_planes > kMaxPlanes || n_slots < 1 || n_slots > kMaxSlots || n_runs < 0 || total_vecs < 0)
    return ORL_ERR_ARG;
  if (cu_out_dev != nullptr && (n_seg < 0 || (n_seg > 0 && seg_len_dev == nullptr))) return ORL_ERR_ARG;
  if (total_vecs > 0 && n_runs == 0) return ORL_ERR_ARG;
  if (total_vecs == 0 && cu_out_dev == nullptr) return ORL_OK;
  if (total_vecs > 0 && (runs_dev == nullptr || src_bases == nullptr || dst_bases == nullptr)) return ORL_ERR_ARG;
  PackBases b{};
  for (int i = 0; i < n_planes * n_slots; ++i) {
    b.src[i] = static_cast<const uint8_t*>(src_bases ? src_bases[i] : nullptr);
    b.dst[i] = static_cast<uint8_t*>(dst_bases ? dst_bases[i] : nullptr);
    if ((reinterpret_cast<uintptr_t>(b.src[i]) | reinterpret_cast<uintptr_t>(b.dst[i])) & 15u) return ORL_ERR_ALIGN;
  }
  int dev = 0, sms = 148, per_sm = 4;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pack_kernel, kPackThreads, 0);
  const long long tiles_per_plane = (total_vecs + kPackTile - 1) / kPackTile;
  long long blocks = tiles_per_plane * n_planes;
  const long long cap = static_cast<long long>(sms) * (per_sm > 0 ? per_sm : 1);   // one resident wave
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  pack_kernel<<<static_cast<int>(blocks), kPackThreads, 0, stream>>>(runs_dev, n_runs, total_vecs, tiles_per_plane,
                                                                     n_planes, n_slots, b, seg_len_dev, n_seg,
                                                                     cu_out_dev);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

extern "C" int orl_lse_merge(void* o1, float* lse1, const void* o2, const float* lse2, long long n, long long ld1,
                             long long ld2, int heads, int head_dim, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (o1 == nullptr || o2 == nullptr || lse1 == nullptr || lse2 == nullptr || n < 0 || heads <= 0) return ORL_ERR_ARG;
  if (!merge_head_dim_ok(head_dim)) return ORL_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(o1) | reinterpret_cast<uintptr_t>(o2)) & 15u) != 0) return ORL_ERR_ALIGN;
  if (n == 0) return ORL_OK;
  const long long blocks = (n * heads * (head_dim / 8) + 255) / 256;
  lse_merge_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(o1), lse1, static_cast<const __nv_bfloat16*>(o2), lse2, n, ld1, ld2, heads,
      head_dim);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

extern "C" int orl_lse_merge_acc(float* acc, float* lse_acc, const void* part, const float* lse_part, long long n,
                                 long long ld1, long long ld2, int heads, int head_dim, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (acc == nullptr || lse_acc == nullptr || part == nullptr || lse_part == nullptr || n < 0 || heads <= 0)
    return ORL_ERR_ARG;
  if (!merge_head_dim_ok(head_dim)) return ORL_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(acc) | reinterpret_cast<uintptr_t>(part)) & 15u) != 0) return ORL_ERR_ALIGN;
  if (n == 0) return ORL_OK;
  const long long blocks = (n * heads * (head_dim / 8) + 255) / 256;
  lse_merge_acc_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      acc, lse_acc, static_cast<const __nv_bfloat16*>(part), lse_part, n, ld1, ld2, heads, head_dim);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
