// Gather/pack kernel and LSE merge.
//
// orl_pack executes a prepared run table: every run copies one contiguous byte range (a run of rows) from a source
// base to a destination base. It replaces the torch.cat copies that assemble each packed segment of the reference
// (src/onereel/attention.py:60-61, 69; src/onereel/models/hunyuan15.py:164, 168, 225; parallel/comm.py:200) and the
// scatter of outputs back to token rows (hunyuan15.py:231-235; wan.py:117-118). All runs of all planes (e.g. K and V
// sharing one table) are one flat space of 16-byte vectors; each thread moves kVecPerThread vectors with all loads
// issued before the stores (memory-level parallelism), consecutive threads on consecutive vectors (coalesced).
// The run of a vector is found by binary search over the runs' vector prefix (vec0), staged in shared memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"

namespace orl {

constexpr int kPackThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int kMaxSlots = 8;
constexpr int kMaxPlanes = 3;
constexpr int kSmemRuns = 2048;   // run prefixes staged in shared memory (larger tables read global memory)

struct PackBases {
  const uint8_t* src[kMaxPlanes * kMaxSlots];
  uint8_t* dst[kMaxPlanes * kMaxSlots];
};

__device__ __forceinline__ int find_run(const long long* vec0, int n_runs, long long v) {
  int lo = 0, hi = n_runs - 1;   // last run with vec0 <= v
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (vec0[mid] <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(const CopyRun* __restrict__ runs, int n_runs,
                                                            long long total_vecs, int n_planes, int n_slots,
                                                            PackBases bases, const int32_t* __restrict__ seg_len,
                                                            int n_seg, int32_t* __restrict__ cu_out) {
  __shared__ long long s_vec0[kSmemRuns];
  const bool staged = n_runs <= kSmemRuns;
  if (staged)
    for (int i = threadIdx.x; i < n_runs; i += blockDim.x) s_vec0[i] = runs[i].vec0;
  __syncthreads();
  if (cu_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    int32_t acc = 0;
    cu_out[0] = 0;
    for (int i = 0; i < n_seg; ++i) {
      acc += seg_len[i];
      cu_out[i + 1] = acc;
    }
  }
  const long long all = total_vecs * n_planes;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long base = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; base < all;
       base += stride * kVecPerThread) {
    uint4 val[kVecPerThread];
    uint4* dst[kVecPerThread];
#pragma unroll
    for (int u = 0; u < kVecPerThread; ++u) {
      const long long g = base + u * stride;
      dst[u] = nullptr;
      if (g < all) {
        const int plane = static_cast<int>(g / total_vecs);
        const long long v = g - static_cast<long long>(plane) * total_vecs;
        const int r = staged ? find_run(s_vec0, n_runs, v) : [&] {
          int lo = 0, hi = n_runs - 1;
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (runs[mid].vec0 <= v) lo = mid; else hi = mid - 1;
          }
          return lo;
        }();
        const CopyRun run = runs[r];
        const long long off = (v - run.vec0) * 16;
        const uint4* src =
            reinterpret_cast<const uint4*>(bases.src[plane * n_slots + run.src_slot] + run.src_off + off);
        dst[u] = reinterpret_cast<uint4*>(bases.dst[plane * n_slots + run.dst_slot] + run.dst_off + off);
        val[u] = __ldg(src);
      }
    }
#pragma unroll
    for (int u = 0; u < kVecPerThread; ++u)
      if (dst[u] != nullptr) *dst[u] = val[u];
  }
}

// o1 = (o1 * w1 + o2 * w2) / (w1 + w2), lse1 = m + log(w1 + w2) with m = max(lse1, lse2) (0 when both are -inf).
// One warp per (row, head); each lane handles head_dim / 32 contiguous elements.
__global__ void lse_merge_kernel(__nv_bfloat16* __restrict__ o1, float* __restrict__ lse1,
                                 const __nv_bfloat16* __restrict__ o2, const float* __restrict__ lse2, long long n,
                                 long long ld1, long long ld2, int heads, int head_dim) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= n * heads) return;
  const long long row = wid / heads;
  const int h = static_cast<int>(wid - row * heads);
  const float l1 = lse1[h * ld1 + row], l2 = lse2[h * ld2 + row];
  float m = fmaxf(l1, l2);
  if (isinf(m)) m = 0.f;
  const float w1 = __expf(l1 - m), w2 = __expf(l2 - m);
  const float den = w1 + w2;
  const float a = w1 / den, b = w2 / den;
  const int per = head_dim / 32;
  __nv_bfloat16* p1 = o1 + (row * heads + h) * head_dim + lane * per;
  const __nv_bfloat16* p2 = o2 + (row * heads + h) * head_dim + lane * per;
  for (int i = 0; i < per; ++i)
    p1[i] = __float2bfloat16_rn(__bfloat162float(p1[i]) * a + __bfloat162float(p2[i]) * b);
  __syncwarp();
  if (lane == 0) lse1[h * ld1 + row] = m + __logf(den);
}

// fp32 accumulator version (parallel/ring.py:63-70 `_merge`): acc (fp32, in/out) with lse_acc merged with a bf16
// partial result and its lse.
__global__ void lse_merge_acc_kernel(float* __restrict__ acc, float* __restrict__ lse_acc,
                                     const __nv_bfloat16* __restrict__ part, const float* __restrict__ lse_part,
                                     long long n, long long ld1, long long ld2, int heads, int head_dim) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= n * heads) return;
  const long long row = wid / heads;
  const int h = static_cast<int>(wid - row * heads);
  const float l1 = lse_acc[h * ld1 + row], l2 = lse_part[h * ld2 + row];
  float m = fmaxf(l1, l2);
  if (isinf(m)) m = 0.f;
  const float w1 = __expf(l1 - m), w2 = __expf(l2 - m);
  const float den = w1 + w2;
  const float a = w1 / den, b = w2 / den;
  const int per = head_dim / 32;
  float* p1 = acc + (row * heads + h) * head_dim + lane * per;
  const __nv_bfloat16* p2 = part + (row * heads + h) * head_dim + lane * per;
  for (int i = 0; i < per; ++i) p1[i] = p1[i] * a + __bfloat162float(p2[i]) * b;
  __syncwarp();
  if (lane == 0) lse_acc[h * ld1 + row] = m + __logf(den);
}

}  // namespace orl

using namespace orl;

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
  if ((total_vecs == 0 || n_runs == 0) && cu_out_dev == nullptr) return ORL_OK;
  if (total_vecs > 0 && (runs_dev == nullptr || src_bases == nullptr || dst_bases == nullptr)) return ORL_ERR_ARG;
  PackBases b{};
  for (int i = 0; i < n_planes * n_slots; ++i) {
    b.src[i] = static_cast<const uint8_t*>(src_bases ? src_bases[i] : nullptr);
    b.dst[i] = static_cast<uint8_t*>(dst_bases ? dst_bases[i] : nullptr);
    if ((reinterpret_cast<uintptr_t>(b.src[i]) | reinterpret_cast<uintptr_t>(b.dst[i])) & 15u) return ORL_ERR_ALIGN;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long all = total_vecs * n_planes;
  long long blocks = (all + kPackThreads * kVecPerThread - 1) / (kPackThreads * kVecPerThread);
  const long long cap = static_cast<long long>(sms) * 8;   // 8 resident 256-thread CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  pack_kernel<<<static_cast<int>(blocks), kPackThreads, 0, stream>>>(
      runs_dev, total_vecs > 0 ? n_runs : 0, total_vecs, n_planes, n_slots, b, seg_len_dev, n_seg, cu_out_dev);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

extern "C" int orl_lse_merge(void* o1, float* lse1, const void* o2, const float* lse2, long long n, long long ld1,
                             long long ld2, int heads, int head_dim, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (o1 == nullptr || o2 == nullptr || lse1 == nullptr || lse2 == nullptr || n < 0 || heads <= 0) return ORL_ERR_ARG;
  if (head_dim % 32 != 0 || head_dim <= 0) return ORL_ERR_UNSUPPORTED;
  if (n == 0) return ORL_OK;
  const long long warps = n * heads;
  const long long blocks = (warps * 32 + 255) / 256;
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
  if (head_dim % 32 != 0 || head_dim <= 0) return ORL_ERR_UNSUPPORTED;
  if (n == 0) return ORL_OK;
  const long long blocks = (n * heads * 32 + 255) / 256;
  lse_merge_acc_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      acc, lse_acc, static_cast<const __nv_bfloat16*>(part), lse_part, n, ld1, ld2, heads, head_dim);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
