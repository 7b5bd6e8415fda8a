// Gather/pack kernel and LSE merge.
//
// orl_pack executes a prepared run table: every run copies one contiguous byte range (a run of rows) from a source
// base to a destination base. It replaces the torch.cat copies that assemble each packed segment of the reference
// (src/onereel/attention.py:60-61, 69; src/onereel/models/hunyuan15.py:164, 168, 225; parallel/comm.py:200) and the
// scatter of outputs back to token rows (hunyuan15.py:231-235; wan.py:117-118). The copies run on the TMA engine as
// untiled bulk copies staged through shared memory: all runs of a plane (e.g. K, then V sharing the same table) are
// one flat byte space cut into tiles of kPackTile bytes; a CTA (one per SM, one issuing thread) takes tiles in a
// grid-stride loop, cuts each into pieces of at most kPackStage bytes that stay inside one run, and keeps a ring of
// kPackStages pieces in flight: bulk load global -> shared (completion on the stage's mbarrier), then, kPackLag
// pieces later, bulk store shared -> global; a stage is reloaded once its store has finished reading it. Every byte
// crosses HBM once each way and no thread touches the data.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "orl_common.h"
#include "ptx.cuh"

namespace orl {

constexpr int kPackStages = 6;
constexpr int kPackLag = 3;                          // stores trail loads by this many pieces
constexpr int kPackStage = 32 * 1024;                // bytes per piece / shared-memory stage
constexpr long long kPackTile = 256 * 1024;          // bytes per grid-stride tile
constexpr int kPackSmem = kPackStages * kPackStage + kPackStages * 8 + 16;
constexpr int kMaxSlots = 16;                     // e.g. one per peer GPU of an exchange plus locals
constexpr int kMaxPlanes = 3;
static_assert(kPackLag < kPackStages, "a stage must be stored before it is reloaded");

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

__global__ void __launch_bounds__(32) pack_kernel(const CopyRun* __restrict__ runs, int n_runs,
                                                  long long total_bytes, long long tiles_per_plane, int n_planes,
                                                  int n_slots, PackBases bases, const int32_t* __restrict__ seg_len,
                                                  int n_seg, int32_t* __restrict__ cu_out, int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t pack_smem[];
  if (threadIdx.x != 0) return;
  if (cu_out != nullptr && blockIdx.x == 0) {
    int32_t acc = 0;
    cu_out[0] = 0;
    for (int i = 0; i < n_seg; ++i) {
      acc += seg_len[i];
      cu_out[i + 1] = acc;
    }
  }
  const uint32_t stage0 = smem_u32(pack_smem);
  const uint32_t bar0 = stage0 + kPackStages * kPackStage;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(pack_smem + kPackStages * kPackStage + kPackStages * 8);
  *abort_flag = 0;
  for (int st = 0; st < kPackStages; ++st) mbar_init(bar0 + 8u * st, 1);
  fence_mbar_init();
  const uint64_t pol = policy_evict_first();         // sources are read once
  uint8_t* pdst[kPackStages] = {};                   // destination and size of the piece in each stage
  uint32_t pbytes[kPackStages] = {};
  long long issued = 0, stored = 0;                  // pieces loaded / stored
  bool ok = true;
  auto store = [&](long long j) -> bool {
    const int st = static_cast<int>(j % kPackStages);
    if (!mbar_wait(bar0 + 8u * st, static_cast<uint32_t>((j / kPackStages) & 1), abort_flag)) return false;
    bulk_store(pdst[st], stage0 + st * kPackStage, pbytes[st]);
    bulk_commit();
    return true;
  };
  const long long n_tiles = tiles_per_plane * n_planes;
  for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
    const int plane = static_cast<int>(tile / tiles_per_plane);
    long long b = (tile - plane * tiles_per_plane) * kPackTile;
    const long long e = b + kPackTile < total_bytes ? b + kPackTile : total_bytes;
    int r = find_run(runs, n_runs, b >> 4);
    while (ok && b < e) {
      const long long r0 = __ldg(&runs[r].vec0) << 4;
      const long long r1 = r + 1 < n_runs ? __ldg(&runs[r + 1].vec0) << 4 : total_bytes;
      if (b >= r1) {                                   // past this run (or an empty one): the next
        ++r;
        continue;
      }
      long long pe = b + kPackStage;
      if (pe > r1) pe = r1;
      if (pe > e) pe = e;
      const int st = static_cast<int>(issued % kPackStages);
      if (issued >= kPackStages) bulk_wait_read<kPackStages - kPackLag - 1>();   // store of piece issued - S read
      const int ss = __ldg(&runs[r].src_slot), ds = __ldg(&runs[r].dst_slot);
      const uint8_t* src = bases.src[plane * n_slots + ss] + __ldg(&runs[r].src_off) + (b - r0);
      pdst[st] = bases.dst[plane * n_slots + ds] + __ldg(&runs[r].dst_off) + (b - r0);
      pbytes[st] = static_cast<uint32_t>(pe - b);
      mbar_expect_tx(bar0 + 8u * st, pbytes[st]);
      bulk_load(stage0 + st * kPackStage, src, pbytes[st], bar0 + 8u * st, pol);
      ++issued;
      if (issued > kPackLag) {
        ok = store(stored);
        stored += ok;
      }
      b = pe;
    }
  }
  while (ok && stored < issued) {
    ok = store(stored);
    stored += ok;
  }
  if (!ok) {
    // wind down: the loads still in flight must land before the CTA's shared memory is released
    for (long long j = stored; j < issued; ++j) {
      const int st = static_cast<int>(j % kPackStages);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(bar0 + 8u * st, static_cast<uint32_t>((j / kPackStages) & 1)))
        if (global_ns() - t0 > kWaitLimitNs) break;
    }
    if (err != nullptr) atomicOr(err, kErrTimeoutPack);
  }
  bulk_wait<0>();
}

// Merge weights of two partial results by their log-sum-exp (m = max(l1, l2), 0 when both are -inf):
// a = w1 / (w1 + w2), b = w2 / (w1 + w2) with w_i = exp(l_i - m), and the merged lse m + log(w1 + w2); when both
// parts are empty (lse -inf) the weights are 0 and the lse stays -inf.
__device__ __forceinline__ float merge_weights(float l1, float l2, float& a, float& b) {
  float m = fmaxf(l1, l2);
  if (isinf(m)) m = 0.f;
  const float w1 = __expf(l1 - m), w2 = __expf(l2 - m);
  const float den = w1 + w2;
  if (!(den > 0.f)) {            // neither part has a key: zero output, lse -inf (as a segment without keys)
    a = b = 0.f;
    return -INFINITY;
  }
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
                        int32_t* cu_out_dev, int* err_dev, void* stream_ptr) {
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
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static std::mutex mu;                              // the shared-memory opt-in, once per device
  static bool smem_set[64] = {};
  if (dev < 0 || dev >= 64) return ORL_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!smem_set[dev]) {
      if (cudaFuncSetAttribute(pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPackSmem) != cudaSuccess)
        return ORL_ERR_LAUNCH;
      smem_set[dev] = true;
    }
  }
  const long long total_bytes = total_vecs * 16;
  const long long tiles_per_plane = (total_bytes + kPackTile - 1) / kPackTile;
  long long blocks = tiles_per_plane * n_planes;
  if (blocks > sms) blocks = sms;                    // one CTA per SM: its shared memory is the copy ring
  if (blocks < 1) blocks = 1;
  pack_kernel<<<static_cast<int>(blocks), 32, kPackSmem, stream>>>(runs_dev, n_runs, total_bytes, tiles_per_plane,
                                                                   n_planes, n_slots, b, seg_len_dev, n_seg,
                                                                   cu_out_dev, err_dev);
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
