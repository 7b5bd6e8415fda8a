// Frame memory on the GPU: per-frame pooling of hidden states and the cosine k-means that picks the representative
// frames (the reference's onereel.frame_memory, src/onereel/frame_memory.py:76-132, runs these as eager torch ops:
// index_add_ per observed layer, then a Python loop of small matmuls, argmaxes and host syncs per Lloyd iteration).
//
// orl_frame_pool: acc[f, c] += sum of hs[row, c] over the rows of frame f and acc[f, C] += their count, rows given in
//   CSR form (rows_by_frame[frame_off[f] .. frame_off[f + 1]]). One block per (frame, 64-column slice): 32 row lanes
//   x 8 column lanes of 16-byte loads, each row lane summing every 32nd row of the frame, then a fixed tree over the
//   row lanes in shared memory — deterministic (no atomics), HBM-bound (every hidden-state byte read once).
// orl_frame_select: one CTA per set (one observed layer) runs the whole selection on device: candidate features =
//   L2-normalised means (sum / max(count, 1), then / max(norm, 1e-12), IEEE division as torch does), farthest-point
//   initialisation from candidate 0 (cosine distance 1 - x.c, running minimum, first maximum), at most `iters` Lloyd
//   steps (assignment = first maximum of x.c; centroid = normalised mean of its members, or unchanged when empty;
//   stop when no centroid changes bit for bit), then per non-empty cluster the medoid (the member with the largest
//   x.c, the lowest candidate on ties — scores within kTieTol count as ties, because two members can be equally near
//   in exact arithmetic, always so in a two-member cluster, and rounding alone would then decide), written sorted.
//   Dot products: fixed lane partition + shuffle tree.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"

namespace orl {
namespace {

constexpr int kPoolCols = 64;      // columns per block
constexpr int kPoolRowLanes = 32;  // rows summed concurrently per block

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__global__ void __launch_bounds__(256) frame_pool_kernel(const T* __restrict__ hs, long long ld_hs, int C,
                                                         const int32_t* __restrict__ rows_by_frame,
                                                         const int32_t* __restrict__ frame_off,
                                                         float* __restrict__ acc, long long ld_acc) {
  __shared__ float part[kPoolRowLanes][kPoolCols + 1];
  const int f = blockIdx.x;
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
  const int col = blockIdx.y * kPoolCols + tx * 8;
  const int r0 = frame_off[f], r1 = frame_off[f + 1];
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (col < C) {
    // rows i, i + 32, i + 64, ... of the frame, added in that order; four rows' loads in flight at a time
    int i = r0 + ty;
    for (; i + 3 * kPoolRowLanes < r1; i += 4 * kPoolRowLanes) {
      int idx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) idx[u] = __ldg(&rows_by_frame[i + u * kPoolRowLanes]);
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8<T>(hs + static_cast<long long>(idx[u]) * ld_hs + col, v[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] += v[u][e];
    }
    for (; i < r1; i += kPoolRowLanes) {
      float v[8];
      load8<T>(hs + static_cast<long long>(rows_by_frame[i]) * ld_hs + col, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] += v[e];
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[ty][tx * 8 + e] = s[e];
  __syncthreads();
  for (int stride = kPoolRowLanes / 2; stride > 0; stride >>= 1) {
    if (ty < stride) {
#pragma unroll
      for (int e = 0; e < 8; ++e) part[ty][tx * 8 + e] += part[ty + stride][tx * 8 + e];
    }
    __syncthreads();
  }
  if (ty == 0 && col < C) {
    float* a = acc + static_cast<long long>(f) * ld_acc + col;
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] += part[0][tx * 8 + e];
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) acc[static_cast<long long>(f) * ld_acc + C] += static_cast<float>(r1 - r0);
}

// ------------------------------------------------------------------------------------------------ selection

constexpr int kSelThreads = 1024;
constexpr float kTieTol = 1e-6f;   // medoid scores (cosines) this close count as a tie
constexpr int kSelWarps = kSelThreads / 32;

struct ArgMax {
  float v;
  int i;
};

// larger value wins; equal values: the lower index (torch.argmax returns the first maximum)
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  return a;
}

// first maximum of vals[0 .. n) over the block (every thread gets the index)
__device__ int block_argmax(const float* vals, int n, ArgMax* red) {
  ArgMax a{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < n; i += blockDim.x) a = better(a, ArgMax{vals[i], i});
  a = warp_argmax(a);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = a;
  __syncthreads();
  if (w == 0) {
    a = l < kSelWarps ? red[l] : ArgMax{-INFINITY, 0x7fffffff};
    a = warp_argmax(a);
    if (l == 0) red[0] = a;
  }
  __syncthreads();
  const int res = red[0].i;
  __syncthreads();
  return res;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// dot of two C-vectors by one warp: lane l sums columns l, l + 32, ... in order, then a fixed shuffle tree
__device__ __forceinline__ float warp_dot(const float* a, const float* b, int C) {
  float s = 0.f;
  for (int c = threadIdx.x & 31; c < C; c += 32) s = fmaf(a[c], b[c], s);
  return warp_sum(s);
}

__global__ void __launch_bounds__(kSelThreads) frame_select_kernel(float* __restrict__ feat_base, long long ld,
                                                                   long long set_stride, int C, int normalize,
                                                                   const int32_t* __restrict__ cand, int n_cand, int k,
                                                                   int iters, float* __restrict__ scratch_base,
                                                                   long long scratch_stride,
                                                                   int32_t* __restrict__ reps_base) {
  __shared__ ArgMax red[kSelWarps];
  __shared__ int centre_sh[64];
  __shared__ int changed;
  float* feat = feat_base + blockIdx.x * set_stride;
  float* scratch = scratch_base + blockIdx.x * scratch_stride;
  int32_t* reps = reps_base + blockIdx.x * (k + 1);
  float* cur = scratch;                                   // [k, C] centroids
  float* nxt = cur + static_cast<long long>(k) * C;       // [k, C] next centroids
  float* dots = nxt + static_cast<long long>(k) * C;      // [n_cand, k]
  float* dist = dots + static_cast<long long>(n_cand) * k; // [n_cand]
  int* z = reinterpret_cast<int*>(dist + n_cand);         // [n_cand] assignment
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto row = [&](int i) { return feat + static_cast<long long>(cand[i]) * ld; };

  // candidate features: normalised means, in place over the accumulated sums
  if (normalize) {
    for (int i = warp; i < n_cand; i += kSelWarps) {
      float* x = row(i);
      const float cnt = fmaxf(x[C], 1.0f);
      float ss = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float m = __fdiv_rn(x[c], cnt);
        x[c] = m;
        ss = fmaf(m, m, ss);
      }
      const float nrm = fmaxf(__fsqrt_rn(warp_sum(ss)), 1e-12f);
      __syncwarp();
      for (int c = lane; c < C; c += 32) x[c] = __fdiv_rn(x[c], nrm);
    }
    __syncthreads();
  }

  // farthest-point initialisation: centre 0 = candidate 0, then the candidate farthest from its nearest centre
  if (threadIdx.x == 0) centre_sh[0] = 0;
  __syncthreads();
  for (int t = 0; t < k; ++t) {
    const int ct = centre_sh[t];
    for (int i = warp; i < n_cand; i += kSelWarps) {
      const float d = 1.0f - warp_dot(row(i), row(ct), C);
      if (lane == 0) dist[i] = t == 0 ? d : fminf(dist[i], d);
    }
    __syncthreads();
    if (t + 1 < k) {
      const int nx = block_argmax(dist, n_cand, red);
      if (threadIdx.x == 0) centre_sh[t + 1] = nx;
      __syncthreads();
    }
  }
  for (int idx = threadIdx.x; idx < k * C; idx += blockDim.x) cur[idx] = row(centre_sh[idx / C])[idx % C];
  __syncthreads();

  auto assign = [&]() {
    for (int p = warp; p < n_cand * k; p += kSelWarps) {
      const float d = warp_dot(row(p / k), cur + static_cast<long long>(p % k) * C, C);
      if (lane == 0) dots[p] = d;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
      int best = 0;
      for (int j = 1; j < k; ++j)
        if (dots[i * k + j] > dots[i * k + best]) best = j;
      z[i] = best;
    }
    __syncthreads();
  };

  for (int it = 0; it < iters; ++it) {
    assign();
    // next centroids: members summed in candidate order, mean, then normalised; empty clusters keep theirs
    for (int j = 0; j < k; ++j) {
      int cnt = 0;
      for (int i = 0; i < n_cand; ++i) cnt += z[i] == j;
      float* nj = nxt + static_cast<long long>(j) * C;
      const float* cj = cur + static_cast<long long>(j) * C;
      if (cnt == 0) {
        for (int c = threadIdx.x; c < C; c += blockDim.x) nj[c] = cj[c];
        continue;
      }
      float ss = 0.f;
      for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float s = 0.f;
        for (int i = 0; i < n_cand; ++i)
          if (z[i] == j) s += row(i)[c];
        const float m = __fdiv_rn(s, static_cast<float>(cnt));
        nj[c] = m;
        ss = fmaf(m, m, ss);
      }
      // norm: per-warp partials, then a fixed tree over the warps
      ss = warp_sum(ss);
      __shared__ float wsum[kSelWarps];
      if (lane == 0) wsum[warp] = ss;
      __syncthreads();
      if (warp == 0) {
        float t = lane < kSelWarps ? wsum[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) wsum[0] = t;
      }
      __syncthreads();
      const float nrm = fmaxf(__fsqrt_rn(wsum[0]), 1e-12f);
      __syncthreads();
      for (int c = threadIdx.x; c < C; c += blockDim.x) nj[c] = __fdiv_rn(nj[c], nrm);
    }
    if (threadIdx.x == 0) changed = 0;
    __syncthreads();
    for (int idx = threadIdx.x; idx < k * C; idx += blockDim.x)
      if (__float_as_uint(nxt[idx]) != __float_as_uint(cur[idx])) changed = 1;
    __syncthreads();
    const bool stop = changed == 0;
    __syncthreads();
    if (stop) break;
    float* t = cur;
    cur = nxt;
    nxt = t;
  }
  assign();
  // medoid of every non-empty cluster, then the indices sorted
  if (warp == 0) {
    int out[64];
    int n = 0;
    for (int j = 0; j < k; ++j) {
      ArgMax a{-INFINITY, 0x7fffffff};
      for (int i = lane; i < n_cand; i += 32)
        if (z[i] == j) a = better(a, ArgMax{dots[i * k + j], i});
      a = warp_argmax(a);
      if (a.i == 0x7fffffff) continue;
      // the lowest member within kTieTol of the best: members equally near the centroid in exact arithmetic (both
      // members of a two-member cluster always are) resolve to the lowest candidate, not to rounding
      int first = 0x7fffffff;
      for (int i = lane; i < n_cand; i += 32)
        if (z[i] == j && dots[i * k + j] >= a.v - kTieTol) first = min(first, i);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
      out[n++] = cand[first];
    }
    if (lane == 0) {
      for (int a = 1; a < n; ++a)
        for (int b = a; b > 0 && out[b - 1] > out[b]; --b) {
          const int t = out[b];
          out[b] = out[b - 1];
          out[b - 1] = t;
        }
      reps[0] = n;
      for (int j = 0; j < n; ++j) reps[1 + j] = out[j];
      for (int j = n; j < k; ++j) reps[1 + j] = -1;
    }
  }
}

}  // namespace
}  // namespace orl

using namespace orl;

extern "C" int orl_frame_pool(const void* hs, int dtype, long long ld_hs, int C, const int32_t* rows_by_frame,
                              const int32_t* frame_off, int n_frames, float* acc, long long ld_acc, void* stream) {
  if (hs == nullptr || rows_by_frame == nullptr || frame_off == nullptr || acc == nullptr) return ORL_ERR_ARG;
  if (C <= 0 || n_frames < 0 || ld_hs < C || ld_acc < C + 1 || (dtype != 0 && dtype != 1)) return ORL_ERR_ARG;
  const int esz = dtype == 0 ? 2 : 4;
  if (C % 8 != 0 || (ld_hs * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(hs) & 15u) != 0) return ORL_ERR_ALIGN;
  if (n_frames == 0) return ORL_OK;
  dim3 grid(n_frames, (C + kPoolCols - 1) / kPoolCols);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == 0)
    frame_pool_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(hs), ld_hs, C,
                                                         rows_by_frame, frame_off, acc, ld_acc);
  else
    frame_pool_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(hs), ld_hs, C, rows_by_frame, frame_off,
                                                 acc, ld_acc);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

extern "C" long long orl_frame_select_scratch(int C, int n_cand, int k) {
  if (C <= 0 || n_cand < 0 || k <= 0) return ORL_ERR_ARG;
  return 2ll * k * C + static_cast<long long>(n_cand) * k + 2ll * n_cand;
}

extern "C" int orl_frame_select(float* feat, long long ld, long long set_stride, int n_sets, int C, int normalize,
                                const int32_t* cand, int n_cand, int k, int iters, float* scratch,
                                long long scratch_stride, int32_t* reps, void* stream) {
  if (feat == nullptr || cand == nullptr || scratch == nullptr || reps == nullptr) return ORL_ERR_ARG;
  if (n_sets <= 0 || C <= 0 || ld < C + (normalize ? 1 : 0) || n_cand <= 0 || k <= 0 || k > n_cand || k > 64 ||
      iters < 0)
    return ORL_ERR_ARG;
  if (scratch_stride < orl_frame_select_scratch(C, n_cand, k)) return ORL_ERR_CAPACITY;
  frame_select_kernel<<<n_sets, kSelThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      feat, ld, set_stride, C, normalize, cand, n_cand, k, iters, scratch, scratch_stride, reps);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
