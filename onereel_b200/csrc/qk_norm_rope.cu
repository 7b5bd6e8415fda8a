// Fused q/k RMSNorm + rotary embedding, bf16 in / bf16 out, HBM-bound.
//
// Replaces the per-layer q/k preparation of the reference processors:
//   - Wan2.2 (src/onereel/models/wan.py:64-74 `_qk`, a torch.compile'd Triton kernel): RMSNorm over the whole hidden
//     dimension (H * D) with a learned weight, then the interleaved RoPE (cos[..., 0::2], sin[..., 1::2]);
//   - HunyuanVideo-1.5 (src/onereel/models/hunyuan15.py:187-190): RMSNorm per head (over D, weight [D]), then
//     diffusers' apply_rotary_emb over interleaved pairs (cos / sin repeated per pair).
// Both rotations are out[2i] = x[2i] c_i - x[2i+1] s_i, out[2i+1] = x[2i] s_i + x[2i+1] c_i with c_i = cos[row][2i]
// and s_i = sin[row][2i + sin_shift] (sin_shift 0 for the repeated tables, 1 for Wan's).
// One block per kRowsPerBlock rows, one thread per 8 consecutive elements of each (16-byte loads and stores; all of a
// thread's loads — its x vectors, cos / sin entries and weights — issued before any reduction, for memory-level
// parallelism): the sum of squares is reduced over the group's threads (per-head norm: the head_dim / 8 consecutive
// lanes of a head, by shuffles; hidden norm: the whole block, shuffles then shared memory), in fp32. A thread's cos /
// sin entries are table columns d .. d + 7 of its head position d; the output goes to row_map[row] (or row) —
// straight into a packed layout when a row map is given.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"

namespace orl {

constexpr int kRowsPerBlock = 2;

__global__ void __launch_bounds__(1024) qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ x,
                                                           __nv_bfloat16* __restrict__ y,
                                                           const __nv_bfloat16* __restrict__ weight,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, long long rows,
                                                           int hidden, int head_dim, int per_head, float eps,
                                                           int sin_shift, long long rope_ld,
                                                           const int32_t* __restrict__ row_map) {
  __shared__ float part[kRowsPerBlock][32];
  const int t = threadIdx.x;
  const int e = 8 * t;                                   // first element of this thread in a row
  const bool active = e < hidden;
  const int d = active ? e % head_dim : 0;               // position within the head (8 elements never straddle heads)
  const long long row0 = static_cast<long long>(blockIdx.x) * kRowsPerBlock;
  uint4 raw[kRowsPerBlock];
  float4 c[kRowsPerBlock][2], sn4[kRowsPerBlock][2];
  uint4 wr = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int k = 0; k < kRowsPerBlock; ++k) {
    const long long row = row0 + k;
    raw[k] = make_uint4(0u, 0u, 0u, 0u);
    if (active && row < rows) raw[k] = __ldcs(reinterpret_cast<const uint4*>(x + row * hidden + e));
  }
#pragma unroll
  for (int k = 0; k < kRowsPerBlock; ++k) {
    const long long row = row0 + k;
    if (active && row < rows) {
      const float4* cr = reinterpret_cast<const float4*>(cos_t + row * rope_ld + d);
      const float4* sr = reinterpret_cast<const float4*>(sin_t + row * rope_ld + d);
      c[k][0] = __ldg(cr);
      c[k][1] = __ldg(cr + 1);
      sn4[k][0] = __ldg(sr);
      sn4[k][1] = __ldg(sr + 1);
    }
  }
  if (active) wr = __ldg(reinterpret_cast<const uint4*>(weight + (per_head ? d : e)));
  float v[kRowsPerBlock][8], ss[kRowsPerBlock];
#pragma unroll
  for (int k = 0; k < kRowsPerBlock; ++k) {
    const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
    ss[k] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      v[k][2 * i] = f.x;
      v[k][2 * i + 1] = f.y;
      ss[k] += f.x * f.x + f.y * f.y;
    }
  }
  float inv[kRowsPerBlock];
  if (per_head) {
    // head_dim / 8 lanes per head (a power of two <= 32, heads aligned to those lane groups)
#pragma unroll
    for (int k = 0; k < kRowsPerBlock; ++k) {
      for (int o = (head_dim >> 4); o > 0; o >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], o);
      inv[k] = rsqrtf(ss[k] / head_dim + eps);
    }
  } else {
#pragma unroll
    for (int k = 0; k < kRowsPerBlock; ++k) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], o);
      if ((t & 31) == 0) part[k][t >> 5] = ss[k];
    }
    __syncthreads();
    if (t < 32) {
#pragma unroll
      for (int k = 0; k < kRowsPerBlock; ++k) {
        float a = t < static_cast<int>(blockDim.x >> 5) ? part[k][t] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (t == 0) part[k][0] = a;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kRowsPerBlock; ++k) inv[k] = rsqrtf(part[k][0] / hidden + eps);
  }
  if (!active) return;
  const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
  for (int k = 0; k < kRowsPerBlock; ++k) {
    const long long row = row0 + k;
    if (row >= rows) break;
    const float cs[4] = {c[k][0].x, c[k][0].z, c[k][1].x, c[k][1].z};
    const float sn[4] = {sin_shift ? sn4[k][0].y : sn4[k][0].x, sin_shift ? sn4[k][0].w : sn4[k][0].z,
                         sin_shift ? sn4[k][1].y : sn4[k][1].x, sin_shift ? sn4[k][1].w : sn4[k][1].z};
    uint4 packed;
    uint32_t* o = &packed.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 wf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
      const float a = v[k][2 * i] * inv[k] * wf.x, b = v[k][2 * i + 1] * inv[k] * wf.y;
      const __nv_bfloat162 r = __floats2bfloat162_rn(a * cs[i] - b * sn[i], a * sn[i] + b * cs[i]);
      o[i] = *reinterpret_cast<const uint32_t*>(&r);
    }
    const long long orow = row_map ? row_map[row] : row;
    *reinterpret_cast<uint4*>(y + orow * hidden + e) = packed;
  }
}

// In-place rotation of listed rows (no norm): row rows[i] of x is rotated with table row i (pairs as above). Used to
// move shared-frame keys of a packed K to their adjacent temporal positions (hunyuan15.py:127-150 `_move_shared`:
// the two rotations R(-src) then R(dst) composed into one table by the host).
__global__ void rope_rows_kernel(__nv_bfloat16* __restrict__ x, const int32_t* __restrict__ rows, long long n_rows,
                                 int hidden, int head_dim, const float* __restrict__ cos_t,
                                 const float* __restrict__ sin_t, long long rope_ld, int sin_shift) {
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= n_rows) return;
  __nv_bfloat16* xr = x + static_cast<long long>(rows[warp_id]) * hidden;
  const float* cr = cos_t + warp_id * rope_ld;
  const float* sr = sin_t + warp_id * rope_ld;
  for (int e = lane * 8; e < hidden; e += 32 * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(xr + e);
    __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      const int d = (e + 2 * i) % head_dim;
      const float cs = cr[d], sn = sr[d + sin_shift];
      h2[i] = __floats2bfloat162_rn(f.x * cs - f.y * sn, f.x * sn + f.y * cs);
    }
    *reinterpret_cast<uint4*>(xr + e) = raw;
  }
}

}  // namespace orl

using namespace orl;

extern "C" int orl_qk_norm_rope(const void* x, void* y, const void* weight, const float* cos_t, const float* sin_t,
                                long long rows, int heads, int head_dim, int per_head, float eps, int sin_shift,
                                long long rope_ld, const int32_t* row_map, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (x == nullptr || y == nullptr || weight == nullptr || cos_t == nullptr || sin_t == nullptr) return ORL_ERR_ARG;
  if (rows < 0 || heads <= 0 || head_dim <= 0 || (head_dim & 7) || sin_shift < 0 || sin_shift > 1 || rope_ld < head_dim)
    return ORL_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) return ORL_ERR_ALIGN;
  const int hidden = heads * head_dim;
  // per-head norm: head_dim / 8 lanes per head must be a power of two within a warp; one thread per 8 elements
  if (per_head && ((head_dim >> 3) > 32 || ((head_dim >> 3) & ((head_dim >> 3) - 1)) != 0)) return ORL_ERR_UNSUPPORTED;
  if (hidden / 8 > 1024) return ORL_ERR_UNSUPPORTED;
  // 16-byte vectors of the tables and the weight
  if ((rope_ld & 3) || ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t) |
                         reinterpret_cast<uintptr_t>(weight)) & 15u))
    return ORL_ERR_ALIGN;
  if (rows == 0) return ORL_OK;
  const long long blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks > 0x7fffffffLL) return ORL_ERR_ARG;
  const int threads = ((hidden / 8 + 31) / 32) * 32;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(weight),
      cos_t, sin_t, rows, hidden, head_dim, per_head, eps, sin_shift, rope_ld, row_map);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

extern "C" int orl_rope_rows(void* x, const int32_t* rows, long long n_rows, int heads, int head_dim,
                             const float* cos_t, const float* sin_t, long long rope_ld, int sin_shift,
                             void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (x == nullptr || cos_t == nullptr || sin_t == nullptr || (n_rows > 0 && rows == nullptr)) return ORL_ERR_ARG;
  if (n_rows < 0 || heads <= 0 || head_dim <= 0 || (head_dim & 7) || sin_shift < 0 || sin_shift > 1 ||
      rope_ld < head_dim)
    return ORL_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) & 15u) return ORL_ERR_ALIGN;
  if (n_rows == 0) return ORL_OK;
  const long long blocks = (n_rows * 32 + 255) / 256;
  rope_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), rows, n_rows,
                                                                      heads * head_dim, head_dim, cos_t, sin_t,
                                                                      rope_ld, sin_shift);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
