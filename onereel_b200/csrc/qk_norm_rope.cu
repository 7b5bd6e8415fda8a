// Fused q/k RMSNorm + rotary embedding, bf16 in / bf16 out, HBM-bound.
//
// Replaces the per-layer q/k preparation of the reference processors:
//   - Wan2.2 (src/onereel/models/wan.py:64-74 `_qk`, a torch.compile'd Triton kernel): RMSNorm over the whole hidden
//     dimension (H * D) with a learned weight, then the interleaved RoPE (cos[..., 0::2], sin[..., 1::2]);
//   - HunyuanVideo-1.5 (src/onereel/models/hunyuan15.py:187-190): RMSNorm per head (over D, weight [D]), then
//     diffusers' apply_rotary_emb over interleaved pairs (cos / sin repeated per pair).
// Both rotations are out[2i] = x[2i] c_i - x[2i+1] s_i, out[2i+1] = x[2i] s_i + x[2i+1] c_i with c_i = cos[row][2i]
// and s_i = sin[row][2i + sin_shift] (sin_shift 0 for the repeated tables, 1 for Wan's).
// One warp per (row, group): a group is one head (per-head norm) or the whole row (hidden norm); each lane holds
// 8-element chunks (16-byte loads), the sum of squares is reduced with warp shuffles in fp32, and the output is
// written to out_row_map[row] (or row) — i.e. straight into a packed layout when a row map is given.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "orl_common.h"

namespace orl {

template <int kChunksPerLane>
__global__ void qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                    const __nv_bfloat16* __restrict__ weight, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, long long rows, int heads, int head_dim,
                                    int per_head, float eps, int sin_shift, long long rope_ld,
                                    const int32_t* __restrict__ row_map, long long n_groups_per_row) {
  const long long warp_id = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long row = warp_id / n_groups_per_row;
  if (row >= rows) return;
  const int group = static_cast<int>(warp_id - row * n_groups_per_row);
  const int hidden = heads * head_dim;
  const int glen = per_head ? head_dim : hidden;        // elements normalised together
  const int gbase = group * glen;                        // first element of the group in the row
  const __nv_bfloat16* xr = x + row * hidden + gbase;
  float v[kChunksPerLane][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunksPerLane; ++c) {
    const int e = (c * 32 + lane) * 8;
    if (e < glen) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + e);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[c][2 * i] = f.x;
        v[c][2 * i + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / glen + eps);
  const long long orow = row_map ? row_map[row] : row;
  __nv_bfloat16* yr = y + orow * hidden + gbase;
  const float* cr = cos_t + row * rope_ld;
  const float* sr = sin_t + row * rope_ld;
#pragma unroll
  for (int c = 0; c < kChunksPerLane; ++c) {
    const int e = (c * 32 + lane) * 8;
    if (e >= glen) continue;
    uint4 packed;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int g = gbase + e + 2 * i;                   // element index in the row
      const int d = g % head_dim;                        // position within the head (pairs never straddle heads)
      const float w0 = __bfloat162float(weight[per_head ? d : g]);
      const float w1 = __bfloat162float(weight[per_head ? d + 1 : g + 1]);
      const float a = v[c][2 * i] * inv * w0, b = v[c][2 * i + 1] * inv * w1;
      const float cs = cr[d], sn = sr[d + sin_shift];
      o2[i] = __floats2bfloat162_rn(a * cs - b * sn, a * sn + b * cs);
    }
    *reinterpret_cast<uint4*>(yr + e) = packed;
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
  if (rows == 0) return ORL_OK;
  const int glen = per_head ? head_dim : heads * head_dim;
  const int chunks = (glen / 8 + 31) / 32;
  const long long groups = per_head ? heads : 1;
  const long long warps = rows * groups;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return ORL_ERR_ARG;
#define ORL_QKNR(N)                                                                                               \
  qk_norm_rope_kernel<N><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(                                 \
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y),                                       \
      static_cast<const __nv_bfloat16*>(weight), cos_t, sin_t, rows, heads, head_dim, per_head, eps, sin_shift,   \
      rope_ld, row_map, groups)
  if (chunks <= 1) ORL_QKNR(1);
  else if (chunks <= 2) ORL_QKNR(2);
  else if (chunks <= 4) ORL_QKNR(4);
  else if (chunks <= 8) ORL_QKNR(8);
  else if (chunks <= 16) ORL_QKNR(16);
  else return ORL_ERR_UNSUPPORTED;
#undef ORL_QKNR
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
