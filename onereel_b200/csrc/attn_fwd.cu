// Packed variable-length scene attention, forward, bf16 in / fp32 accumulate / bf16 out, for sm_100a.
//
// Replaces the FlashAttention varlen call of the reference (src/onereel/attention.py:39-53 `varlen` / `varlen_lse`,
// reached from `packed` / `packed_lse` at 56-71): for every segment i, rows cu_q[i]..cu_q[i+1] of q attend to rows
// cu_k[i]..cu_k[i+1] of k / v, non-causal, softmax scale `scale` (D^-0.5 by default), optional natural-log LSE [H, Nq].
//
// One CTA computes one work item = (segment, head, up to 256 query rows as two 128-row tiles):
//   warp 0      TMA producer: Q tiles once, then K_j / V_j tiles of 128 rows into a ring of shared-memory stages
//   warp 1      TMEM owner and MMA issuer (one elected thread): S_t = Q_t K_j^T (SS form), O_t += P_t V_j (TS form,
//               P read from TMEM in two 64-key halves), each committed to an mbarrier
//   warps 4-11  softmax, all eight on one tile at a time (tile 0, then tile 1, per 128-key step): a warp owns 16
//               TMEM lanes (query rows), a quad of threads one row, 32 of its 128 scores per thread. Loads S,
//               exponentiates against the running max while reducing the tile max (rescaling O in TMEM only when
//               the max jumps by more than 2^64), writes P (bf16) over the S columns, then normalises O and stores
//               the bf16 rows and their LSE.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+D), O1 [256+D,256+2D).
// Warpgroup 0 runs on kRegsLow registers per thread and the softmax warpgroups on kRegsHigh (setmaxnreg).
// Every mbarrier wait is bounded (ptx.cuh kWaitLimitNs): a stuck pipeline sets the error word and winds down.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "orl_common.h"
#include "ptx.cuh"

namespace orl {

template <int D>
struct AttnCfg {
  static constexpr int kChunks = D / 64;              // 128-byte swizzle columns per row
  static constexpr int kTileBytes = 128 * D * 2;      // one 128-row bf16 tile
  static constexpr int kChunkBytes = 128 * 128;       // one 128-row x 64-column chunk
  static constexpr int kStages = (D == 128) ? 2 : 4;  // K/V ring depth
  static constexpr int kQOff = 0;
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  // barriers: q_full, k_full[S], v_full[S], kv_empty[S], s_full[t], p_full[t][half], all_done, drain
  static constexpr int kBarQ = 0;
  static constexpr int kBarK = 1;
  static constexpr int kBarV = kBarK + kStages;
  static constexpr int kBarE = kBarV + kStages;
  static constexpr int kBarS = kBarE + kStages;      // + t
  static constexpr int kBarP = kBarS + 2;            // + 2 t + half
  static constexpr int kBarDone = kBarP + 4;
  static constexpr int kBarDrain = kBarDone + 1;
  static constexpr int kNumBars = kBarDrain + 1;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  // TMEM columns: S of tile t (128 fp32 columns; its P is 64 bf16x2 columns at the same start), O of tile t
  __host__ __device__ static constexpr uint32_t col_s(int t) { return 128u * t; }
  __host__ __device__ static constexpr uint32_t col_o(int t) { return 256u + D * t; }
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

constexpr int kThreads = 384;
constexpr int kMaxDevices = 64;
// register split: the launch has 384 threads x 168 registers; warpgroup 0 (producer, MMA issuer, two idle warps)
// keeps kRegsLow, the two softmax warpgroups get kRegsHigh (4 x 32 x kRegsLow + 8 x 32 x kRegsHigh = 384 x 168)
constexpr int kLaunchRegs = 168, kRegsLow = 120, kRegsHigh = 192;
static_assert(4 * kRegsLow + 8 * kRegsHigh == 12 * kLaunchRegs, "register split must add up to the launch total");
// The softmax exponentiates against the running max it already has and computes the tile's max alongside; only
// when a score exceeds that max by more than 2^kMaxJump (in exp2 units) is the tile redone against the new max and
// O rescaled. Below that, P <= 2^kMaxJump stays far inside bf16 / fp32 range and the final O / l is exact.
constexpr float kMaxJump = 64.0f;

__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* err) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrTimeoutDrain);
      return;
    }
  }
}

struct AttnShared {
  uint32_t sbase;        // shared-window address of the 1024-aligned tile area
  uint32_t bar0;         // address of barrier 0
  volatile int* abort_flag;
  __device__ uint32_t bar(int i) const { return bar0 + 8u * i; }
};

// ---------------------------------------------------------------------------------------------- TMA producer
template <int D>
__device__ __forceinline__ void producer_role(const AttnShared& sh, const CUtensorMap* tm_q, const CUtensorMap* tm_k,
                                              const CUtensorMap* tm_v, const AttnWork& wi, int n_qt, int n_kv,
                                              int* err) {
  using C = AttnCfg<D>;
  tma_prefetch_map(tm_q);
  tma_prefetch_map(tm_k);
  tma_prefetch_map(tm_v);
  const uint64_t pol_q = policy_evict_first();
  const uint64_t pol_kv = policy_evict_last();
  const int x0 = wi.head * D;
  mbar_expect_tx(sh.bar(C::kBarQ), n_qt * C::kTileBytes);
  for (int t = 0; t < n_qt; ++t)
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_2d(sh.sbase + C::kQOff + t * C::kTileBytes + c * C::kChunkBytes, tm_q, sh.bar(C::kBarQ), x0 + 64 * c,
                  wi.q_row0 + 128 * t, pol_q);
  int issued = 0;
  for (int j = 0; j < n_kv; ++j) {
    const int s = j % C::kStages;
    if (j >= C::kStages && !mbar_wait(sh.bar(C::kBarE + s), ((j / C::kStages) - 1) & 1, sh.abort_flag)) {
      atomicOr(err, kErrTimeoutLoad);
      break;
    }
    const int y = wi.k_row0 + 128 * j;
    mbar_expect_tx(sh.bar(C::kBarK + s), C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_2d(sh.sbase + C::kKOff + s * C::kTileBytes + c * C::kChunkBytes, tm_k, sh.bar(C::kBarK + s),
                  x0 + 64 * c, y, pol_kv);
    mbar_expect_tx(sh.bar(C::kBarV + s), C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_2d(sh.sbase + C::kVOff + s * C::kTileBytes + c * C::kChunkBytes, tm_v, sh.bar(C::kBarV + s),
                  x0 + 64 * c, y, pol_kv);
    issued = j + 1;
  }
  if (*sh.abort_flag) {
    // wind down: every copy this thread started must land before the CTA's shared memory is released
    drain_wait(sh.bar(C::kBarQ), 0, err);
    for (int j = issued > C::kStages ? issued - C::kStages : 0; j < issued; ++j) {
      const int s = j % C::kStages;
      drain_wait(sh.bar(C::kBarK + s), (j / C::kStages) & 1, err);
      drain_wait(sh.bar(C::kBarV + s), (j / C::kStages) & 1, err);
    }
  }
}

// ---------------------------------------------------------------------------------------------- MMA issuer
// Per 128-key tile j: S_t = Q_t K_j^T (both operands from shared memory) and O_t += P_t V_j (A = P from TMEM,
// B = V MN-major), P handed over in two 64-key halves so the PV of the first half starts while the softmax warps
// still exponentiate the second. Issue order: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1): the tensor pipe computes one
// tile while the softmax warps work on the other.
template <int D>
__device__ __forceinline__ void mma_role(const AttnShared& sh, uint32_t tmem, int n_qt, int n_kv, int* err) {
  using C = AttnCfg<D>;
  constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, D, false, true);
  auto issue_s = [&](int t, int s) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * C::kChunkBytes + (kk & 3) * 32;
      const uint64_t a = smem_desc_sw128(sh.sbase + C::kQOff + t * C::kTileBytes + off, 16, 1024);
      const uint64_t b = smem_desc_sw128(sh.sbase + C::kKOff + s * C::kTileBytes + off, 16, 1024);
      mma_ss(tmem + C::col_s(t), a, b, kIdescS, kk > 0 ? 1u : 0u);
    }
  };
  auto issue_o = [&](int t, int half, int s, bool acc) {
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      const int kk = 4 * half + k4;
      const uint64_t b = smem_desc_sw128(sh.sbase + C::kVOff + s * C::kTileBytes + kk * 2048, C::kChunkBytes, 1024);
      mma_ts(tmem + C::col_o(t), tmem + C::col_s(t) + kk * 8, b, kIdescO, (acc || kk > 0) ? 1u : 0u);
    }
  };
  bool ok = mbar_wait(sh.bar(C::kBarQ), 0, sh.abort_flag) && mbar_wait(sh.bar(C::kBarK), 0, sh.abort_flag);
  if (ok) {
    for (int t = 0; t < n_qt; ++t) {
      issue_s(t, 0);
      mma_commit(sh.bar(C::kBarS + t));
    }
  }
  for (int j = 0; ok && j < n_kv; ++j) {
    const int s = j % C::kStages;
    const int s2 = (j + 1) % C::kStages;
    const bool more = j + 1 < n_kv;
    bool k_next = false;                 // K of tile j + 1 waited for (lazily, before its first S)
    ok = mbar_wait(sh.bar(C::kBarV + s), (j / C::kStages) & 1, sh.abort_flag);
    for (int t = 0; ok && t < n_qt; ++t) {
      for (int half = 0; ok && half < 2; ++half) {
        ok = mbar_wait(sh.bar(C::kBarP + 2 * t + half), j & 1, sh.abort_flag);
        if (!ok) break;
        tc_fence_after();
        issue_o(t, half, s, j > 0);
      }
      if (!ok) break;
      if (t == n_qt - 1) mma_commit(sh.bar(C::kBarE + s));
      if (more) {
        if (!k_next) {
          ok = mbar_wait(sh.bar(C::kBarK + s2), ((j + 1) / C::kStages) & 1, sh.abort_flag);
          if (!ok) break;
          k_next = true;
        }
        issue_s(t, s2);
        mma_commit(sh.bar(C::kBarS + t));
      }
    }
  }
  if (ok) {
    mma_commit(sh.bar(C::kBarDone));
  } else {
    atomicOr(err, kErrTimeoutMma);
    mma_commit(sh.bar(C::kBarDrain));
    drain_wait(sh.bar(C::kBarDrain), 0, err);
  }
}

// ---------------------------------------------------------------------------------------------- softmax
__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
}

// All eight softmax warps work on one query tile at a time (tile 0, then tile 1, per 128-key step), so each tile's
// softmax — the link between its S MMA and its PV MMA — takes half as long as with one warpgroup per tile. Warp sw
// (0..7) owns TMEM lanes 32 (sw % 4) + 16 (sw / 4) + [0, 16); each thread holds two rows (lanes l/4, l/4 + 8 of that
// block) and 32 of their 128 scores, a quad of threads shares a row (row max by two shuffles; row sums stay per
// thread until the end). Per 128-key tile: exponentiate against the running max while reducing the tile's max
// alongside (the first tile takes its max first); if the tile's max exceeds the running one by more than kMaxJump
// (exp2 units) the rows are redone against the new max and their O rescaled in TMEM (PV of the previous tile has
// completed: S of this tile was issued after it). P (bf16) goes over the S columns in two 64-key halves, each handed
// to the MMA warp as soon as all eight warps stored it.
template <int D>
__device__ __forceinline__ void softmax_role(const AttnShared& sh, uint32_t tmem, int sw, int lane,
                                             const AttnWork& wi, int n_qt, int n_kv, float scale_log2,
                                             __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                                             long long nq_total, int heads, int* err) {
  using C = AttnCfg<D>;
  const int cq = lane & 3;
  const int lrow = 32 * (sw & 3) + 16 * (sw >> 2) + (lane >> 2);     // tile row of the first of the two rows
  const uint32_t lane_off = static_cast<uint32_t>(32 * (sw & 3) + 16 * (sw >> 2)) << 16;
  float m_run[2][2] = {{-INFINITY, -INFINITY}, {-INFINITY, -INFINITY}};
  float l_run[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  bool ok = n_kv > 0;
  // One tile's softmax on the scores sv (already loaded and waited for): mask, max, exponentials, P in two halves.
  // Everything up to the store of P's second half; finish_tile then waits for that store and hands it over.
  struct TileState {
    float m0, m1, l0, l1;
  };
  auto tile_front = [&](int j, int t, int valid, uint32_t (&sv)[64], uint32_t (&pb)[16]) -> TileState {
    const uint32_t s_addr = tmem + C::col_s(t) + lane_off;
    if (valid < 128) {
#pragma unroll
      for (int r = 0; r < 16; ++r)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (8 * r + 2 * cq + (k & 1) >= valid) sv[4 * r + k] = __float_as_uint(-INFINITY);
    }
    auto tile_max = [&](int i) {
      float a = __uint_as_float(sv[2 * i]), b = __uint_as_float(sv[2 * i + 1]);
#pragma unroll
      for (int r = 1; r < 16; r += 2) {
        a = fmax3(a, __uint_as_float(sv[4 * r + 2 * i]), __uint_as_float(sv[4 * r + 2 * i + 1]));
        if (r + 1 < 16) b = fmax3(b, __uint_as_float(sv[4 * (r + 1) + 2 * i]), __uint_as_float(sv[4 * (r + 1) + 2 * i + 1]));
      }
      return quad_max(fmaxf(a, b));
    };
    // exponentials of keys [64 h, 64 h + 64) of both rows against neg_i = -m_i * log2e * scale: P words for a
    // 16x128b store (register 2r + i: row i, word 4r + cq) and the two rows' sums, each row's two keys summed as
    // one f32x2 pair (half the add instructions)
    auto exp_half = [&](int h, float neg0, float neg1, uint32_t (&p)[16], float& sum0, float& sum1) {
      F2 acc0 = f2(0.f, 0.f), acc1 = f2(0.f, 0.f);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int base = 4 * (8 * h + r);
        const float x0 = ex2(fmaf(__uint_as_float(sv[base + 0]), scale_log2, neg0));
        const float x1 = ex2(fmaf(__uint_as_float(sv[base + 1]), scale_log2, neg0));
        const float y0 = ex2(fmaf(__uint_as_float(sv[base + 2]), scale_log2, neg1));
        const float y1 = ex2(fmaf(__uint_as_float(sv[base + 3]), scale_log2, neg1));
        acc0 = fadd2(acc0, f2(x0, x1));
        acc1 = fadd2(acc1, f2(y0, y1));
        p[2 * r + 0] = pack_bf16x2(x0, x1);
        p[2 * r + 1] = pack_bf16x2(y0, y1);
      }
      const float2 u0 = f2_split(acc0), u1 = f2_split(acc1);
      sum0 = u0.x + u0.y;
      sum1 = u1.x + u1.y;
    };
    float* mr = m_run[t];
    float* lr = l_run[t];
    float m_use0 = mr[0], m_use1 = mr[1];
    uint32_t pa[16];
    float sa0, sa1;
    if (j == 0) {
      m_use0 = tile_max(0);
      m_use1 = tile_max(1);
      exp_half(0, -m_use0 * scale_log2, -m_use1 * scale_log2, pa, sa0, sa1);
    } else {
      exp_half(0, -mr[0] * scale_log2, -mr[1] * scale_log2, pa, sa0, sa1);   // speculative
      const float mx0 = tile_max(0), mx1 = tile_max(1);
      const bool redo0 = (mx0 - mr[0]) * scale_log2 > kMaxJump, redo1 = (mx1 - mr[1]) * scale_log2 > kMaxJump;
      if (__any_sync(0xffffffffu, redo0 || redo1)) {
        // the warp redoes its tile together (TMEM loads and stores are warp-wide), but only rows whose max jumped
        // take the new max: the others keep theirs (factor exactly 1, P unchanged), so a row's result never
        // depends on which rows share its warp or work item
        m_use0 = redo0 ? fmaxf(mr[0], mx0) : mr[0];
        m_use1 = redo1 ? fmaxf(mr[1], mx1) : mr[1];
        const float al0 = redo0 ? ex2((mr[0] - m_use0) * scale_log2) : 1.0f;
        const float al1 = redo1 ? ex2((mr[1] - m_use1) * scale_log2) : 1.0f;
        exp_half(0, -m_use0 * scale_log2, -m_use1 * scale_log2, pa, sa0, sa1);
        lr[0] *= al0;
        lr[1] *= al1;
        const uint32_t o_addr = tmem + C::col_o(t) + lane_off;
#pragma unroll
        for (int ch = 0; ch < D / 64; ++ch) {
          uint32_t o[32];
          tmem_ld_16x256b_x8(o_addr + 64 * ch, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * ((e & 2) ? al1 : al0));
          tmem_st_16x256b_x8(o_addr + 64 * ch, o);
        }
      }
    }
    tmem_st_16x128b_x8(s_addr, pa);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(sh.bar(C::kBarP + 2 * t + 0));
    float sb0, sb1;
    exp_half(1, -m_use0 * scale_log2, -m_use1 * scale_log2, pb, sb0, sb1);
    tmem_st_16x128b_x8(s_addr + 32, pb);
    return TileState{m_use0, m_use1, sa0 + sb0, sa1 + sb1};
  };
  auto tile_back = [&](int t, const TileState& st) {
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(sh.bar(C::kBarP + 2 * t + 1));
    l_run[t][0] += st.l0;
    l_run[t][1] += st.l1;
    m_run[t][0] = st.m0;
    m_run[t][1] = st.m1;
  };
  auto load_s = [&](int t, uint32_t (&sv)[64]) {
    const uint32_t s_addr = tmem + C::col_s(t) + lane_off;
    tmem_ld_16x256b_x8(s_addr, sv);
    tmem_ld_16x256b_x8(s_addr + 64, sv + 32);
  };
  uint32_t s[64], s2[64];                      // s[4r + 2i + e]: row i, key 8r + 2 cq + e
  uint32_t pb[16];
  for (int j = 0; ok && j < n_kv; ++j) {
    const int valid = wi.k_len - 128 * j;
    ok = mbar_wait(sh.bar(C::kBarS + 0), j & 1, sh.abort_flag);
    if (!ok) break;
    tc_fence_after();
    load_s(0, s);
    tmem_wait_ld();
    const TileState st0 = tile_front(j, 0, valid, s, pb);
    tile_back(0, st0);
    if (n_qt == 2) {
      ok = mbar_wait(sh.bar(C::kBarS + 1), j & 1, sh.abort_flag);
      if (!ok) break;
      tc_fence_after();
      load_s(1, s2);
      tmem_wait_ld();
      const TileState st1 = tile_front(j, 1, valid, s2, pb);
      tile_back(1, st1);
    }
  }
  if (ok) ok = mbar_wait(sh.bar(C::kBarDone), 0, sh.abort_flag);
  if (ok) {
    tc_fence_after();
    for (int t = 0; t < n_qt; ++t) {
      const float l0 = quad_sum(l_run[t][0]), l1 = quad_sum(l_run[t][1]);
      const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
      const int r0 = 128 * t + lrow, r1 = r0 + 8;
      const bool v0 = r0 < wi.q_len, v1 = r1 < wi.q_len;
      __nv_bfloat16* o0 = out + (static_cast<long long>(wi.q_row0) + r0) * heads * D + wi.head * D + 2 * cq;
      __nv_bfloat16* o1 = o0 + 8ll * heads * D;
      const uint32_t o_addr = tmem + C::col_o(t) + lane_off;
#pragma unroll
      for (int ch = 0; ch < D / 64; ++ch) {
        uint32_t o[32];
        tmem_ld_16x256b_x8(o_addr + 64 * ch, o);
        tmem_wait_ld();
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int col = 64 * ch + 8 * r;
          if (v0)
            *reinterpret_cast<uint32_t*>(o0 + col) =
                pack_bf16x2(__uint_as_float(o[4 * r + 0]) * inv0, __uint_as_float(o[4 * r + 1]) * inv0);
          if (v1)
            *reinterpret_cast<uint32_t*>(o1 + col) =
                pack_bf16x2(__uint_as_float(o[4 * r + 2]) * inv1, __uint_as_float(o[4 * r + 3]) * inv1);
        }
      }
      if (lse != nullptr && cq == 0) {
        const long long lb = static_cast<long long>(wi.head) * nq_total + wi.q_row0;
        if (v0) lse[lb + r0] = (m_run[t][0] * scale_log2 + lg2(l0)) * 0.69314718055994530942f;
        if (v1) lse[lb + r1] = (m_run[t][1] * scale_log2 + lg2(l1)) * 0.69314718055994530942f;
      }
    }
  } else if (n_kv > 0) {
    atomicOr(err, kErrTimeoutSoftmax);
  } else {
    // a segment without keys: zero output, LSE -inf
    for (int t = 0; t < n_qt; ++t) {
      const int r0 = 128 * t + lrow;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rr = r0 + 8 * i;
        if (rr >= wi.q_len) continue;
        __nv_bfloat16* orow = out + (static_cast<long long>(wi.q_row0) + rr) * heads * D + wi.head * D + 2 * cq;
        for (int col = 0; col < D; col += 8) *reinterpret_cast<uint32_t*>(orow + col) = 0u;
        if (lse != nullptr && cq == 0) lse[static_cast<long long>(wi.head) * nq_total + wi.q_row0 + rr] = -INFINITY;
      }
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnWork* __restrict__ work,
                    __nv_bfloat16* __restrict__ out, float* __restrict__ lse, long long nq_total, int heads,
                    float scale_log2, int* __restrict__ err, const int* __restrict__ n_items_dev) {
  using C = AttnCfg<D>;
  // a grid sized by an upper bound (work list planned on the device): CTAs past the planned count have no item
  if (n_items_dev != nullptr && static_cast<int>(blockIdx.x) >= __ldg(n_items_dev)) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + C::kNumBars * 8);
  AttnShared sh;
  sh.sbase = smem_u32(smem);
  sh.bar0 = sh.sbase + C::kBarOff;
  sh.abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AttnWork wi = work[blockIdx.x];
  const int n_qt = wi.q_len > 128 ? 2 : 1;
  const int n_kv = (wi.k_len + 127) >> 7;

  if (threadIdx.x == 0) {
    mbar_init(sh.bar(C::kBarQ), 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(sh.bar(C::kBarK + s), 1);
      mbar_init(sh.bar(C::kBarV + s), 1);
      mbar_init(sh.bar(C::kBarE + s), 1);
    }
    for (int t = 0; t < 2; ++t) mbar_init(sh.bar(C::kBarS + t), 1);
    for (int i = 0; i < 4; ++i) mbar_init(sh.bar(C::kBarP + i), 256);
    mbar_init(sh.bar(C::kBarDone), 1);
    mbar_init(sh.bar(C::kBarDrain), 1);
    *sh.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // warpgroup 0 returns registers at one program point (all four warps), then splits into its roles
    regs_dec<kRegsLow>();
    if (warp == 0) {
      if (elect_one() && n_kv > 0) producer_role<D>(sh, &tm_q, &tm_k, &tm_v, wi, n_qt, n_kv, err);
    } else if (warp == 1) {
      if (elect_one() && n_kv > 0) mma_role<D>(sh, tmem, n_qt, n_kv, err);
    }
  } else {
    regs_inc<kRegsHigh>();
    softmax_role<D>(sh, tmem, warp - 4, lane, wi, n_qt, n_kv, scale_log2, out, lse, nq_total, heads, err);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------ host side

// cuTensorMapEncodeTiled (driver API, cuda.h), fetched through the runtime so the library needs no -lcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 map over rows x (heads * D) with 128-row x 64-column boxes, 128-byte swizzle, zero fill out of bounds.
static int make_rows_map(CUtensorMap* map, const void* base, long long rows, int row_elems) {
  auto fn = encode_fn();
  if (fn == nullptr) return ORL_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_elems), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_elems) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ORL_OK : ORL_ERR_TENSOR_MAP;
}

template <int D>
static int launch_attn(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                       long long nk, int heads, float scale, const AttnWork* work, int n_items, int* err,
                       cudaStream_t stream, const int* n_items_dev = nullptr) {
  using C = AttnCfg<D>;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_rows_map(&mq, q, nq, heads * D)) != ORL_OK) return rc;
  if ((rc = make_rows_map(&mk, k, nk, heads * D)) != ORL_OK) return rc;
  if ((rc = make_rows_map(&mv, v, nk, heads * D)) != ORL_OK) return rc;
  // the shared-memory opt-in is a per-device attribute: set once for every device the kernel runs on
  static std::mutex mu;
  static bool attr_set[kMaxDevices] = {};
  static int launch_regs = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ORL_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      if (cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
          cudaSuccess)
        return ORL_ERR_LAUNCH;
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, attn_fwd_kernel<D>) != cudaSuccess) return ORL_ERR_LAUNCH;
      launch_regs = fa.numRegs;
      attr_set[dev] = true;
    }
  }
  // the setmaxnreg split assumes exactly kLaunchRegs registers per thread at launch; any other count could leave
  // the increasing warpgroups waiting for registers that were never freed, so such a build is never launched
  if (launch_regs != kLaunchRegs) return ORL_ERR_UNSUPPORTED;
  const float scale_log2 = scale * 1.4426950408889634f;
  attn_fwd_kernel<D><<<n_items, kThreads, C::kSmemBytes, stream>>>(
      mq, mk, mv, work, static_cast<__nv_bfloat16*>(out), lse, nq, heads, scale_log2, err, n_items_dev);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}

}  // namespace orl

using namespace orl;

extern "C" int orl_attn_plan_ranges(const int32_t* q_start, const int32_t* q_len, const int32_t* k_start,
                                    const int32_t* k_len, int n_seg, int heads, AttnWork* work, int capacity) {
  if (q_start == nullptr || q_len == nullptr || k_start == nullptr || k_len == nullptr || n_seg < 0 || heads <= 0)
    return ORL_ERR_ARG;
  std::vector<int> order;
  long long need = 0;
  for (int i = 0; i < n_seg; ++i) {
    if (q_len[i] < 0 || k_len[i] < 0 || q_start[i] < 0 || k_start[i] < 0) return ORL_ERR_ARG;
    if (q_len[i] == 0) continue;
    order.push_back(i);
    need += static_cast<long long>(heads) * ((q_len[i] + 255) / 256);
  }
  if (need > 0x3fffffff) return ORL_ERR_ARG;
  if (work == nullptr || capacity < need) return -static_cast<int>(need) - 1000;   // caller sizes the buffer
  // longest key range first (largest items first), items of one (segment, head) adjacent so their K/V share L2
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return k_len[a] > k_len[b]; });
  int n = 0;
  for (int i : order)
    for (int h = 0; h < heads; ++h)
      for (int p = 0; p < q_len[i]; p += 256) {
        AttnWork w;
        w.q_row0 = q_start[i] + p;
        w.q_len = std::min(256, q_len[i] - p);
        w.k_row0 = k_start[i];
        w.k_len = k_len[i];
        w.head = h;
        w.seg = i;
        w.pad0 = w.pad1 = 0;
        work[n++] = w;
      }
  return n;
}

extern "C" int orl_attn_plan(const int32_t* cu_q, const int32_t* cu_k, int n_seg, int heads, AttnWork* work,
                             int capacity) {
  if (cu_q == nullptr || cu_k == nullptr || n_seg < 0) return ORL_ERR_ARG;
  std::vector<int32_t> qs(n_seg), ql(n_seg), ks(n_seg), kl(n_seg);
  for (int i = 0; i < n_seg; ++i) {
    qs[i] = cu_q[i];
    ql[i] = cu_q[i + 1] - cu_q[i];
    ks[i] = cu_k[i];
    kl[i] = cu_k[i + 1] - cu_k[i];
  }
  return orl_attn_plan_ranges(qs.data(), ql.data(), ks.data(), kl.data(), n_seg, heads, work, capacity);
}

extern "C" int orl_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                            long long nk, int heads, int head_dim, float scale, const AttnWork* work_dev,
                            int n_items, int* err_dev, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || work_dev == nullptr || err_dev == nullptr)
    return ORL_ERR_ARG;
  if (nq < 0 || nk < 0 || heads <= 0 || n_items < 0 || !(scale > 0.f)) return ORL_ERR_ARG;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
    return ORL_ERR_ALIGN;
  if (n_items == 0 || nq == 0) return ORL_OK;
  if (nk == 0) {   // every item has k_len 0 and loads nothing; the K/V maps only need a valid address
    k = v = q;
    nk = nq;
  }
  switch (head_dim) {
    case 64:
      return launch_attn<64>(q, k, v, out, lse, nq, nk, heads, scale, work_dev, n_items, err_dev, stream);
    case 128:
      return launch_attn<128>(q, k, v, out, lse, nq, nk, heads, scale, work_dev, n_items, err_dev, stream);
    default:
      return ORL_ERR_UNSUPPORTED;
  }
}

// ------------------------------------------------------------------------------------------------ device plan
// orl_attn_fwd_cu: the varlen call with cu_seqlens already on the device (the reference hands FlashAttention device
// tensors, attention.py:28-29, 39-43) — the work list is planned on the device, so the call never waits for the GPU.
// One block reads cu_q / cu_k, checks them (non-decreasing, inside [0, nq] / [0, nk]), orders the segments with query
// rows by key count, descending and stable — the order orl_attn_plan_ranges uses, so the items and the results are
// identical — and writes the item count into slot 0 of the work buffer and the items after it. The attention grid is
// sized by the upper bound heads x (ceil(nq / 256) + n_seg); CTAs past the planned count return at once.
namespace orl {

constexpr int kDevPlanMaxSeg = 4096;

__global__ void __launch_bounds__(1024) plan_device_kernel(const int32_t* __restrict__ cu_q,
                                                           const int32_t* __restrict__ cu_k, int n_seg, int heads,
                                                           long long nq, long long nk, AttnWork* __restrict__ work,
                                                           long long capacity, int* __restrict__ err) {
  extern __shared__ int plan_smem[];
  int* s_lq = plan_smem;                    // [n_seg] query rows
  int* s_lk = s_lq + n_seg;                 // [n_seg] key rows
  int* s_seg = s_lk + n_seg;                // [n_seg] segment at each rank (ranks of segments with query rows)
  int* s_end = s_seg + n_seg;               // [n_seg] end of each rank's items (inclusive scan in rank order)
  __shared__ int bad, n_ranked, total;
  const int t = threadIdx.x;
  if (t == 0) {
    bad = 0;
    n_ranked = 0;
    total = 0;
  }
  __syncthreads();
  for (int i = t; i < n_seg; i += blockDim.x) {
    const long long q0 = cu_q[i], q1 = cu_q[i + 1], k0 = cu_k[i], k1 = cu_k[i + 1];
    if (q0 < 0 || q1 < q0 || q1 > nq || k0 < 0 || k1 < k0 || k1 > nk) bad = 1;
    s_lq[i] = static_cast<int>(q1 - q0);
    s_lk[i] = static_cast<int>(k1 - k0);
  }
  __syncthreads();
  if (bad) {
    if (t == 0) {
      work[0].q_row0 = 0;
      atomicOr(err, kErrPlan);
    }
    return;
  }
  // rank of segment i among the segments with query rows: more keys first, then the lower index; its items start
  // after those of every segment ranked before it
  for (int i = t; i < n_seg; i += blockDim.x) {
    const int lq = s_lq[i], lk = s_lk[i];
    if (lq == 0) continue;
    int rank = 0;
    long long before = 0;
    for (int j = 0; j < n_seg; ++j) {
      const int lqj = s_lq[j], lkj = s_lk[j];
      if (lqj > 0 && (lkj > lk || (lkj == lk && j < i))) {
        ++rank;
        before += static_cast<long long>(heads) * ((lqj + 255) >> 8);
      }
    }
    const long long cnt = static_cast<long long>(heads) * ((lq + 255) >> 8);
    s_seg[rank] = i;
    s_end[rank] = static_cast<int>(before + cnt);
    atomicAdd(&n_ranked, 1);
    atomicAdd(&total, static_cast<int>(cnt));
  }
  __syncthreads();
  const int n = total, m = n_ranked;
  if (static_cast<long long>(n) + 1 > capacity) {
    if (t == 0) {
      work[0].q_row0 = 0;
      atomicOr(err, kErrPlan);
    }
    return;
  }
  for (int it = t; it < n; it += blockDim.x) {
    int lo = 0, hi = m - 1;                 // first rank whose items end after it
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (s_end[mid] > it) hi = mid; else lo = mid + 1;
    }
    const int i = s_seg[lo];
    const int lq = s_lq[i];
    const int chunks = (lq + 255) >> 8;
    const int r = it - (lo > 0 ? s_end[lo - 1] : 0);
    const int h = r / chunks, c = r - h * chunks;
    AttnWork w;
    w.q_row0 = cu_q[i] + 256 * c;
    w.q_len = min(256, lq - 256 * c);
    w.k_row0 = cu_k[i];
    w.k_len = s_lk[i];
    w.head = h;
    w.seg = i;
    w.pad0 = w.pad1 = 0;
    work[1 + it] = w;
  }
  if (t == 0) work[0].q_row0 = n;
}

}  // namespace orl

extern "C" long long orl_attn_fwd_cu_capacity(long long nq, int n_seg, int heads) {
  if (nq < 0 || n_seg < 0 || heads <= 0) return ORL_ERR_ARG;
  return 1 + static_cast<long long>(heads) * ((nq + 255) / 256 + n_seg);
}

extern "C" int orl_attn_fwd_cu(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                               long long nk, int heads, int head_dim, float scale, const int32_t* cu_q_dev,
                               const int32_t* cu_k_dev, int n_seg, orl_attn_work* work_dev, long long work_capacity,
                               int* err_dev, void* stream_ptr) {
  using namespace orl;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || cu_q_dev == nullptr || cu_k_dev == nullptr ||
      work_dev == nullptr || err_dev == nullptr)
    return ORL_ERR_ARG;
  if (nq < 0 || nk < 0 || heads <= 0 || n_seg < 0 || !(scale > 0.f)) return ORL_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return ORL_ERR_UNSUPPORTED;
  if (n_seg > kDevPlanMaxSeg) return ORL_ERR_CAPACITY;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
    return ORL_ERR_ALIGN;
  const long long bound = orl_attn_fwd_cu_capacity(nq, n_seg, heads);
  if (work_capacity < bound) return ORL_ERR_CAPACITY;
  if (bound - 1 > 0x7fffffffLL) return ORL_ERR_ARG;
  if (n_seg == 0 || nq == 0) return ORL_OK;
  const int smem = 16 * n_seg;
  static std::mutex mu;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ORL_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      if (cudaFuncSetAttribute(plan_device_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               16 * kDevPlanMaxSeg) != cudaSuccess)
        return ORL_ERR_LAUNCH;
      attr_set[dev] = true;
    }
  }
  plan_device_kernel<<<1, 1024, smem, stream>>>(cu_q_dev, cu_k_dev, n_seg, heads, nq, nk, work_dev, work_capacity,
                                                err_dev);
  if (cudaGetLastError() != cudaSuccess) return ORL_ERR_LAUNCH;
  const void* kk = k;
  const void* vv = v;
  long long nkk = nk;
  if (nk == 0) {   // every item has k_len 0 and loads nothing; the K/V maps only need a valid address
    kk = vv = q;
    nkk = nq;
  }
  const int grid = static_cast<int>(bound - 1);
  const int* count = reinterpret_cast<const int*>(work_dev);   // slot 0: the planned item count
  return head_dim == 64
             ? launch_attn<64>(q, kk, vv, out, lse, nq, nkk, heads, scale, work_dev + 1, grid, err_dev, stream, count)
             : launch_attn<128>(q, kk, vv, out, lse, nq, nkk, heads, scale, work_dev + 1, grid, err_dev, stream, count);
}

// ------------------------------------------------------------------------------------------------ allocation-free
// orl_attn_fwd_noalloc serves callers that cannot call cudaMalloc at all — code running where the CUDA allocator
// is off limits (inside another framework's memory pool or a custom allocator hook, in a plugin host that owns
// device memory, or in a process whose allocations are accounted elsewhere) and therefore cannot provide the work
// list and error word that orl_attn_fwd takes as caller scratch. This variant keeps that scratch in the file-scope
// array below instead: every GPU that loads the library holds it (kNoAllocScratchBytes, about 512 KiB) until the
// process exits. Its limits: at most kNoAllocMaxSegments segments and kNoAllocMaxItems work items (one item = one
// head x up to 256 query rows of one segment); larger calls are rejected with ORL_ERR_CAPACITY before any work.
//
// The host orders the segments (the schedule of orl_attn_plan) into a table that travels as a kernel parameter;
// a one-block kernel expands it into the work list inside the array and clears the error word, then the attention
// kernel runs on it. No host buffer is read after the call returns. Every call shares the array and it keeps the
// last call's contents; calls whose kernels overlap on one GPU (issued on two streams, or from two host threads)
// race on it, so callers serialise their calls per device; calls on different GPUs do not interact (each GPU has
// its own copy). The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that
// device current) and caches it per device ordinal; make that first call before any stream capture. The cached
// address does not survive cudaDeviceReset (the module, and with it the array, is loaded anew).
namespace orl {

constexpr int kNoAllocMaxItems = 16384;
constexpr int kNoAllocMaxSegments = 1024;
constexpr int kNoAllocHeaderBytes = 256;   // error word at offset 0, work items from offset 256
constexpr int kNoAllocScratchBytes = kNoAllocHeaderBytes + kNoAllocMaxItems * static_cast<int>(sizeof(AttnWork));
constexpr int kNoAllocMaxDevices = kMaxDevices;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// the ordered segment table, passed by value as the expand kernel's parameter (about 20 KiB, inside the 32 KiB
// kernel-parameter limit of sm_70 and later)
struct NoAllocTable {
  int n_seg;                          // segments with query rows, in schedule order
  int heads;
  int n_items;
  int pad;
  int4 seg[kNoAllocMaxSegments];      // (q_row0, q_len, k_row0, k_len)
  int index[kNoAllocMaxSegments];     // the segment's position in the caller's cu_seqlens
};
static_assert(sizeof(NoAllocTable) < 32000, "kernel parameter limit");

// One block: item counts per segment, an inclusive scan in shared memory, then every item written by one thread
// (item i -> its segment by binary search over the scan). Items of one segment: head-major, 256-row chunks inside.
__global__ void __launch_bounds__(1024) noalloc_expand_kernel(const __grid_constant__ NoAllocTable tab,
                                                              AttnWork* __restrict__ work, int* __restrict__ err) {
  __shared__ int end[kNoAllocMaxSegments];
  const int t = threadIdx.x;
  if (t == 0) *err = 0;
  int cnt = 0;
  if (t < tab.n_seg) cnt = tab.heads * ((tab.seg[t].y + 255) >> 8);
  end[t] = cnt;
  __syncthreads();
  for (int d = 1; d < kNoAllocMaxSegments; d <<= 1) {
    const int add = t >= d ? end[t - d] : 0;
    __syncthreads();
    end[t] += add;
    __syncthreads();
  }
  for (int i = t; i < tab.n_items; i += blockDim.x) {
    int lo = 0, hi = tab.n_seg - 1;            // first segment whose scan end exceeds i
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (end[mid] > i) hi = mid; else lo = mid + 1;
    }
    const int4 sg = tab.seg[lo];
    const int r = i - (lo > 0 ? end[lo - 1] : 0);
    const int chunks = (sg.y + 255) >> 8;
    const int h = r / chunks, c = r - h * chunks;
    AttnWork w;
    w.q_row0 = sg.x + 256 * c;
    w.q_len = min(256, sg.y - 256 * c);
    w.k_row0 = sg.z;
    w.k_len = sg.w;
    w.head = h;
    w.seg = tab.index[lo];
    w.pad0 = w.pad1 = 0;
    work[i] = w;
  }
}

static std::mutex g_noalloc_mutex;
static unsigned char* g_noalloc_dev[kNoAllocMaxDevices];        // device address of the array, per device ordinal

// cuStreamGetDevice from the driver (CUDA 12.8 and later), fetched through the runtime; null when absent
using StreamDeviceFn = CUresult (*)(CUstream, CUdevice*);
static StreamDeviceFn stream_device_fn() {
  static StreamDeviceFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamGetDevice", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<StreamDeviceFn>(p);
  });
  return fn;
}

// device memory (or managed memory) on device `dev`
static bool on_device(const void* p, int dev) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

}  // namespace orl

extern "C" int orl_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                                    long long nk, int heads, int head_dim, float scale, const int32_t* cu_q_host,
                                    const int32_t* cu_k_host, int n_seg, int* status_host, void* stream_ptr) {
  using namespace orl;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || cu_q_host == nullptr || cu_k_host == nullptr)
    return ORL_ERR_ARG;
  if (nq < 0 || nk < 0 || heads <= 0 || n_seg < 0 || !(scale > 0.f)) return ORL_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return ORL_ERR_UNSUPPORTED;
  if (n_seg > kNoAllocMaxSegments) return ORL_ERR_CAPACITY;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
    return ORL_ERR_ALIGN;
  // validate the segments and count the work items before touching any device state
  long long items = 0;
  if (cu_q_host[0] < 0 || cu_k_host[0] < 0) return ORL_ERR_ARG;
  for (int i = 0; i < n_seg; ++i) {
    const long long lq = static_cast<long long>(cu_q_host[i + 1]) - cu_q_host[i];
    const long long lk = static_cast<long long>(cu_k_host[i + 1]) - cu_k_host[i];
    if (lq < 0 || lk < 0) return ORL_ERR_ARG;
    items += static_cast<long long>(heads) * ((lq + 255) / 256);
  }
  if (n_seg > 0 && (cu_q_host[n_seg] > nq || cu_k_host[n_seg] > nk)) return ORL_ERR_ARG;
  if (items > kNoAllocMaxItems) return ORL_ERR_CAPACITY;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return ORL_ERR_LAUNCH;
  // the array's address below belongs to the current device: the tensors and the stream must live there too
  if (items > 0 && nq > 0) {
    if (!on_device(q, dev) || !on_device(out, dev) || (nk > 0 && (!on_device(k, dev) || !on_device(v, dev))) ||
        (lse != nullptr && !on_device(lse, dev)))
      return ORL_ERR_ARG;
  }
  if (auto fn = stream_device_fn()) {
    CUdevice sd = -1;
    if (fn(reinterpret_cast<CUstream>(stream), &sd) == CUDA_SUCCESS && static_cast<int>(sd) != dev)
      return ORL_ERR_ARG;
  }

  // the schedule of orl_attn_plan: segments with query rows by key count, descending (stable insertion sort)
  NoAllocTable tab;
  tab.n_seg = 0;
  tab.heads = heads;
  tab.n_items = static_cast<int>(items);
  tab.pad = 0;
  for (int i = 0; i < n_seg; ++i) {
    const int lq = cu_q_host[i + 1] - cu_q_host[i];
    if (lq == 0) continue;
    const int lk = cu_k_host[i + 1] - cu_k_host[i];
    int pos = tab.n_seg++;
    while (pos > 0 && tab.seg[pos - 1].w < lk) {
      tab.seg[pos] = tab.seg[pos - 1];
      tab.index[pos] = tab.index[pos - 1];
      --pos;
    }
    tab.seg[pos] = make_int4(cu_q_host[i], lq, cu_k_host[i], lk);
    tab.index[pos] = i;
  }

  unsigned char* scratch;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_dev[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return ORL_ERR_LAUNCH;
      g_noalloc_dev[dev] = static_cast<unsigned char*>(p);
    }
    scratch = g_noalloc_dev[dev];
  }
  int* err_dev = reinterpret_cast<int*>(scratch);
  AttnWork* work_dev = reinterpret_cast<AttnWork*>(scratch + kNoAllocHeaderBytes);

  // clears the error word and writes the work list (also when there is no work, so status reads 0)
  noalloc_expand_kernel<<<1, 1024, 0, stream>>>(tab, work_dev, err_dev);
  if (cudaGetLastError() != cudaSuccess) return ORL_ERR_LAUNCH;
  int rc = ORL_OK;
  if (items > 0 && nq > 0) {
    const void* kk = k;
    const void* vv = v;
    long long nkk = nk;
    if (nk == 0) {   // every item has k_len 0 and loads nothing; the K/V maps only need a valid address
      kk = vv = q;
      nkk = nq;
    }
    const int n = static_cast<int>(items);
    rc = head_dim == 64 ? launch_attn<64>(q, kk, vv, out, lse, nq, nkk, heads, scale, work_dev, n, err_dev, stream)
                        : launch_attn<128>(q, kk, vv, out, lse, nq, nkk, heads, scale, work_dev, n, err_dev, stream);
    if (rc != ORL_OK) return rc;
  }
  if (status_host != nullptr) {
    if (cudaMemcpyAsync(status_host, err_dev, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return ORL_ERR_LAUNCH;
  }
  return rc;
}
