/* onereel_b200 — C ABI of the B200-native scene-packed attention path.
 *
 * A drop-in for the device work of OneReel's scene attention (reference repository UIUC-MLSys/OneReel):
 *   - orl_attn_plan / orl_attn_fwd replace the FlashAttention varlen call of src/onereel/attention.py:39-53
 *     (`varlen`, `varlen_lse`), which `packed` / `packed_lse` (attention.py:56-71) and the scene processors
 *     (src/onereel/models/hunyuan15.py:212-303, src/onereel/models/wan.py:110-152) reach;
 *   - orl_pack replaces the torch.cat row copies that assemble every packed segment's q / k / v
 *     (attention.py:60-61, 69; hunyuan15.py:164, 168, 225; comm.py:200 `HaloExchange.rows`) and the output
 *     scatter back to token rows (hunyuan15.py:231-235, wan.py:117-118), and emits cu_seqlens (attention.py:28-29);
 *   - orl_lse_merge replaces the log-sum-exp merge of two partial results (hunyuan15.py:274-276, ring.py:63-70);
 *   - the planner entry points restate comm.py:18-112 (Algorithm 1, exchange sets, Eq. 2) natively.
 *
 * Conventions: device pointers are CUDA global memory on the current device; `stream` is a cudaStream_t (NULL =
 * legacy default stream). Every entry point returns 0 (ORL_OK) or a negative ORL_ERR_* code and never throws.
 * No entry point allocates device memory; scratch (work lists, error words) is passed in by the caller.
 * Tensors are row-major: q [nq, heads, head_dim], k / v [nk, heads, head_dim], bf16, rows contiguous.
 */
#ifndef ONEREEL_B200_H
#define ONEREEL_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define ORL_API __attribute__((visibility("default")))
#else
#define ORL_API
#endif

#define ORL_OK 0
#define ORL_ERR_ARG (-1)          /* invalid argument (null pointer, negative size, inconsistent cu_seqlens) */
#define ORL_ERR_ALIGN (-2)        /* a pointer or row size is not 16-byte aligned */
#define ORL_ERR_UNSUPPORTED (-3)  /* head_dim not in {64, 128} */
#define ORL_ERR_DRIVER (-4)       /* cuTensorMapEncodeTiled unavailable */
#define ORL_ERR_TENSOR_MAP (-5)   /* the driver rejected a tensor map */
#define ORL_ERR_LAUNCH (-6)       /* kernel launch failed */
#define ORL_ERR_CAPACITY (-7)     /* a caller buffer is too small */
#define ORL_ERR_COMM (-8)         /* NCCL reported an error (the communicator is aborted after a failed wait) */
#define ORL_ERR_TIMEOUT (-9)      /* orl_comm_wait gave up: the communicator was aborted */

/* One attention work item: up to 256 query rows of one segment and one head. */
typedef struct orl_attn_work {
  int32_t q_row0; /* first packed query row */
  int32_t q_len;  /* query rows in this item, 1..256 */
  int32_t k_row0; /* first packed key row of the segment */
  int32_t k_len;  /* keys of the segment (0 gives a zero output and LSE -inf) */
  int32_t head;
  int32_t seg;    /* segment index, for diagnostics */
  int32_t pad0, pad1;
} orl_attn_work;

/* Library version string. */
ORL_API const char* orl_version(void);

/* Message for an ORL_ERR_* code. */
ORL_API const char* orl_error_string(int code);

/* Bits the kernels set in the caller's error word when a bounded wait gave up (the kernel then winds down). */
ORL_API int orl_error_bits_describe(int bits, char* buf, int cap);

/* Failure-path self test of the kernels' bounded waits: a one-CTA kernel waits on an mbarrier nothing arrives at,
 * gives up after limit_ns (<= 1 s) and writes the timeout bits to status_dev (nonzero = the wait ran out, as it
 * must). Has no counterpart in the reference (which has no device-side failure detection). */
ORL_API int orl_selftest_timeout(int* status_dev, unsigned long long limit_ns, void* stream);

/* Work list of a packed varlen call: replaces the scheduling FlashAttention does internally for
 * attention.py:39-43. cu_q / cu_k: HOST int32 [n_seg + 1] (attention.py:28-29 cu_seqlens). Writes up to
 * `capacity` items (largest key range first; items of one segment and head adjacent) and returns their count.
 * If `work` is NULL or too small, returns -(needed + 1000) so the caller can size the buffer. */
ORL_API int orl_attn_plan(const int32_t* cu_q, const int32_t* cu_k, int n_seg, int heads, orl_attn_work* work,
                          int capacity);

/* As orl_attn_plan, with each segment's query and key rows given as (start, length): key ranges may overlap and
 * need not be in order, so contiguous per-scene key ranges are read in place without a pack. Replaces the FA3
 * `cu_seqlens_k` offsets + `seqused_k` call of attention.py:74-84 (`overlapping_ranges`). HOST int32 [n_seg] each. */
ORL_API int orl_attn_plan_ranges(const int32_t* q_start, const int32_t* q_len, const int32_t* k_start,
                                 const int32_t* k_len, int n_seg, int heads, orl_attn_work* work, int capacity);

/* Packed varlen attention forward (attention.py:39-53 `varlen` / `varlen_lse`): out = softmax(q k^T * scale) v per
 * segment, out [nq, heads, head_dim] bf16; lse (optional, may be NULL) [heads, nq] fp32 natural-log LSE.
 * work_dev: the plan's items in device memory; err_dev: a device int the kernel ORs timeout bits into (the caller
 * zeroes it; nonzero after the call means the result is invalid). head_dim 64 or 128. */
ORL_API int orl_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse, long long nq, long long nk,
                 int heads, int head_dim, float scale, const orl_attn_work* work_dev, int n_items, int* err_dev,
                 void* stream);

/* The varlen call with cu_seqlens in DEVICE memory, as the reference passes them to FlashAttention
 * (attention.py:28-29 `cu_seqlens`, 39-43 `varlen`): cu_q_dev / cu_k_dev int32 [n_seg + 1] on the device. The work
 * list is planned on the device (same items and order as orl_attn_plan), so the call returns without waiting for the
 * GPU. work_dev: caller scratch of work_capacity items, at least orl_attn_fwd_cu_capacity(nq, n_seg, heads) (slot 0
 * receives the planned item count). cu_seqlens that decrease or leave [0, nq] / [0, nk] compute nothing and set an
 * error bit in err_dev (orl_error_bits_describe). At most 4096 segments. head_dim 64 or 128. */
ORL_API int orl_attn_fwd_cu(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                            long long nk, int heads, int head_dim, float scale, const int32_t* cu_q_dev,
                            const int32_t* cu_k_dev, int n_seg, orl_attn_work* work_dev, long long work_capacity,
                            int* err_dev, void* stream);

/* Work-list slots orl_attn_fwd_cu needs: 1 + heads * (ceil(nq / 256) + n_seg). */
ORL_API long long orl_attn_fwd_cu_capacity(long long nq, int n_seg, int heads);

/* Allocation-free variant of orl_attn_fwd, for callers that cannot call cudaMalloc (code inside another
 * framework's memory pool or allocator hook, or a plugin host that owns all device memory) and so cannot supply the
 * work list and error word orl_attn_fwd needs. Has no counterpart in the reference. The scratch lives in a
 * file-scope device array of the library (about 512 KiB per GPU that loads it, held until the process exits); the
 * call orders the segments on the host (cu_q_host / cu_k_host: HOST int32 [n_seg + 1]), passes that table to the
 * GPU as a kernel parameter and allocates nothing. Limits: at most 1024 segments and 16384 work items (heads x
 * ceil(q rows / 256) summed over segments): larger calls return ORL_ERR_CAPACITY before any work. q, k, v, out, lse
 * and the stream must belong to the current device (else ORL_ERR_ARG). Calls share the array (it keeps the last
 * call's contents; the error word is cleared per call): calls that overlap on one GPU race, so serialise them per
 * device. The first call on a device looks up the array's address and caches it (a cudaDeviceReset invalidates the
 * cache); make that first call before any stream capture. status_host (optional): when not NULL the call waits for
 * the kernel and stores its timeout bits (0 = ok). */
ORL_API int orl_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* out, float* lse, long long nq,
                                 long long nk, int heads, int head_dim, float scale, const int32_t* cu_q_host,
                                 const int32_t* cu_k_host, int n_seg, int* status_host, void* stream);

/* One row-range copy of a pack: `nbytes` from base[src_slot] + src_off to base[dst_slot] + dst_off. */
typedef struct orl_copy_run {
  int32_t src_slot; /* index into src_bases */
  int32_t dst_slot; /* index into dst_bases */
  int64_t src_off;  /* bytes */
  int64_t dst_off;  /* bytes */
  int64_t vec0;     /* first 16-byte vector of this run in the pack (prefix sum, filled by orl_pack_prepare) */
} orl_copy_run;

/* Fills runs[i].vec0 (prefix sums of nbytes[i] / 16) and returns the pack's total 16-byte vectors, or an error if
 * a size or offset is not a multiple of 16. nbytes: HOST int64 [n_runs]. */
ORL_API long long orl_pack_prepare(orl_copy_run* runs, const int64_t* nbytes, int n_runs);

/* Gather/pack kernel: executes the prepared run table (device copy, runs_dev [n_runs]) for `n_planes` planes at
 * once (e.g. K and V share one run table): plane p reads src_bases[p * n_slots + slot] and writes
 * dst_bases[p * n_slots + slot]. TMA bulk copies staged through shared memory, HBM-bound. When cu_out_dev is not
 * NULL, also writes cu_seqlens: cu_out_dev[0 .. n_seg] = [0, cumsum(seg_len_dev)] (int32, attention.py:28-29).
 * err_dev (optional device int): a bounded wait that gave up ORs its bit in (see orl_error_bits_describe).
 * At most 16 slots and 3 planes. Sources may be another GPU's memory mapped into this process (symmetric memory
 * of the K/V exchange): the bulk loads carry no multicast. */
ORL_API int orl_pack(const orl_copy_run* runs_dev, int n_runs, long long total_vecs, int n_planes, int n_slots,
             const void* const* src_bases, void* const* dst_bases, const int32_t* seg_len_dev, int n_seg,
             int32_t* cu_out_dev, int* err_dev, void* stream);

/* Log-sum-exp merge of two partial attention results over disjoint key sets (hunyuan15.py:274-276, ring.py:63-70):
 * o1 [n, heads, head_dim] bf16 (in/out) with its lse1 [heads, ld_lse1] fp32 (in/out), o2 / lse2 [heads, ld_lse2]
 * the second part; rows [0, n) of each. head_dim a multiple of 32. */
ORL_API int orl_lse_merge(void* o1, float* lse1, const void* o2, const float* lse2, long long n, long long ld_lse1,
                  long long ld_lse2, int heads, int head_dim, void* stream);

/* As orl_lse_merge with an fp32 accumulator (parallel/ring.py:63-70 `_merge`, which keeps o in fp32 across the ring
 * steps): acc [n, heads, head_dim] fp32 and lse_acc [heads, ld_lse1] (in/out) merged with a bf16 part and its lse. */
ORL_API int orl_lse_merge_acc(float* acc, float* lse_acc, const void* part, const float* lse_part, long long n,
                              long long ld_lse1, long long ld_lse2, int heads, int head_dim, void* stream);

/* Fused q/k RMSNorm + rotary embedding (the q/k preparation of hunyuan15.py:187-190 and wan.py:64-74 `_qk`, which
 * the reference runs as separate ops / a torch.compile'd Triton kernel): x, y [rows, heads * head_dim] bf16 (y may
 * alias x); weight bf16 [head_dim] (per_head = 1: RMSNorm over each head, Hunyuan) or [heads * head_dim] (per_head =
 * 0: over the whole row, Wan); cos_t / sin_t fp32 [rows, rope_ld], pair i of a head rotated by cos[2i] and
 * sin[2i + sin_shift] (sin_shift 0: tables repeated per pair, Hunyuan; 1: Wan's cos[..., 0::2] / sin[..., 1::2]).
 * row_map (optional): output row of each input row (write straight into a packed layout). */
ORL_API int orl_qk_norm_rope(const void* x, void* y, const void* weight, const float* cos_t, const float* sin_t,
                             long long rows, int heads, int head_dim, int per_head, float eps, int sin_shift,
                             long long rope_ld, const int32_t* row_map, void* stream);

/* In-place rotary rotation of listed rows (no norm), for moving shared-frame keys of a packed K to their adjacent
 * temporal positions (hunyuan15.py:127-150 `_move_shared`, which applies R(-src) then R(dst) with two
 * apply_rotary_emb calls): x [*, heads * head_dim] bf16; row rows[i] rotated by table row i of cos_t / sin_t
 * (fp32 [n_rows, rope_ld], pair i by cos[2i], sin[2i + sin_shift]). */
ORL_API int orl_rope_rows(void* x, const int32_t* rows, long long n_rows, int heads, int head_dim, const float* cos_t,
                          const float* sin_t, long long rope_ld, int sin_shift, void* stream);

/* Device barrier of the peer-memory K/V exchange (replaces the synchronisation NCCL's send/recv gives the
 * reference's HaloExchange, parallel/comm.py:126-201): pads[p] = rank p's signal pad (int[world] in symmetric memory,
 * zeroed before first use; peer addresses valid in this process). Writes epoch into slot `rank` of every pad, then
 * waits until every slot of pads[rank] holds at least epoch; epochs must grow by one per call. After timeout_ns the
 * wait gives up and ORs its bit into err_dev (no hang). world <= 16. */
ORL_API int orl_peer_barrier(int* const* pads, int world, int rank, int epoch, unsigned long long timeout_ns,
                             int* err_dev, void* stream);

/* All-to-all of the Ulysses path by pulls over peer memory (replaces the NCCL all_to_all_single calls of
 * parallel/comm.py:276-295 a2a_heads / a2a_tokens): for every plane pl < planes (<= 3), peer p < n_peers (<= 16),
 * row i < rows, copies seg_bytes from src[pl * n_peers + p] + src_row0 + i * src_stride to
 * dst[pl] + p * dst_pstride + i * dst_stride. src may be other GPUs' memory mapped into this process (symmetric
 * buffers, after orl_peer_barrier). Offsets, strides and sizes multiples of 16 bytes. */
ORL_API int orl_peer_gather(const void* const* src, void* const* dst, int planes, int n_peers, long long rows,
                            long long seg_bytes, long long src_row0, long long src_stride, long long dst_pstride,
                            long long dst_stride, void* stream);

/* ---------------------------------------------------------------- frame memory (src/onereel/frame_memory.py) */

/* Per-frame pooling of one layer's hidden states (frame_memory.py:76-85 `collect`, an index_add_ of the rows into
 * per-frame sums and counts): acc[f * ld_acc + c] += sum of hs[row * ld_hs + c] over the rows of frame f and
 * acc[f * ld_acc + C] += their number. Rows in CSR form: rows_by_frame[frame_off[f] .. frame_off[f + 1]] (device
 * int32; rows of no frame are simply not listed). hs: bf16 (dtype 0) or fp32 (dtype 1), C a multiple of 8, rows
 * 16-byte aligned; acc fp32 with ld_acc >= C + 1. Deterministic (fixed summation order, no atomics). */
ORL_API int orl_frame_pool(const void* hs, int dtype, long long ld_hs, int C, const int32_t* rows_by_frame,
                           const int32_t* frame_off, int n_frames, float* acc, long long ld_acc, void* stream);

/* fp32 elements of scratch orl_frame_select needs per set. */
ORL_API long long orl_frame_select_scratch(int C, int n_cand, int k);

/* Representative frames by cosine k-means (frame_memory.py:87-132 `finish` + `select`), for n_sets feature sets at
 * once (one per observed layer; set s at feat + s * set_stride, fp32 rows of stride ld). normalize = 1: rows hold
 * [sums (C), count] and the candidate rows are first replaced by their L2-normalised means (in place); 0: rows are
 * already normalised features. cand: device int32 [n_cand] candidate frames; k clusters (1..min(n_cand, 64)), at
 * most `iters` Lloyd steps. reps: device int32 [n_sets, k + 1]: the number of representatives n, then n frame
 * indices ascending (-1 after). scratch: device fp32, scratch_stride >= orl_frame_select_scratch per set. */
ORL_API int orl_frame_select(float* feat, long long ld, long long set_stride, int n_sets, int C, int normalize,
                             const int32_t* cand, int n_cand, int k, int iters, float* scratch,
                             long long scratch_stride, int32_t* reps, void* stream);

/* ---------------------------------------------------------------- native planner (comm.py:18-112, layout.py:54-78) */

/* A scene layout (layout.py:10-18 SceneLayout): lengths[n_scenes] latent frames per scene, halo frames of the
 * neighbours on `sides` (0 'adj', 1 'prev', 2 'next'), extra frames per scene in CSR form
 * (extra_frames[extra_offsets[j] .. extra_offsets[j + 1]]; both may be NULL for none). */
typedef struct orl_layout {
  const int32_t* lengths;
  int32_t n_scenes;
  int32_t halo;
  int32_t sides;
  const int32_t* extra_offsets;
  const int32_t* extra_frames;
} orl_layout;

#define ORL_MODE_SCENE 0
#define ORL_MODE_ULYSSES 1
#define ORL_GRAN_BALANCED 0
#define ORL_GRAN_TOKENS 1
#define ORL_GRAN_SCENES 2

/* Eq. 2 inputs and decision (comm.py:104-108). */
typedef struct orl_path {
  long long remote_rows; /* max over ranks of the K/V rows (per tensor) a rank gathers */
  double V_G;            /* 2 * remote_rows */
  double V_U;            /* 4 L (P - 1) / P^2 */
  int32_t gather;        /* 1: 'scene' (K/V gathering), 0: 'ulysses' */
} orl_path;

/* Scene j's key frames: own frames, then halo and extra frames (layout.py:54-73). Returns the count, or
 * -(count + 1000) when `frames` is NULL or too small. */
ORL_API int orl_key_frames(const orl_layout* layout, int scene, int32_t* frames, int capacity);

/* Per scene, the cost of one video query (comm.py:18-22): cost[n_scenes]; text may be NULL. */
ORL_API int orl_query_cost(const orl_layout* layout, long long T, const int32_t* text, long long extra_keys,
                           double* cost);

/* Paper Algorithm 1 (comm.py:25-40): bounds[0..n] cuts of sum(sizes) queries into n work-balanced ranges. */
ORL_API int orl_balanced(const int64_t* sizes, const double* cost, int n_scenes, int n, int64_t* bounds);

/* Per-rank video token ranges (comm.py:43-66): bounds[0..n]; mode ORL_MODE_*, granularity ORL_GRAN_*. */
ORL_API int orl_partition(const orl_layout* layout, long long T, int n, int mode, const int32_t* text,
                          long long extra_keys, int granularity, int64_t* bounds);

/* Token intervals outside [own_lo, own_hi) that the scenes intersecting it read (comm.py:88-96), plus the
 * `extra` frames; intervals[2 * i], intervals[2 * i + 1]. Returns the count or -(count + 1000) if too small. */
ORL_API int orl_needed(const orl_layout* layout, long long T, long long own_lo, long long own_hi, const int32_t* extra,
                       int n_extra, int64_t* intervals, int capacity);

/* Eq. 2 path choice for a partition (comm.py:99-112). */
ORL_API int orl_choose_path(const orl_layout* layout, long long T, const int64_t* bounds, int n, double theta,
                            const int32_t* extra, int n_extra, orl_path* path);

/* ---------------------------------------------------------------------------------------------------------------
 * Collectives of the multi-GPU path over NCCL (loaded with dlopen at the first call; a process that already loaded
 * NCCL shares it). They replace the torch.distributed calls of src/onereel/parallel/comm.py for C / C++ callers:
 * HaloExchange (126-201, batch_isend_irecv of K then V per interval and peer) -> orl_comm_exchange; rows every peer
 * reads -> orl_comm_broadcast; a2a_heads / a2a_tokens (276-295, all_to_all_single) -> orl_comm_all_to_all; the text
 * rows' dist.all_reduce -> orl_comm_all_reduce_f32. Operations are enqueued on the caller's stream; orl_comm_wait is
 * the timeout-aware completion check. */
typedef struct orl_comm orl_comm;  /* opaque: one NCCL communicator of one rank */

typedef struct orl_p2p {
  int32_t peer;    /* rank of the other side */
  int32_t pad;
  void* ptr;       /* device buffer */
  long long bytes;
} orl_p2p;

/* 1 if NCCL could be loaded, else 0. */
ORL_API int orl_comm_available(void);

/* A new NCCL unique id (128 bytes) on the rank that creates the communicator; the caller distributes it. */
ORL_API int orl_comm_unique_id(uint8_t* id_out);

/* Joins the communicator of `world` ranks identified by `id` as `rank`, on CUDA device `device` (blocks until every
 * rank has joined). */
ORL_API int orl_comm_init(orl_comm** comm, const uint8_t* id, int world, int rank, int device);

ORL_API int orl_comm_destroy(orl_comm* comm);

/* One grouped exchange: every send and receive of the lists, per peer in list order on both sides. */
ORL_API int orl_comm_exchange(orl_comm* comm, const orl_p2p* sends, int n_send, const orl_p2p* recvs, int n_recv,
                              void* stream);

/* In-place broadcast of `bytes` from `root`. */
ORL_API int orl_comm_broadcast(orl_comm* comm, void* buf, long long bytes, int root, void* stream);

/* Equal-split all-to-all: block p (bytes_per_peer) of send goes to rank p, block p of recv comes from rank p. */
ORL_API int orl_comm_all_to_all(orl_comm* comm, const void* send, void* recv, long long bytes_per_peer, void* stream);

/* In-place sum over the ranks of n floats. */
ORL_API int orl_comm_all_reduce_f32(orl_comm* comm, float* buf, long long n, void* stream);

/* Waits until `stream` is idle, polling NCCL's asynchronous error. An NCCL error or `timeout_ns` without completion
 * aborts the communicator (its in-flight operations end) and returns ORL_ERR_COMM / ORL_ERR_TIMEOUT; the
 * communicator is then unusable except for orl_comm_destroy. */
ORL_API int orl_comm_wait(orl_comm* comm, void* stream, unsigned long long timeout_ns);

#ifdef __cplusplus
}
#endif

#endif /* ONEREEL_B200_H */
