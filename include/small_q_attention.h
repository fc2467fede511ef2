/*
 * small_q_attention.h -- C ABI of the B200 (sm_100a) small-q paged attention path.
 *
 * Operator: causal paged multi-token-prediction (MTP / speculative-decoding)
 * attention with a uniform draft length q_len.  For batch element b, draft row
 * qi and query head qh:
 *
 *   kvh   = qh / (Hq / Hkv)
 *   valid = seq_lens[b] - q_len + qi + 1           (tokens 0 .. valid-1 visible)
 *   out[b,qi,qh,:] = softmax(K[b,:valid,kvh] . q[b,qi,qh] / sqrt(128)) V[b,:valid,kvh]
 *
 * where token t of sequence b lives in page block_tables[b, t / 16], slot t % 16.
 * This is the contract of the upstream paged_mtp_attention_reference
 * (src/small_q_attention/reference.py:10-74) and of its CUDA entry points
 * (src/small_q_attention/cuda.py:177-214 -> csrc/small_q_attention_ext.cu:1132-1210).
 *
 * Layout (all row-major, contiguous):
 *   query        fp16 or bf16 (sqa_args.dtype)  [batch, q_len, num_q_heads, 128]
 *   key_cache    same type  [num_pages, 16, num_kv_heads, 128]
 *   value_cache  same type  [num_pages, 16, num_kv_heads, 128]
 *   block_tables int32 [batch, max_pages]   (row stride max_pages)
 *   seq_lens     int32 [batch]              (total length incl. the q_len drafts)
 *   out          same type  [batch, q_len, num_q_heads, 128]
 * Supported: head_dim 128, page_size 16, num_q_heads == 4 * num_kv_heads,
 * 1 <= q_len <= 16.  All pointers are device pointers; query/out/caches must
 * be 16-byte aligned.
 *
 * Nothing here allocates device memory: the caller passes a workspace of at
 * least sqa_workspace_bytes() bytes (fp32 split-KV partials and a device
 * status word).  Every entry point is asynchronous on
 * the given stream and returns a status code; no C++ exception crosses the ABI.
 */
#ifndef SMALL_Q_ATTENTION_H_
#define SMALL_Q_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SQA_API __attribute__((visibility("default")))
#else
#define SQA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SQA_HEAD_DIM 128
#define SQA_PAGE_SIZE 16
#define SQA_GQA_GROUP 4
#define SQA_MAX_Q_LEN 16

/* Host-side status codes returned by the entry points. */
typedef enum sqa_status {
  SQA_OK = 0,
  SQA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape or misaligned pointer */
  SQA_ERR_UNSUPPORTED = 2,      /* shape outside the supported contract        */
  SQA_ERR_WORKSPACE_TOO_SMALL = 3,
  SQA_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed            */
  SQA_ERR_DEVICE = 5            /* sqa_read_device_status found a device error  */
} sqa_status;

/* Bits of the device status word (sticky until cleared by sqa_read_device_status). */
#define SQA_DEV_TIMEOUT 1u         /* a bounded wait gave up; output is not valid       */
#define SQA_DEV_SEQ_TOO_LONG 2u    /* seq_lens[b] > 16 * max_pages: clamped to the table */
#define SQA_DEV_SEQ_TOO_SHORT 4u   /* seq_lens[b] < q_len (full mode only)              */
#define SQA_DEV_BAD_PAGE 8u        /* a page id outside [0, num_pages): read as page 0  */
#define SQA_DEV_CHECK 16u          /* a -DSQA_DEBUG_CHECKS bounds check failed; the word
                                      after the status word holds (check << 24) | index  */

typedef struct sqa_args {
  const void* query;           /* fp16 [batch, q_len, num_q_heads, 128]           */
  const void* key_cache;       /* fp16 [num_pages, 16, num_kv_heads, 128]         */
  const void* value_cache;     /* fp16 [num_pages, 16, num_kv_heads, 128]         */
  const int32_t* block_tables; /* int32 [batch, max_pages]                        */
  const int32_t* seq_lens;     /* int32 [batch]: tokens held for each sequence     */
  /* Optional int32 [batch], NULL = seq_lens.  The causal length used for the
   * spec-dec mask: row qi sees token t iff t < seq_lens[b] and
   * t < mask_lens[b] - q_len + qi + 1.  A shard that holds tokens
   * [offset, offset + seq_lens[b]) of a longer sequence passes
   * mask_lens[b] = whole_length - offset. */
  const int32_t* mask_lens;
  /* Full mode: out != NULL, fp16 [batch, q_len, num_q_heads, 128].
   * Partial mode: out == NULL and out_partial/out_lse != NULL: the normalised
   * fp32 output [batch, q_len, num_q_heads, 128] and its natural-log
   * log-sum-exp [batch, q_len, num_q_heads] (-inf for a row that sees no key),
   * ready for sqa_merge_partials. */
  void* out;
  float* out_partial;
  float* out_lse;
  int32_t batch;
  int32_t q_len;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;            /* must be 128 */
  int32_t page_size;           /* must be 16  */
  int32_t num_pages;           /* pages in the cache pool                          */
  int32_t max_pages;           /* block_tables row stride                          */
  /* Upper bound of seq_lens (0 = unknown: 16 * max_pages is used).  Only sizes
   * the launch; never read on the device, so no host synchronisation. */
  int32_t max_seq_len;
  /* Tuning: CTAs of the split-KV kernel (0 = auto: 2 per SM, fewer for short
   * work) and the minimum pages one CTA takes (0 = auto). */
  int32_t num_ctas;
  int32_t min_pages_per_cta;
  /* Kernel choice: 0 = auto (tcgen05 for q_len >= 9, for q_len 5..8 above 512
   * page-units, for q_len 3..4 from 2048 and for q_len <= 2 from 12288
   * page-units, where a page-unit is one page of one KV head, bounded by
   * max_seq_len or max_pages; warp-level otherwise),
   * 1 = warp-level mma.sync kernel, 2 = tcgen05 / tensor-memory kernel.
   * Both compute the same operator. */
  int32_t kernel;
  /* Element type of query, key_cache, value_cache and out: SQA_DTYPE_F16 or
   * SQA_DTYPE_BF16 (all four the same; accumulation is fp32 either way).  The
   * upstream supports fp16 only (src/small_q_attention/cuda.py:197-211). */
  int32_t dtype;
  /* Cache layout: SQA_KV_NHD = [num_pages, 16, num_kv_heads, 128] (the upstream's,
   * ext.cu:466) or SQA_KV_HND = [num_pages, num_kv_heads, 16, 128] (one KV head's
   * page contiguous; the default layout of FlashInfer's paged decode). */
  int32_t kv_layout;
  /* Softmax scale applied to q.k (0 = 1/sqrt(128), the upstream's,
   * src/small_q_attention/reference.py:46) and a factor applied to every output
   * row (0 = 1); e.g. FlashInfer's bmm1_scale / bmm2_scale. */
  float sm_scale;
  float out_scale;
  /* Elements from one page to the next in key_cache and value_cache (0 = the
   * caches are contiguous tensors, 16 * num_kv_heads * 128).  Larger values
   * address one layer of a bigger pool or K and V interleaved per page
   * ([num_pages, 2, ...]); a multiple of 8 (16-byte aligned pages). */
  int64_t page_stride;
  /* Element type of key_cache / value_cache: SQA_KV_SAME (as dtype) or
   * SQA_KV_FP8_E4M3 (1 byte, with fp16 or bf16 queries and output; tcgen05 kernel).
   * The tensor core reads the fp8 K/V as they are (kind::f8f6f4); each query
   * row (scaled by a power of two) and each probability enter as the sum of
   * two e4m3 parts, about 8 significant bits (measured max error 0.3 of the
   * fp16 tolerance).  Fold the caches' dequantisation scales into sm_scale (K)
   * and out_scale (V). */
  int32_t kv_dtype;
  /* Lower bound of seq_lens (0 = unknown).  Like max_seq_len, only steers the
   * launch: with both bounds within 15% of each other (near-uniform lengths)
   * and few enough (sequence, KV head) segments for two or more CTAs each, the
   * tcgen05 kernel splits every segment evenly over a thread-block cluster and
   * reduces the parts through distributed shared memory (no merge launch) on
   * short segments, or evenly over k CTAs without a cluster (merged by the merge
   * kernel; no CTA crosses a segment boundary) on long ones.  A wrong hint still
   * gives the right result, only a slower launch. */
  int32_t min_seq_len;
  /* Cluster mode: 0 = auto (above), 1 = off (segments cut into cost-balanced
   * CTA ranges, or with both length hints split evenly over k CTAs, merged by a
   * second kernel), 2 / 4 / 8 / 16 = that many CTAs per segment in one cluster
   * (tcgen05 kernel; 16-CTA clusters where the device allows them).
   * No upstream counterpart (the upstream splits with chunk_keys, ext.cu:1178). */
  int32_t cluster;
} sqa_args;

#define SQA_DTYPE_F16 0
#define SQA_DTYPE_BF16 1
#define SQA_KV_NHD 0
#define SQA_KV_HND 1
#define SQA_KV_SAME 0
#define SQA_KV_FP8_E4M3 1

/* Workspace bytes sqa_forward needs for these arguments on `device`
 * (-1 = the current device).  Depends only on shapes and tuning fields.
 * Returns 0 and sets *status on invalid arguments. */
SQA_API size_t sqa_workspace_bytes(const sqa_args* args, int device, int* status);

/* Run the operator on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Replaces small_q_attention_v3(...) (csrc/small_q_attention_ext.cu:1132-1210),
 * which the upstream binds as forward_v3 (:1384) and wraps in
 * small_q_attention.cuda.forward_v3 (src/small_q_attention/cuda.py:177-214).
 * Launches the split-KV partial kernel and the log-sum-exp merge kernel (which
 * only combines sequences split over several CTAs).  No device allocation, no host
 * synchronisation. */
SQA_API int sqa_forward(const sqa_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* sqa_forward that also records the caller's CUDA events (cudaEvent_t, may be
 * NULL) on `stream` immediately before and after the split-KV kernel launch,
 * so the dominant kernel can be timed with events on its own stream.  Under
 * stream capture the records become event-record nodes on side branches of the
 * graph: each depends on the work captured before it, and nothing captured later
 * depends on it, so consecutive launches keep their programmatic (early-launch)
 * overlap; event_before then fires when the previous call's last kernel ends and
 * event_after when the split-KV kernel ends (its duration inside a replay of
 * back-to-back calls).  Does the same work as sqa_forward.  No upstream
 * counterpart (measurement hook). */
SQA_API int sqa_forward_timed(const sqa_args* args, void* workspace, size_t workspace_bytes, void* stream,
                              void* event_before, void* event_after);

/* Merge num_parts partial results (e.g. one per GPU of a split sequence) into
 * one.  parts_o: fp32 [num_parts, rows, 128]; parts_lse: fp32 [num_parts, rows]
 * natural-log; rows = batch * q_len * num_q_heads.  Writes fp16 out[rows,128]
 * when out != NULL, and/or fp32 out_o[rows,128] and out_lse[rows] when those
 * are non-NULL.  Same arithmetic as the upstream split-KV merge
 * (csrc/small_q_attention_ext.cu:339-366): a row whose parts all have
 * lse = -inf gets 0. */
SQA_API int sqa_merge_partials(const float* parts_o, const float* parts_lse, int32_t num_parts,
                       int64_t rows, void* out, float* out_o, float* out_lse, void* stream);

/* Read (and optionally clear) the sticky device status word in a workspace
 * used by sqa_forward.  Synchronises `stream`.  *device_bits receives the
 * SQA_DEV_* bits; returns SQA_ERR_DEVICE when any bit is set. */
SQA_API int sqa_read_device_status(void* workspace, uint32_t* device_bits, int clear, void* stream);

/* The kernel sqa_forward would launch for these arguments on `device` (-1 =
 * the current device): 1 = warp-level mma.sync kernel, 2 = tcgen05 kernel,
 * 2 + 100 * C = tcgen05 kernel in clusters of C CTAs per segment,
 * 2 + 10000 * k = tcgen05 kernel with every segment split evenly over k CTAs;
 * minus the SQA_ERR_* code on invalid arguments.  Resolves kernel = 0 (auto).
 * No upstream counterpart (introspection for measurement and tests). */
SQA_API int sqa_selected_kernel(const sqa_args* args, int device);

/* Zero a workspace before its first use (asynchronous). */
SQA_API int sqa_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Size of the scratch array built into the library for sqa_forward_noalloc. */
#define SQA_NOALLOC_SCRATCH_BYTES (16u << 20)

/* sqa_forward for callers that cannot allocate device memory: the workspace
 * comes from a SQA_NOALLOC_SCRATCH_BYTES array of device memory inside this
 * library instead of from the caller.  Callers that cannot allocate include
 * bindings that call this C ABI directly from a language without a CUDA
 * allocator, and serving engines that give almost all of HBM to their
 * KV-cache pool and forbid allocations (which could fail, and which
 * synchronise the device) in the middle of a decode step.
 * - Every GPU that loads the library holds the array until the process exits.
 * - The first call with a device current looks up the array's device address
 *   on that device; make that first call before any stream capture.  The
 *   address is kept for the device's primary context: calls after
 *   cudaDeviceReset, or under another context, are not supported.
 * - Shapes whose sqa_workspace_bytes() exceeds SQA_NOALLOC_SCRATCH_BYTES are
 *   rejected with SQA_ERR_WORKSPACE_TOO_SMALL.
 * - All calls share the one array: calls that overlap on the GPU (other
 *   streams, other threads) race and must be serialised by the caller.
 * - The device status bits are cleared at the start of every call; read the
 *   last call's bits with sqa_noalloc_read_device_status.  Host-side
 *   validation is the same as sqa_forward's.
 * No counterpart in the reference (its launcher allocates scratch per call
 * with torch::empty, csrc/small_q_attention_ext.cu:1183-1185). */
SQA_API int sqa_forward_noalloc(const sqa_args* args, void* stream);

/* sqa_read_device_status for the scratch array of sqa_forward_noalloc on the
 * current device: the SQA_DEV_* bits of the last call (sticky until cleared;
 * every sqa_forward_noalloc call clears them first).  Synchronises `stream`.
 * No counterpart in the reference. */
SQA_API int sqa_noalloc_read_device_status(uint32_t* device_bits, int clear, void* stream);

/* ---- Cache append: the step before attention in MTP decoding ----
 * Writes the K/V of the q_len new tokens of every sequence into their page
 * slots: token qi of sequence b is position t = seq_lens[b] - q_len + qi
 * (seq_lens is the length after the append, as the attention takes it,
 * src/small_q_attention/reference.py:25), stored in page block_tables[b, t/16],
 * slot t % 16.  The upstream leaves this step to its caller; no upstream
 * function is replaced.  A sequence with seq_lens < q_len or more pages than
 * max_pages is skipped whole (SQA_DEV_SEQ_TOO_SHORT / SQA_DEV_SEQ_TOO_LONG), a
 * token whose page id is outside [0, num_pages) is skipped (SQA_DEV_BAD_PAGE);
 * the bits are ORed into *status (a device word, e.g. the first word of a
 * workspace; may be NULL).  Two
 * tokens mapped to the same slot race.  Asynchronous on `stream`; a pure copy.
 *   new_keys, new_values  fp16 [batch, q_len, num_kv_heads, 128], 16-byte aligned
 *   key_cache, value_cache [num_pages, 16, num_kv_heads, 128] (NHD) or
 *                          [num_pages, num_kv_heads, 16, 128] (HND), 16-byte aligned.
 *   Any 2-byte element type (fp16 or bf16: the append is a copy), or fp8 e4m3
 *   with kv_dtype = SQA_KV_FP8_E4M3 (new K/V already in fp8). */
typedef struct sqa_append_args {
  const void* new_keys;
  const void* new_values;
  void* key_cache;
  void* value_cache;
  const int32_t* block_tables; /* [batch, max_pages] */
  const int32_t* seq_lens;     /* [batch], lengths after the append */
  uint32_t* status;            /* device status word or NULL */
  int32_t batch;
  int32_t q_len;
  int32_t num_kv_heads;
  int32_t head_dim;            /* must be 128 */
  int32_t page_size;           /* must be 16 */
  int32_t num_pages;
  int32_t max_pages;
  int32_t kv_layout;           /* SQA_KV_NHD or SQA_KV_HND, as in sqa_args */
  int64_t page_stride;         /* elements from page to page, 0 = contiguous (as in sqa_args) */
  int32_t kv_dtype;            /* SQA_KV_SAME (2-byte elements) or SQA_KV_FP8_E4M3 (1-byte) */
} sqa_append_args;

SQA_API int sqa_cache_append(const sqa_append_args* args, void* stream);

/* ---- Long-context split across the GPUs of one node ----
 * One sequence's pages are cut into contiguous ranges, one per rank (one
 * process per GPU); every rank computes the shard form of the operator over
 * its range (sqa_forward in partial mode, mask_lens in whole-sequence
 * coordinates) and these calls merge the partial (O, LSE) on rank 0: every rank
 * stores its partial into its slot in rank 0's memory with peer stores over
 * NVLink and sets a flag; rank 0 waits for the flags (bounded waits), merges
 * with the arithmetic of sqa_merge_partials and acknowledges every rank.  No
 * collective library is involved; the steady state allocates nothing, does not
 * synchronise the host and can be captured in a CUDA graph (the step counter
 * lives in device memory).  The upstream has no multi-GPU code; this replaces
 * an all-gather of the partials to every rank plus a merge on every rank.
 *
 * Set-up, on every rank with its device current:
 *   sqa_lc_create(rank, world, rows, &group, handle)   allocates this rank's
 *     exchange block (cudaMalloc) and writes its IPC handle (sqa_lc_handle_bytes()
 *     bytes) to `handle`; rows = batch * q_len * num_q_heads of the merged output;
 *   exchange the handles between the ranks (any host channel), then
 *   sqa_lc_connect(group, handles)   maps the other ranks' blocks; `handles` holds
 *     world handles back to back in rank order.
 * Every step, in the same order on every rank, on the stream of the partial:
 *   sqa_lc_exchange(group, o, lse, out, out_bf16, stream)   o fp32 [rows, 128] and
 *     lse fp32 [rows] (natural log, -inf for a row without keys) of this rank;
 *     on rank 0 `out` receives the merged [rows, 128] fp16 (bf16 with out_bf16),
 *     elsewhere it is ignored (may be NULL).
 * A wait that gives up (about a second: a rank that stopped) sets
 * SQA_DEV_TIMEOUT in the group's status word, read with sqa_lc_read_status
 * (synchronises the stream).  Tear-down, with no exchange in flight: every rank
 * calls sqa_lc_disconnect (unmaps the other ranks' blocks), then after a
 * barrier sqa_lc_destroy (frees its own block).  world <= 8. */
typedef struct sqa_lc_group sqa_lc_group;
SQA_API size_t sqa_lc_handle_bytes(void);
SQA_API int sqa_lc_create(int32_t rank, int32_t world, int64_t rows, sqa_lc_group** group, void* handle_out);
SQA_API int sqa_lc_connect(sqa_lc_group* group, const void* handles);
SQA_API int sqa_lc_exchange(sqa_lc_group* group, const float* o, const float* lse, void* out, int32_t out_bf16,
                            void* stream);
SQA_API int sqa_lc_read_status(sqa_lc_group* group, uint32_t* device_bits, int clear, void* stream);
SQA_API int sqa_lc_disconnect(sqa_lc_group* group);
SQA_API int sqa_lc_destroy(sqa_lc_group* group);

/* Static description of a status code. */
SQA_API const char* sqa_status_string(int status);

/* Version of this ABI (major * 100 + minor). */
SQA_API int sqa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SMALL_Q_ATTENTION_H_ */
