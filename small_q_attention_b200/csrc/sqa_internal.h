// sqa_internal.h -- declarations shared by the kernel and C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sqa {

constexpr int kHeadDim = 128;
constexpr int kPageSize = 16;
constexpr int kGroup = 4;                 // query heads per KV head
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one TMA producer warp
constexpr int kStageBytes = 4 * 2048;     // K and V of one page of one KV head, two 64-dim halves each
constexpr int kMaxStages = 16;
constexpr int kCombineStride = kHeadDim + 4;  // fp32 row stride of the combine buffer (bank-conflict free)

// Which warp shape a q_len uses.  A KV head owns R = 4 * q_len packed query
// rows; each consumer warp holds 8 * nt of them (nt n8-tiles of the swapped
// MMA), wr warps split the rows, and the 4 / wr token groups split the pages.
struct WarpShape {
  int nt;        // n8 tiles (rows / 8) per warp: 1 or 2
  int wr;        // warps across the rows: 1, 2 or 4
  int rows_pad;  // 8 * nt * wr >= 4 * q_len
  int wt() const { return kConsumerWarps / wr; }
};

inline WarpShape warp_shape_for(int q_len) {
  const int rows = kGroup * q_len;
  if (rows <= 8) return {1, 1, 8};
  if (rows <= 16) return {2, 1, 16};
  if (rows <= 32) return {2, 2, 32};
  return {2, 4, 64};
}

struct SplitKvParams {
  const __half* q;              // [B, q_len, Hq, 128] (fp16 or bf16 bits)
  const int32_t* block_tables;  // [B, max_pages]
  const int32_t* seq_lens;      // [B]
  const int32_t* mask_lens;     // [B] or nullptr
  __half* out;                  // full mode
  float* out_o;                 // partial mode
  float* out_lse;               // partial mode
  float* ws_o;                  // [pieces, rows_pad, 128]
  float* ws_lse;                // [pieces, rows_pad]
  unsigned int* status;
  int batch, q_len, hq, hkv, max_pages, num_pages;
  int num_stages;
  int num_pieces;               // workspace partial slots
  int rows_pad;                 // workspace rows per piece
  unsigned long long* timeline; // -DSQA_DEBUG_TIMELINE: 8 stamps per CTA, else nullptr
  float scale_log2;             // head_dim^-0.5 * log2(e)
  int bf16;                     // q / caches / out hold bf16 (else fp16) bits
  int hnd;                      // caches are [P, Hkv, 16, 128] (else [P, 16, Hkv, 128])
  float out_scale;              // multiplies every output row (1 = plain attention)
  int kv_fp8;                   // caches hold fp8 e4m3, read as fp8 by the tensor core (tcgen05 kernel):
                                // 2 in blocks of 4 pages, 3 in blocks of 8 pages
  int seg_cost;                 // schedule: units a segment start costs a CTA (one more epilogue)
  int cluster;                  // tcgen05 kernel: 0, or C >= 2 = segment blockIdx.x / C split evenly over
                                // a thread-block cluster of C CTAs, partials reduced through DSMEM
  int seg_split;                // tcgen05 kernel: 0, or k >= 2 = segment blockIdx.x / k split evenly over
                                // k CTAs (no cluster), partials merged by the merge kernel
};

struct MergeParams {
  const float* parts_o;         // piece i, row r at parts_o + (i * piece_rows + r) * 128 (+ first offset)
  const float* parts_lse;
  const int32_t* seq_lens;      // per-call merge: empty sequences are written as 0 / -inf
  unsigned int* status;         // per-call merge: device status word
  unsigned long long* timeline; // -DSQA_DEBUG_TIMELINE: 4 stamps per merge CTA, else nullptr
  __half* out;
  float* out_o;
  float* out_lse;
  long long rows;               // cross-device merge: total rows; per-call merge: unused
  int num_parts;                // cross-device merge: parts; per-call merge: workspace partial slots
  int piece_rows;               // rows per piece (rows_pad for the per-call merge)
  int batch, q_len, hq, hkv, max_pages;
  int bf16;                     // out holds bf16 (else fp16)
  int split_grid, seg_cost;     // per-call merge: the split-KV launch's schedule (pieces of a segment)
  int seg_split;                // per-call merge: k >= 2 when the split-KV launch split every segment
                                // evenly over k CTAs (SplitKvParams::seg_split)
};

// Launchers (stream-ordered, no allocation).  Return cudaGetLastError().
cudaError_t launch_split_kv(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                            int grid, int smem_bytes, cudaStream_t stream);
cudaError_t launch_segment_merge(const MergeParams& p, int rows_pad, cudaStream_t stream);
cudaError_t launch_partials_merge(const MergeParams& p, cudaStream_t stream);

// Dynamic shared memory of the split-KV kernel for a warp shape and stage count.
int split_kv_smem_bytes(const WarpShape& ws, int num_stages);

// The tcgen05 / tensor-memory variant of the split-KV kernel (any q_len <= 16).
cudaError_t launch_split_kv_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               int grid, int smem_bytes, cudaStream_t stream);
int split_kv_tc_smem_bytes(int num_blocks, int kv_fp8 = 0);
int split_kv_tc_block_bytes(int kv_fp8 = 0);
// Clusters of `cluster` tcgen05 CTAs (with `smem_bytes` each) that can be resident at once on
// the current device (0 when that cluster size cannot be launched).
int split_kv_tc_max_clusters(int cluster, int smem_bytes);

}  // namespace sqa
