// sqa_merge.cu -- log-sum-exp merge of split-KV partials.
//
// One warp merges one output row: each lane accumulates a float4 column of
// the 128-dim row over the parts with weights exp(lse_i - LSE), 8 parts per
// memory round trip (sqa_merge_row.cuh).  A row whose parts all have
// lse = -inf (no visible key) is written as 0 (and -inf).  This is the
// arithmetic of the upstream split-KV merge (csrc/small_q_attention_ext.cu:
// 339-366: global max, rescale, sum, divide, 0 when the denominator is 0) on
// normalised partials.
#include "sqa_internal.h"
#include "sqa_merge_row.cuh"
#include "sqa_ptx.cuh"
#include "sqa_schedule.cuh"

namespace sqa {
namespace {

// Per-call merge: grid (B * Hkv, ceil(4 * q_len / 4)), 4 warps = 4 rows per CTA.
// Before its dependency wait each warp works out its segment's pieces from
// seq_lens (an input the split kernel does not write: final before that kernel
// started) with the split kernel's own schedule; after the wait one round trip
// brings the partials.
__global__ void __launch_bounds__(128) sqa_segment_merge_kernel(const MergeParams p) {
  unsigned long long* tl =
      p.timeline ? p.timeline + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 4 : nullptr;
  if (threadIdx.x == 0) SQA_STAMP(tl, 0);
  // The next kernel may launch now: it waits for this grid's completion before
  // it touches memory, and until then its CTAs take SMs as the split-KV CTAs
  // leave them (and prefetch).
  allow_dependent_launch();
  const int s = blockIdx.x;
  const int b = s / p.hkv;
  const int h = s - b * p.hkv;
  const int2 info = p.seg_split
                        ? aligned_segment_pieces(p.seq_lens, p.max_pages, p.hkv, p.seg_split, b, h)
                        : segment_pieces(p.seq_lens, p.batch, p.max_pages, p.hkv, p.seg_cost, p.split_grid, b, h);
  grid_dependency_wait();    // the split-KV grid has finished writing the partials
  if (threadIdx.x == 0) SQA_STAMP(tl, 1);
  const int rows = kGroup * p.q_len;
  const int row = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const size_t out_row = (size_t)(b * p.q_len + (row >> 2)) * p.hq + h * kGroup + (row & 3);
  __half* out = p.out ? p.out + out_row * kHeadDim : nullptr;
  float* out_o = p.out_o ? p.out_o + out_row * kHeadDim : nullptr;
  float* out_lse = p.out_lse ? p.out_lse + out_row : nullptr;

  if (info.y == 0) {  // no page was processed for this sequence: nothing is visible
    if (out) reinterpret_cast<uint2*>(out)[lane] = make_uint2(0u, 0u);  // +0 in fp16 and bf16
    if (out_o) reinterpret_cast<float4*>(out_o)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (out_lse && lane == 0) *out_lse = -INFINITY;
    return;
  }
  if (info.y <= 1) return;  // written directly by the split-KV kernel
  if (!SQA_CHECK(info.x >= 0 && info.x + info.y <= p.num_parts, p.status, 8, s)) return;
  const size_t first = (size_t)info.x * p.piece_rows + row;
  merge_row<false>(p.parts_o + first * kHeadDim, (size_t)p.piece_rows * kHeadDim, p.parts_lse + first,
            (size_t)p.piece_rows, info.y, out, out_o, out_lse, p.bf16 != 0);
  if (threadIdx.x == 0) SQA_STAMP(tl, 2);
}

// Cross-device merge: rows given explicitly, 4 rows per CTA.
__global__ void __launch_bounds__(128) sqa_partials_merge_kernel(const MergeParams p) {
  allow_dependent_launch();
  grid_dependency_wait();
  const long long row = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  merge_row<false>(p.parts_o + row * kHeadDim, (size_t)p.rows * kHeadDim, p.parts_lse + row, (size_t)p.rows,
            p.num_parts, p.out ? p.out + row * kHeadDim : nullptr,
            p.out_o ? p.out_o + row * kHeadDim : nullptr, p.out_lse ? p.out_lse + row : nullptr, p.bf16 != 0);
}

// 128-thread launch that may overlap the previous kernel's tail (programmatic
// dependent launch); the kernel waits for it before touching memory.
cudaError_t launch_pdl(void (*kernel)(const MergeParams), dim3 grid, const MergeParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, p);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_segment_merge(const MergeParams& p, int rows_pad, cudaStream_t stream) {
  (void)rows_pad;
  const int rows = kGroup * p.q_len;
  return launch_pdl(sqa_segment_merge_kernel, dim3(p.batch * p.hkv, (rows + 3) / 4), p, stream);
}

cudaError_t launch_partials_merge(const MergeParams& p, cudaStream_t stream) {
  return launch_pdl(sqa_partials_merge_kernel, dim3((unsigned)((p.rows + 3) / 4)), p, stream);
}

}  // namespace sqa
