// sqa_merge.cu -- log-sum-exp merge of split-KV partials.
//
// One warp merges one output row: lanes load the parts' log-sum-exps 32 at a
// time, take the max, and each lane then accumulates a float4 column of the
// 128-dim row over the parts with weights exp(lse_i - LSE).  A row whose parts
// all have lse = -inf (no visible key) is written as 0 (and -inf).  This is
// the arithmetic of the upstream split-KV merge
// (csrc/small_q_attention_ext.cu:339-366: global max, rescale, sum, divide,
// 0 when the denominator is 0) on normalised partials.
#include "sqa_internal.h"
#include "sqa_ptx.cuh"

namespace sqa {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Merge `cnt` parts of one row; part i's row is at o + i * o_stride and
// lse + i * lse_stride.  Writes to whichever of out / out_o / out_lse is set.
__device__ __forceinline__ void merge_row(const float* o, size_t o_stride, const float* lse,
                                          size_t lse_stride, int cnt, __half* out, float* out_o,
                                          float* out_lse) {
  const int lane = threadIdx.x & 31;
  float mmax = -INFINITY;
  for (int i = lane; i < cnt; i += 32) mmax = fmaxf(mmax, __ldg(lse + i * lse_stride));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, off));
  const float base = (mmax == -INFINITY) ? 0.f : mmax;

  float total = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i0 = 0; i0 < cnt; i0 += 32) {
    const int i = i0 + lane;
    const float wl = (i < cnt) ? ex2((__ldg(lse + i * lse_stride) - base) * kLog2e) : 0.f;
    const int m = min(32, cnt - i0);
    for (int j = 0; j < m; ++j) {
      const float wgt = __shfl_sync(0xffffffffu, wl, j);
      total += wgt;
      const float4 v = __ldg(reinterpret_cast<const float4*>(o + (i0 + j) * o_stride) + lane);
      acc.x += wgt * v.x;
      acc.y += wgt * v.y;
      acc.z += wgt * v.z;
      acc.w += wgt * v.w;
    }
  }
  const float inv = (total > 0.f) ? 1.f / total : 0.f;
  acc.x *= inv;
  acc.y *= inv;
  acc.z *= inv;
  acc.w *= inv;
  if (out != nullptr) {
    uint2 h;
    h.x = pack_half2(acc.x, acc.y);
    h.y = pack_half2(acc.z, acc.w);
    reinterpret_cast<uint2*>(out)[lane] = h;
  }
  if (out_o != nullptr) reinterpret_cast<float4*>(out_o)[lane] = acc;
  if (out_lse != nullptr && lane == 0) *out_lse = (total > 0.f) ? base + __logf(total) : -INFINITY;
  (void)kLn2;
}

// Per-call merge: grid (B * Hkv, ceil(4 * q_len / 4)), 4 warps = 4 rows per CTA.
__global__ void __launch_bounds__(128) sqa_segment_merge_kernel(const MergeParams p) {
  const int s = blockIdx.x;
  const int b = s / p.hkv;
  const int h = s - b * p.hkv;
  const int rows = kGroup * p.q_len;
  const int row = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const size_t out_row = (size_t)(b * p.q_len + (row >> 2)) * p.hq + h * kGroup + (row & 3);
  __half* out = p.out ? p.out + out_row * kHeadDim : nullptr;
  float* out_o = p.out_o ? p.out_o + out_row * kHeadDim : nullptr;
  float* out_lse = p.out_lse ? p.out_lse + out_row : nullptr;

  const int len = max(__ldg(p.seq_lens + b), 0);
  if (len == 0) {  // no page was processed for this sequence: nothing is visible
    if (out) reinterpret_cast<uint2*>(out)[lane] = make_uint2(0u, 0u);
    if (out_o) reinterpret_cast<float4*>(out_o)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (out_lse && lane == 0) *out_lse = -INFINITY;
    return;
  }
  const int2 info = p.seg_info[s];
  if (info.y <= 1) return;  // written directly by the split-KV kernel
  if (!SQA_CHECK(info.x >= 0 && info.x + info.y <= p.num_parts, p.status, 8, s)) return;
  const size_t first = (size_t)info.x * p.piece_rows + row;
  merge_row(p.parts_o + first * kHeadDim, (size_t)p.piece_rows * kHeadDim, p.parts_lse + first,
            (size_t)p.piece_rows, info.y, out, out_o, out_lse);
}

// Cross-device merge: rows given explicitly, 4 rows per CTA.
__global__ void __launch_bounds__(128) sqa_partials_merge_kernel(const MergeParams p) {
  const long long row = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  merge_row(p.parts_o + row * kHeadDim, (size_t)p.rows * kHeadDim, p.parts_lse + row, (size_t)p.rows,
            p.num_parts, p.out ? p.out + row * kHeadDim : nullptr,
            p.out_o ? p.out_o + row * kHeadDim : nullptr, p.out_lse ? p.out_lse + row : nullptr);
}

}  // namespace

cudaError_t launch_segment_merge(const MergeParams& p, int rows_pad, cudaStream_t stream) {
  (void)rows_pad;
  const int rows = kGroup * p.q_len;
  const dim3 grid(p.batch * p.hkv, (rows + 3) / 4);
  sqa_segment_merge_kernel<<<grid, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_partials_merge(const MergeParams& p, cudaStream_t stream) {
  const long long blocks = (p.rows + 3) / 4;
  sqa_partials_merge_kernel<<<(unsigned)blocks, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace sqa
