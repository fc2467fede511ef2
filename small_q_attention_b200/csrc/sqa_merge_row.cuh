// sqa_merge_row.cuh -- log-sum-exp merge of one output row (one warp).
//
// Used by the separate merge kernels (sqa_merge.cu).  Arithmetic of the upstream
// split-KV merge (csrc/small_q_attention_ext.cu:339-366: global max, rescale
// by exp(stat - max), sum, divide; 0 when the total weight is 0) applied to
// normalised partials with natural-log LSEs.
#pragma once

#include "sqa_internal.h"
#include "sqa_ptx.cuh"

namespace sqa {

constexpr float kMergeLog2e = 1.4426950408889634f;

// Merge `cnt` parts of one row; part i's row is at o + i * o_stride and
// lse + i * lse_stride.  Writes to whichever of out (fp16, or bf16 with
// out_bf16) / out_o / out_lse is set.
// Parts are taken kBatch at a time with all loads of a batch issued before use: one
// memory round trip per batch (8 for the usual few parts; 24 when a row has more, as
// when one sequence is split over every CTA of the GPU).
// kCoherent reads through L2 (ld.global.cg): required when the parts were
// written by other CTAs of the same kernel; otherwise the read-only path.
template <bool kCoherent, int kBatch = 8>
__device__ __forceinline__ void merge_row_batched(const float* o, size_t o_stride, const float* lse,
                                                  size_t lse_stride, int cnt, __half* out, float* out_o,
                                                  float* out_lse, bool out_bf16) {
  const int lane = threadIdx.x & 31;
  auto load_f = [](const float* ptr) { return kCoherent ? __ldcg(ptr) : __ldg(ptr); };
  auto load_f4 = [](const float4* ptr) { return kCoherent ? __ldcg(ptr) : __ldg(ptr); };
  // Batches of 8 parts, every load of a batch in flight at once (one memory
  // round trip per batch); a running max rescales what earlier batches summed.
  // With at most 8 parts this is: global max, weights exp(lse_i - max), sum.
  float base = -INFINITY, total = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i0 = 0; i0 < cnt; i0 += kBatch) {
    float4 v[kBatch];
    float l[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const bool ok = i0 + j < cnt;
      v[j] = ok ? load_f4(reinterpret_cast<const float4*>(o + (i0 + j) * o_stride) + lane)
                : make_float4(0.f, 0.f, 0.f, 0.f);
      l[j] = ok ? load_f(lse + (i0 + j) * lse_stride) : -INFINITY;
    }
    float mx = base;
#pragma unroll
    for (int j = 0; j < kBatch; ++j) mx = fmaxf(mx, l[j]);
    if (mx == -INFINITY) continue;  // nothing visible so far
    if (mx > base && base != -INFINITY) {
      const float scale = ex2((base - mx) * kMergeLog2e);
      total *= scale;
      acc.x *= scale;
      acc.y *= scale;
      acc.z *= scale;
      acc.w *= scale;
    }
    base = mx;
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const float wgt = ex2((l[j] - base) * kMergeLog2e);  // -inf -> 0
      total += wgt;
      acc.x += wgt * v[j].x;
      acc.y += wgt * v[j].y;
      acc.z += wgt * v[j].z;
      acc.w += wgt * v[j].w;
    }
  }
  const float inv = (total > 0.f) ? 1.f / total : 0.f;
  acc.x *= inv;
  acc.y *= inv;
  acc.z *= inv;
  acc.w *= inv;
  if (out != nullptr) {
    uint2 h;
    h.x = out_bf16 ? pack_bf162(acc.x, acc.y) : pack_half2(acc.x, acc.y);
    h.y = out_bf16 ? pack_bf162(acc.z, acc.w) : pack_half2(acc.z, acc.w);
    reinterpret_cast<uint2*>(out)[lane] = h;
  }
  if (out_o != nullptr) reinterpret_cast<float4*>(out_o)[lane] = acc;
  if (out_lse != nullptr && lane == 0) *out_lse = (total > 0.f) ? base + __logf(total) : -INFINITY;
}

template <bool kCoherent>
__device__ __forceinline__ void merge_row(const float* o, size_t o_stride, const float* lse,
                                          size_t lse_stride, int cnt, __half* out, float* out_o,
                                          float* out_lse, bool out_bf16 = false) {
  if (cnt <= 8)
    merge_row_batched<kCoherent, 8>(o, o_stride, lse, lse_stride, cnt, out, out_o, out_lse, out_bf16);
  else
    merge_row_batched<kCoherent, 24>(o, o_stride, lse, lse_stride, cnt, out, out_o, out_lse, out_bf16);
}

}  // namespace sqa
