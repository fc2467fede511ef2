// sqa_schedule.cuh -- the device-side split-KV schedule shared by both kernels.
//
// One unit is one 16-token page of one KV head of one sequence; the units of
// (b, kvh) form segment s = b * Hkv + kvh.  All units are laid end to end and
// cut into gridDim.x equal ranges, one per CTA; each (CTA, segment) overlap is
// a "piece".  Warp 0 of every CTA derives its range from seq_lens with a warp
// scan, so the host never synchronises.
#pragma once

#include "sqa_internal.h"
#include "sqa_ptx.cuh"

namespace sqa {

struct SegWalk {
  int b;          // sequence
  int h;          // KV head
  int pg;         // first page of the current piece within the segment
  int pages;      // pages of sequence b (clamped to the table width)
  int seg_start;  // global unit index of (b, h, page 0)
};

__device__ __forceinline__ int seq_pages(const SplitKvParams& p, int b) {
  const int len = max(__ldg(p.seq_lens + b), 0);
  return min((len + kPageSize - 1) / kPageSize, p.max_pages);
}

__device__ __forceinline__ void next_segment(const SplitKvParams& p, SegWalk& w) {
  w.seg_start += w.pages;
  w.pg = 0;
  if (++w.h == p.hkv) {
    w.h = 0;
    do {
      ++w.b;
      w.pages = (w.b < p.batch) ? seq_pages(p, w.b) : 0;
    } while (w.pages == 0 && w.b < p.batch);
  }
}

// Shared schedule, filled by warp 0 before the CTA-wide barrier.
struct Schedule {
  int start, end;      // this CTA's unit range
  int per_cta;         // units per CTA
  int b0, u_b0;        // sequence containing `start` and the units before it
  int abort;           // set by a timed-out wait
};

// Warp 0: total units, this CTA's range and the sequence it starts in.
__device__ __forceinline__ void build_schedule(const SplitKvParams& p, Schedule* sch) {
  const int lane = threadIdx.x & 31;
  unsigned int flags = 0;
  int total_pages = 0;
  for (int base = 0; base < p.batch; base += 32) {
    const int b = base + lane;
    int pages = 0;
    if (b < p.batch) {
      const int len = __ldg(p.seq_lens + b);
      pages = seq_pages(p, b);
      if (len > p.max_pages * kPageSize) flags |= 2u;                 // SQA_DEV_SEQ_TOO_LONG
      if (p.out != nullptr && len < p.q_len) flags |= 4u;             // SQA_DEV_SEQ_TOO_SHORT
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) pages += __shfl_xor_sync(0xffffffffu, pages, off);
    total_pages += pages;
  }
  flags = __reduce_or_sync(0xffffffffu, flags);
  if (blockIdx.x == 0 && lane == 0 && flags) atomicOr(p.status, flags);

  const int total = total_pages * p.hkv;
  const int per = max(1, (total + (int)gridDim.x - 1) / (int)gridDim.x);
  const int start = min(total, (int)blockIdx.x * per);
  const int end = min(total, start + per);

  // Sequence containing unit `start`: first b whose inclusive unit prefix exceeds it.
  int b0 = p.batch, u_b0 = 0;
  if (start < end) {
    int running = 0;  // units before this 32-sequence block
    for (int base = 0; base < p.batch; base += 32) {
      const int b = base + lane;
      const int units = (b < p.batch) ? seq_pages(p, b) * p.hkv : 0;
      int incl = units;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, running + incl > start);
      if (hit) {
        const int l = __ffs(hit) - 1;
        b0 = base + l;
        u_b0 = running + __shfl_sync(0xffffffffu, incl - units, l);
        break;
      }
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (lane == 0) {
    sch->start = start;
    sch->end = end;
    sch->per_cta = per;
    sch->b0 = b0;
    sch->u_b0 = u_b0;
    sch->abort = 0;
  }
}

__device__ __forceinline__ SegWalk first_segment(const SplitKvParams& p, const Schedule& s) {
  SegWalk w;
  w.b = s.b0;
  w.pages = (s.start < s.end) ? seq_pages(p, s.b0) : 1;
  const int off = s.start - s.u_b0;
  w.h = off / w.pages;
  w.pg = off - w.h * w.pages;
  w.seg_start = s.u_b0 + w.h * w.pages;
  return w;
}

}  // namespace sqa
