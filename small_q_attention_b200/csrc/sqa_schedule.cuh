// sqa_schedule.cuh -- the device-side split-KV schedule shared by both kernels.
//
// One unit is one 16-token page of one KV head of one sequence; the units of
// (b, kvh) form segment s = b * Hkv + kvh.  All units are laid end to end and
// cut into gridDim.x ranges of equal cost, one per CTA; each (CTA, segment)
// overlap is a "piece".  The cost of a range is its units plus p.seg_cost for
// every segment that starts in it: a CTA that crosses into a new segment pays
// one more piece epilogue and a pipeline refill, so it gets fewer pages.  Warp
// 0 of every CTA derives its range from seq_lens with a warp scan, so the host
// never synchronises.
#pragma once

#include "sqa_internal.h"
#include "sqa_ptx.cuh"

namespace sqa {

// The charge for a segment start, only when the average range is at least 64
// units: on calls of a few pages per CTA any charge rounds the busiest CTA's
// share up by a page or more, which costs more than the extra epilogue.
__device__ __forceinline__ int segment_cost(int seg_cost, long long total_units, int grid) {
  return total_units >= 64LL * grid ? seg_cost : 0;
}

struct SegWalk {
  int b;          // sequence
  int h;          // KV head
  int pg;         // first page of the current piece within the segment
  int pages;      // pages of sequence b (clamped to the table width)
  int seg_start;  // global unit index of (b, h, page 0)
};

// kSpec: a read before the dependency wait, through L2 only (ld.global.cg), so
// that no possibly stale line is left in L1 for the reads after the wait.
template <bool kSpec = false>
__device__ __forceinline__ int load_len(const SplitKvParams& p, int b) {
  return kSpec ? __ldcg(p.seq_lens + b) : __ldg(p.seq_lens + b);
}

template <bool kSpec = false>
__device__ __forceinline__ int seq_pages(const SplitKvParams& p, int b) {
  const int len = max(load_len<kSpec>(p, b), 0);
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
  int per_cta;         // cost per CTA (units + p.seg_cost per segment start)
  int b0, u_b0;        // sequence containing `start` and the units before it
  int pages_b0;        // pages of sequence b0
  int abort;           // set by a timed-out wait
};

// Whole warp: total units, this CTA's range and the sequence it starts in
// (every lane gets the result).  Each lane reads the lengths of its sequences
// once: the first kCachedChunks chunks of 32 sequences stay in registers for
// the prefix scan, so a batch of up to 128 costs one memory round trip.
// kSpec: computed before the dependency wait from values that may be stale,
// for prefetches only; no status is raised.
template <bool kSpec>
__device__ __forceinline__ Schedule compute_schedule(const SplitKvParams& p) {
  constexpr int kCachedChunks = 4;
  const int lane = threadIdx.x & 31;
  unsigned int flags = 0;
  int total_pages = 0;
  int cached[kCachedChunks];
  auto pages_of = [&](int b, unsigned int& fl) {
    int pages = 0;
    if (b < p.batch) {
      const int len = load_len<kSpec>(p, b);
      pages = min((max(len, 0) + kPageSize - 1) / kPageSize, p.max_pages);
      if (len > p.max_pages * kPageSize) fl |= 2u;                 // SQA_DEV_SEQ_TOO_LONG
      if (p.out != nullptr && len < p.q_len) fl |= 4u;             // SQA_DEV_SEQ_TOO_SHORT
    }
    return pages;
  };
  auto warp_sum = [](int v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
  };
#pragma unroll
  for (int c = 0; c < kCachedChunks; ++c) {  // every load of the cached chunks in flight at once
    cached[c] = pages_of(c * 32 + lane, flags);
  }
#pragma unroll
  for (int c = 0; c < kCachedChunks; ++c) total_pages += warp_sum(cached[c]);
  for (int base = kCachedChunks * 32; base < p.batch; base += 32) total_pages += warp_sum(pages_of(base + lane, flags));
  if (!kSpec) {
    flags = __reduce_or_sync(0xffffffffu, flags);
    if (blockIdx.x == 0 && lane == 0 && flags) atomicOr(p.status, flags);
  }

  // cost of sequence b: Hkv segments of (pages + seg_cost) when it has pages (32-bit:
  // the host bounds batch x Hkv x (max_pages + seg_cost) by 2^30)
  const int total_units = total_pages * p.hkv;
  const int seg_cost = (int)segment_cost(p.seg_cost, total_units, gridDim.x);
  int nonempty = 0;
  if (seg_cost > 0) {
#pragma unroll
    for (int c = 0; c < kCachedChunks; ++c) nonempty += __popc(__ballot_sync(0xffffffffu, cached[c] > 0));
    for (int base = kCachedChunks * 32; base < p.batch; base += 32) {
      unsigned int unused = 0;
      nonempty += __popc(__ballot_sync(0xffffffffu, pages_of(base + lane, unused) > 0));
    }
  }
  const int total_cost = total_units + seg_cost * nonempty * p.hkv;
  const int per = max(1, (total_cost + (int)gridDim.x - 1) / (int)gridDim.x);
  const int x0 = min(total_cost, (int)blockIdx.x * per);
  const int x1 = min(total_cost, x0 + per);

  // Locate both ends: the sequence whose cost span holds x, then the head and the
  // unit offset (cost positions in a segment's first seg_cost map to its start;
  // with seg_cost 0 cost and units coincide).
  int start = total_units, end = total_units;
  int b0 = p.batch, u_b0 = 0, pages_b0 = 0;
  if (seg_cost == 0) {
    start = x0;
    end = x1;
  }
  if (x0 < x1) {
    int run_cost = 0, run_units = 0;
    bool found0 = false;
    for (int base = 0; base < p.batch; base += 32) {
      const int c = base / 32;
      int pg = 0;
#pragma unroll
      for (int k = 0; k < kCachedChunks; ++k)
        if (k == c) pg = cached[k];
      if (c >= kCachedChunks) {
        unsigned int unused = 0;
        pg = pages_of(base + lane, unused);
      }
      const int units = pg * p.hkv;
      const int cost = pg > 0 ? (pg + seg_cost) * p.hkv : 0;
      int incl = cost, incl_u = units;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        const int yu = __shfl_up_sync(0xffffffffu, incl_u, off);
        if (lane >= off) {
          incl += y;
          incl_u += yu;
        }
      }
      // unit position of cost x inside lane l's sequence (evaluated by every lane for lane l)
      auto unit_at = [&](int x, int l) {
        const int xr = x - run_cost - __shfl_sync(0xffffffffu, incl - cost, l);  // cost into sequence
        const int pgl = __shfl_sync(0xffffffffu, pg, l);
        const int span = pgl + seg_cost;
        const int h = xr / span;
        const int r = xr - h * span;
        return run_units + __shfl_sync(0xffffffffu, incl_u - units, l) + h * pgl + max(r - seg_cost, 0);
      };
      if (!found0) {
        const unsigned hit = __ballot_sync(0xffffffffu, run_cost + incl > x0);
        if (hit) {
          const int l = __ffs(hit) - 1;
          if (seg_cost > 0) start = unit_at(x0, l);
          b0 = base + l;
          u_b0 = run_units + __shfl_sync(0xffffffffu, incl_u - units, l);
          pages_b0 = __shfl_sync(0xffffffffu, pg, l);
          found0 = true;
          if (seg_cost == 0) break;  // end = x1 already
        }
      }
      if (found0) {
        const unsigned hit = __ballot_sync(0xffffffffu, run_cost + incl > x1);
        if (hit) {
          end = unit_at(x1, __ffs(hit) - 1);
          break;
        }
      }
      run_cost += __shfl_sync(0xffffffffu, incl, 31);
      run_units += __shfl_sync(0xffffffffu, incl_u, 31);
    }
  }
  Schedule s;
  s.start = start;
  s.end = max(start, end);
  s.per_cta = (int)per;
  s.b0 = b0;
  s.u_b0 = u_b0;
  s.pages_b0 = pages_b0;
  s.abort = 0;
  return s;
}

// Pages per CTA when a segment of `pages` pages is split evenly over `parts` CTAs:
// in whole 4-page blocks in cluster mode, to the page in the segment-aligned split.
// CTA j of the segment takes [min(pages, j * per), min(pages, (j + 1) * per)), so
// the CTAs with pages are j < ceil(pages / per).
__device__ __forceinline__ int even_split_pages(int pages, int parts, bool whole_blocks) {
  const int per = (pages + parts - 1) / parts;
  return whole_blocks ? (per + 3) / 4 * 4 : per;
}

// Even split of every segment over C CTAs (tcgen05 kernel): cluster mode
// (p.cluster = C >= 2, whole 4-page blocks) or the segment-aligned split
// (p.seg_split = C >= 2, to the page).  CTA blockIdx.x works on segment
// s = blockIdx.x / C, the (blockIdx.x % C)-th of C page ranges (a range may be
// empty), so no CTA crosses a segment boundary.  Whole warp; every lane gets the
// result.  Lengths are read once; block 0 raises the same status bits as
// compute_schedule.
template <bool kSpec>
__device__ __forceinline__ Schedule even_schedule(const SplitKvParams& p) {
  const int lane = threadIdx.x & 31;
  const int C = p.cluster > 1 ? p.cluster : p.seg_split;
  const int seg = (int)blockIdx.x / C;
  const int k = (int)blockIdx.x - seg * C;
  const int b = seg / p.hkv;
  const int h = seg - b * p.hkv;
  unsigned int flags = 0;
  int before = 0, pages_b = 0;
  for (int base = 0; base < p.batch; base += 32) {
    const int i = base + lane;
    int pg = 0;
    if (i < p.batch) {
      const int len = load_len<kSpec>(p, i);
      pg = min((max(len, 0) + kPageSize - 1) / kPageSize, p.max_pages);
      if (len > p.max_pages * kPageSize) flags |= 2u;      // SQA_DEV_SEQ_TOO_LONG
      if (p.out != nullptr && len < p.q_len) flags |= 4u;  // SQA_DEV_SEQ_TOO_SHORT
    }
    int pre = (i < b) ? pg : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, off);
    before += pre;
    if (b >= base && b < base + 32) pages_b = __shfl_sync(0xffffffffu, pg, b - base);
  }
  if (!kSpec) {
    flags = __reduce_or_sync(0xffffffffu, flags);
    if (blockIdx.x == 0 && lane == 0 && flags) atomicOr(p.status, flags);
  }
  const int per = even_split_pages(pages_b, C, p.cluster > 1);
  const int lo = min(pages_b, k * per);
  const int hi = min(pages_b, lo + per);
  Schedule sch;
  sch.b0 = b < p.batch ? b : p.batch;
  sch.u_b0 = before * p.hkv;  // units of the sequences before b
  sch.pages_b0 = pages_b;
  const int seg_start = sch.u_b0 + h * pages_b;
  sch.start = seg_start + lo;
  sch.end = seg_start + hi;
  sch.per_cta = per;
  sch.abort = 0;
  return sch;
}

// Warp 0: the schedule into shared memory, before the CTA-wide barrier.
__device__ __forceinline__ void build_schedule(const SplitKvParams& p, Schedule* sch) {
  const Schedule s = (p.cluster || p.seg_split) ? even_schedule<false>(p) : compute_schedule<false>(p);
  if ((threadIdx.x & 31) == 0) *sch = s;
}

__device__ __forceinline__ SegWalk first_segment(const SplitKvParams& p, const Schedule& s) {
  SegWalk w;
  w.b = s.b0;
  w.pages = (s.start < s.end) ? s.pages_b0 : 1;
  const int off = s.start - s.u_b0;
  w.h = off / w.pages;
  w.pg = off - w.h * w.pages;
  w.seg_start = s.u_b0 + w.h * w.pages;
  return w;
}

// Whole warp: the pieces of segment (b, h) under the schedule of a split-KV
// launch of `grid` CTAs — the first piece's workspace slot (first CTA + segment
// index) and the number of pieces — from the same cost mapping as
// compute_schedule (every lane gets the result; batch up to 128 reads each
// length once).  For the merge kernel, which may run this before its
// dependency wait: seq_lens is an input the split kernel does not write.
__device__ __forceinline__ int2 segment_pieces(const int32_t* seq_lens, int batch, int max_pages, int hkv,
                                               int seg_cost, int grid, int b, int h) {
  constexpr int kCachedChunks = 4;
  const int lane = threadIdx.x & 31;
  auto pages_of = [&](int i) {
    if (i >= batch) return 0;
    const int len = max(__ldcg(seq_lens + i), 0);
    return min((len + kPageSize - 1) / kPageSize, max_pages);
  };
  int cached[kCachedChunks];
#pragma unroll
  for (int c = 0; c < kCachedChunks; ++c) cached[c] = pages_of(c * 32 + lane);
  long long total_pages = 0, pages_before = 0;
  int nonempty = 0, nonempty_before = 0, pages_b = 0;
  for (int base = 0; base < batch; base += 32) {
    const int c = base / 32;
    int pg = 0;
#pragma unroll
    for (int k = 0; k < kCachedChunks; ++k)
      if (k == c) pg = cached[k];
    if (c >= kCachedChunks) pg = pages_of(base + lane);
    const int i = base + lane;
    int sum = pg, before = (i < b) ? pg : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, off);
      before += __shfl_xor_sync(0xffffffffu, before, off);
    }
    total_pages += sum;
    pages_before += before;
    nonempty += __popc(__ballot_sync(0xffffffffu, pg > 0));
    nonempty_before += __popc(__ballot_sync(0xffffffffu, pg > 0 && i < b));
    const unsigned hit = __ballot_sync(0xffffffffu, i == b);
    if (hit) pages_b = __shfl_sync(0xffffffffu, pg, __ffs(hit) - 1);
  }
  if (pages_b == 0) return make_int2(0, 0);
  const int c = segment_cost(seg_cost, total_pages * hkv, grid);
  const int total_cost = (int)total_pages * hkv + c * nonempty * hkv;
  const int per = max(1, (total_cost + grid - 1) / grid);
  const int ne = nonempty_before * hkv + h;                            // non-empty segments before (b, h)
  const int seg_start = (int)pages_before * hkv + h * pages_b;
  const int first_cost = seg_start + c * (ne + 1);
  const int first_cta = first_cost / per;
  const int last_cta = (first_cost + pages_b - 1) / per;
  return make_int2(first_cta + b * hkv + h, last_cta - first_cta + 1);
}

// The pieces of segment s = b * Hkv + h under the segment-aligned split of k CTAs per
// segment: CTA s * k + j writes piece slot (CTA + segment) = s * (k + 1) + j, and the
// CTAs with pages are j < ceil(pages / per) (even_split_pages).  Whole warp (every
// lane reads the one length).
__device__ __forceinline__ int2 aligned_segment_pieces(const int32_t* seq_lens, int max_pages, int hkv, int k,
                                                       int b, int h) {
  const int len = max(__ldcg(seq_lens + b), 0);
  const int pages = min((len + kPageSize - 1) / kPageSize, max_pages);
  if (pages == 0) return make_int2(0, 0);
  const int per = even_split_pages(pages, k, false);
  return make_int2((b * hkv + h) * (k + 1), (pages + per - 1) / per);
}

// Producer warp, before the dependency wait: L2 prefetches of the first
// `budget` pages (at most 32 per segment, two segments at most) and the first
// Q rows this CTA will load, from a schedule and page ids read through L2
// while the previous grid may still be running.  Those values may
// be stale: they only steer prefetches (nothing is consumed or written, and a
// page id outside the pool is skipped), and every value is read again after
// the wait.  The loads after the wait then find their lines in L2.
template <bool F8>
__device__ __forceinline__ void prefetch_start(const SplitKvParams& p, const CUtensorMap* tm_k,
                                               const CUtensorMap* tm_v, int budget) {
  const int lane = threadIdx.x & 31;
  const Schedule s = (p.cluster || p.seg_split) ? even_schedule<true>(p) : compute_schedule<true>(p);
  if (s.start >= s.end) return;
  int b = s.b0;
  int pages = s.pages_b0;
  if (pages <= 0) return;
  const int off = s.start - s.u_b0;
  int h = off / pages;
  int pg = off - h * pages;
  if (h >= p.hkv) return;
  if (lane < p.q_len) {  // the 4 query heads of (b, h) for draft token `lane`: 1 KB
    bulk_prefetch_l2(p.q + ((size_t)(b * p.q_len + lane) * p.hq + h * kGroup) * kHeadDim,
                     kGroup * kHeadDim * 2);
  }
  int unit = s.start;
  for (int seg = 0; seg < 2 && budget > 0 && unit < s.end; ++seg) {
    const int m = min(min(pages - pg, s.end - unit), min(budget, 32));
    if (lane < m) {
      const int id = __ldcg(p.block_tables + (size_t)b * p.max_pages + pg + lane);
      if (id >= 0 && id < p.num_pages) {
        const int k1 = p.hnd ? 0 : h, k2 = p.hnd ? h : 0;  // NHD (dim, head, token, page); HND (dim, token, head, page)
        if constexpr (F8) {  // fp8 maps: one 128-dim box per page
          tma_prefetch_4d(tm_k, 0, k1, k2, id);
          tma_prefetch_4d(tm_v, 0, k1, k2, id);
        } else {  // 16-bit maps: two 64-dim boxes per page
          tma_prefetch_4d(tm_k, 0, k1, k2, id);
          tma_prefetch_4d(tm_k, 64, k1, k2, id);
          tma_prefetch_4d(tm_v, 0, k1, k2, id);
          tma_prefetch_4d(tm_v, 64, k1, k2, id);
        }
      }
    }
    budget -= m;
    unit += m;
    pg += m;
    if (pg >= pages) {  // the next segment: next KV head, or the next sequence with pages
      pg = 0;
      if (++h == p.hkv) {
        h = 0;
        do {
          ++b;
          pages = (b < p.batch) ? seq_pages<true>(p, b) : 0;
        } while (pages == 0 && b < p.batch);
        if (b >= p.batch) break;
      }
    }
  }
}

}  // namespace sqa
