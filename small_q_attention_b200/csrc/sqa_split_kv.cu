// sqa_split_kv.cu -- the split-KV paged attention kernel for sm_100a.
//
// Work decomposition.  One "unit" is one 16-token page of one KV head of one
// sequence; the units of (b, kvh) form segment s = b * Hkv + kvh.  All units
// are laid end to end and cut into gridDim.x ranges of equal cost (units plus
// a fixed charge per segment start, sqa_schedule.cuh), one per CTA, so every
// CTA streams about the same number of K/V bytes whatever the mix of lengths
// (a ragged batch balances like a uniform one).  A CTA range may end inside a
// segment or cover several short ones; each (CTA, segment) overlap is a
// "piece".  A piece that is a whole segment writes the final output directly;
// otherwise it writes a normalised fp32 partial and its log-sum-exp to slot
// (blockIdx.x + s) of the workspace and the merge kernel combines them.  The
// schedule is derived on the device from seq_lens, so the host never
// synchronises.  (Upstream equivalent: a fixed chunk_keys split with
// ceil(max_len / chunk_keys) chunks per row, csrc/small_q_attention_ext.cu:1178.)
//
// Data movement.  Warp 4 is the TMA producer: for each page it reads the page
// id (32 ids per coalesced load, the next 32 prefetched), waits for a free
// stage of the shared-memory ring and issues four 2 KB tensor loads (K and V,
// two 64-dim halves each, 128-byte swizzled) that complete on the stage's
// mbarrier.  Each K/V byte therefore crosses HBM exactly once per KV head
// (the upstream v3 kernel re-reads K/V for every query row, ext.cu:462-508).
//
// Math.  Warps 0-3 are consumers.  The 4 query heads x q_len draft rows of a
// KV head are packed as the N side of mma.sync m16n8k16 with the 16 tokens
// of a page as M ("swapped" orientation): S^T = K_page . Q^T, so q_len = 2
// (8 rows) fills the n8 tile with no padding.  The fp32 online softmax works
// on the S^T fragments (row max over tokens = 3 shuffles), probabilities are
// packed to fp16 and transposed in registers with movmatrix into the B
// operand of O^T += V^T_page . P^T.  Q lives in registers for a whole piece.
#include "sqa_internal.h"
#include "sqa_ptx.cuh"
#include "sqa_schedule.cuh"

namespace sqa {
namespace {

constexpr float kLn2 = 0.6931471805599453f;

// ------------------------------------------------------------------ producer
// Ring protocol.  Page i (the CTA's i-th page) goes to data stage i % S and
// completes on full barrier i % (2S); its stage is released on empty barrier
// i % S.  The token groups consume pages out of order, so one stage's
// consecutive fills are waited on by different groups.  With full barriers
// indexed modulo 2S, the previous fill of barrier i % 2S is page i - 2S, which
// is always complete when page i is awaited (page i - S has been issued,
// which needed page i - 2S consumed), so a parity wait sees only the two
// phases it can tell apart.
#ifdef SQA_DEBUG_CHECKS
__shared__ volatile int debug_progress[4];
#endif

__device__ void producer_loop(const SplitKvParams& p, const Schedule& sch, const CUtensorMap* tm_k,
                              const CUtensorMap* tm_v, uint8_t* stages, uint64_t* full,
                              uint64_t* empty, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_policy_evict_first();
  const int S = p.num_stages;
  SegWalk w = first_segment(p, sch);
  int slot = 0, fslot = 0;  // data stage i % S, full barrier i % 2S
  uint32_t phase = 0;
  unsigned int bad_page = 0;
  int issued = 0;  // pages whose loads were issued (a prefix of the range)
  int unit = sch.start;
  // Page ids are read 32 at a time, one chunk ahead of the loads they feed,
  // across piece boundaries too: a new piece never waits for its table row.
  int ids = 0;
  if (unit < sch.end) {
    const int n0 = min(sch.end, w.seg_start + w.pages) - unit;
    ids = (lane < n0) ? __ldg(p.block_tables + (size_t)w.b * p.max_pages + w.pg + lane) : 0;
  }
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int32_t* row = p.block_tables + (size_t)w.b * p.max_pages + w.pg;
    const int unit_next = unit + n;  // the next piece, for the look-ahead at this piece's last chunk
    SegWalk wn = w;
    if (unit_next < sch.end) next_segment(p, wn);
    for (int c0 = 0; c0 < n; c0 += 32) {
      const int cnt = min(32, n - c0);
      int ids_next = 0;
      if (c0 + 32 < n) {
        ids_next = (c0 + 32 + lane < n) ? __ldg(row + c0 + 32 + lane) : 0;
      } else if (unit_next < sch.end) {
        const int n2 = min(sch.end, wn.seg_start + wn.pages) - unit_next;
        ids_next = (lane < n2) ? __ldg(p.block_tables + (size_t)wn.b * p.max_pages + wn.pg + lane) : 0;
      }
      for (int j = 0; j < cnt; ++j) {
        int page = __shfl_sync(0xffffffffu, ids, j);
        if (page < 0 || page >= p.num_pages) {
          bad_page = 1;
          page = 0;  // never hand TMA a coordinate outside the pool
        }
        const bool in_range = SQA_CHECK(slot < S && fslot < 2 * S, p.status, 1, slot) &&
                              SQA_CHECK(w.b < p.batch && w.h < p.hkv, p.status, 2, w.b) &&
                              SQA_CHECK(w.pg + c0 + j < p.max_pages, p.status, 3, w.pg + c0 + j);
        if (lane == 0 && in_range) {
          const bool got = mbar_wait_bounded(smem_u32(empty + slot), phase ^ 1u, abort, p.status, 1, issued);
#ifdef SQA_DEBUG_CHECKS
          if (!got && p.status[2] == 1u && p.status[4] == blockIdx.x && atomicCAS(p.status + 10, 0u, 1u) == 0u) {
            unsigned int fb = 0, eb = 0;  // phase bits of every barrier
            for (int k2 = 0; k2 < 2 * S; ++k2) {
              uint64_t r;
              asm volatile("ld.shared.b64 %0, [%1];" : "=l"(r) : "r"(smem_u32(full + k2)));
              fb |= (unsigned int)(r >> 63) << k2;
            }
            for (int k2 = 0; k2 < S; ++k2) {
              uint64_t r;
              asm volatile("ld.shared.b64 %0, [%1];" : "=l"(r) : "r"(smem_u32(empty + k2)));
              eb |= (unsigned int)(r >> 63) << k2;
            }
            p.status[15] = fb;
            p.status[16] = eb;
            for (int k2 = 0; k2 < 4; ++k2) p.status[11 + k2] = debug_progress[k2];
          }
#endif
          if (got) {
            const uint32_t f = smem_u32(full + fslot);
            mbar_arrive_expect_tx(f, kStageBytes);
            const uint32_t dst = smem_u32(stages + (size_t)slot * kStageBytes);
            // NHD map: (dim, head, token, page); HND map: (dim, token, head, page)
            const int c1 = p.hnd ? 0 : w.h;
            const int c2 = p.hnd ? w.h : 0;
            tma_load_4d(dst, tm_k, f, 0, c1, c2, page, policy);
            tma_load_4d(dst + 2048, tm_k, f, 64, c1, c2, page, policy);
            tma_load_4d(dst + 4096, tm_v, f, 0, c1, c2, page, policy);
            tma_load_4d(dst + 6144, tm_v, f, 64, c1, c2, page, policy);
            ++issued;
          }
        }
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
        if (++fslot == 2 * S) fslot = 0;
      }
      ids = ids_next;
    }
    unit = unit_next;
    w = wn;
  }
  if (__any_sync(0xffffffffu, bad_page) && lane == 0) atomicOr(p.status, 8u);  // SQA_DEV_BAD_PAGE
  // No bulk copy may still be landing in this CTA's shared memory when it
  // exits.  On the normal path the consumers wait for every page, so only an
  // abort (a timed-out wait) needs this bounded drain.
  if (lane == 0 && *abort) {
    const int bars = min(issued, 2 * S);
    for (int k = 0; k < bars; ++k) {
      const int last = k + 2 * S * ((issued - 1 - k) / (2 * S));  // last page on barrier k
      if (!mbar_drain(smem_u32(full + k), (uint32_t)(last / (2 * S)) & 1u, 100000000ull))
        atomicOr(p.status, 1u);  // SQA_DEV_TIMEOUT
    }
  }
}

// ------------------------------------------------------------------ consumers
template <int NT, int WR, bool BF>
__device__ void consumer_loop(const SplitKvParams& p, const Schedule& sch, uint8_t* stages,
                              uint64_t* full, uint64_t* empty, float* cbuf, float* mbuf, float* lbuf,
                              volatile int* abort) {
  constexpr int WT = kConsumerWarps / WR;  // token groups
  constexpr int ROWS_W = 8 * NT;           // rows per warp
  constexpr int ROWS_PAD = ROWS_W * WR;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;  // 0..127 over the consumer warps
  const int wr = warp % WR;     // row slice
  const int tg = warp / WR;     // token group
  const int g = lane >> 2;      // fragment row group
  const int t = lane & 3;       // fragment column pair
  const int rows = kGroup * p.q_len;

  // ldmatrix lane addressing inside a 128-byte-swizzled [16 tok][64 dim] half tile.
  const int k_row = (lane & 7) + ((lane >> 3) & 1) * 8;  // K: token row of this lane's address
  const int k_cb = lane >> 4;                             // K: +1 chunk for matrices 2, 3
  const int v_row = (lane & 7) + (lane >> 4) * 8;         // V (trans): token row
  const int v_cb = (lane >> 3) & 1;                       // V: +1 chunk for matrices 1, 3

  SegWalk w = first_segment(p, sch);
  int slot = 0, fslot = 0;  // data stage gi % S, full barrier gi % 2S
  uint32_t fphase = 0;
  int gi = 0;  // CTA-wide page counter (selects the token group)
  int unit = sch.start;
  while (unit < sch.end) {
    const int s = w.b * p.hkv + w.h;
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const bool whole = (unit == w.seg_start) && (seg_end <= sch.end);

    const int len_raw = __ldg(p.seq_lens + w.b);
    const int len = min(len_raw, w.pages * kPageSize);
    const int mlen = p.mask_lens ? __ldg(p.mask_lens + w.b) : len_raw;
    const int thr_min = min(len, mlen - p.q_len + 1);  // visible tokens of draft row 0

    // Q^T fragments (B operand of S^T = K Q^T) for this warp's rows, and the
    // per-thread causal limits of its two fragment columns per n-tile.
    uint32_t qf[NT][8][2];
    int thr[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int row = wr * ROWS_W + nt * 8 + g;
      const bool ok = row < rows;
      const __half* qp = p.q + ((size_t)(w.b * p.q_len + (row >> 2)) * p.hq + w.h * kGroup + (row & 3)) * kHeadDim;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qf[nt][kk][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qp + kk * 16 + 2 * t)) : 0u;
        qf[nt][kk][1] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qp + kk * 16 + 8 + 2 * t)) : 0u;
      }
      const int qi = (wr * ROWS_W + nt * 8 + 2 * t) >> 2;  // both columns share qi
      thr[nt] = min(len, mlen - p.q_len + qi + 1);
    }

    float m_run[NT][2], l_run[NT][2];
    float o[8][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int md = 0; md < 8; ++md)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[md][nt][e] = 0.f;
    }

    for (int j = 0; j < n; ++j, ++gi) {
      const int my_slot = slot;
      const int my_fslot = fslot;
      const uint32_t my_fphase = fphase;
      if (++slot == p.num_stages) slot = 0;
      if (++fslot == 2 * p.num_stages) {
        fslot = 0;
        fphase ^= 1u;
      }
      if ((gi % WT) != tg) continue;
      if (!SQA_CHECK(my_slot < p.num_stages, p.status, 4, my_slot)) continue;
#ifdef SQA_DEBUG_CHECKS
      if (lane == 0) debug_progress[warp] = gi;
#endif
      mbar_wait_bounded(smem_u32(full + my_fslot), my_fphase, abort, p.status, 3, gi);
#ifdef SQA_DEBUG_TIMELINE
      if (gi == 0 && lane == 0 && p.timeline) p.timeline[(size_t)blockIdx.x * 8 + 3] = global_timer_ns();
#endif
      uint8_t* st = stages + (size_t)my_slot * kStageBytes;
      const uint32_t k_base = smem_u32(st);
      const uint32_t v_base = k_base + 4096;
      const int tok0 = (w.pg + j) * kPageSize;

      // Tokens at or past the sequence end hold whatever the pool has there:
      // zero their V rows so that p = 0 never meets a NaN/Inf.
      const bool tail = tok0 + kPageSize > len;
      if (tail) {
        const int first = max(len - tok0, 0);
        for (int c = lane; c < (kPageSize - first) * 16; c += 32) {
          const int r = first + (c >> 4);
          *reinterpret_cast<uint4*>(st + 4096 + ((c >> 3) & 1) * 2048 + r * 128 + (c & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }

      // ---- S^T[16 tok x 8*NT rows] = K_page . Q^T, two k-halves in flight
      float sa[NT][4], sb[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        const int chunk = (((kk & 3) << 1) | k_cb) ^ (k_row & 7);
        ldsm_x4(a, k_base + (kk >> 2) * 2048 + k_row * 128 + chunk * 16);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (kk & 1) mma_16816<BF>(sb[nt], a, qf[nt][kk][0], qf[nt][kk][1]);
          else mma_16816<BF>(sa[nt], a, qf[nt][kk][0], qf[nt][kk][1]);
        }
      }

      // ---- online softmax over the page's tokens (base 2, scaled)
      const bool masked = tok0 + kPageSize > thr_min;
      uint32_t pb[NT][2];
      float alpha[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x[e] = (sa[nt][e] + sb[nt][e]) * p.scale_log2;
          if (masked && tok0 + g + ((e >> 1) << 3) >= thr[nt]) x[e] = -INFINITY;
        }
        float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
        const float base0 = (mn0 == -INFINITY) ? 0.f : mn0;
        const float base1 = (mn1 == -INFINITY) ? 0.f : mn1;
        alpha[nt][0] = ex2(m_run[nt][0] - base0);
        alpha[nt][1] = ex2(m_run[nt][1] - base1);
        m_run[nt][0] = mn0;
        m_run[nt][1] = mn1;
        const float p0 = ex2(x[0] - base0), p1 = ex2(x[1] - base1);
        const float p2 = ex2(x[2] - base0), p3 = ex2(x[3] - base1);
        l_run[nt][0] = l_run[nt][0] * alpha[nt][0] + (p0 + p2);
        l_run[nt][1] = l_run[nt][1] * alpha[nt][1] + (p1 + p3);
        // [tok g | tok g+8][rows 2t, 2t+1] -> transpose -> B fragment [tok 2t.., 2t+8..][row g]
        pb[nt][0] = movmatrix_trans(pack2<BF>(p0, p1));
        pb[nt][1] = movmatrix_trans(pack2<BF>(p2, p3));
      }
      bool rescale = false;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) rescale |= (alpha[nt][0] != 1.f) | (alpha[nt][1] != 1.f);
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int md = 0; md < 8; ++md)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            o[md][nt][0] *= alpha[nt][0];
            o[md][nt][1] *= alpha[nt][1];
            o[md][nt][2] *= alpha[nt][0];
            o[md][nt][3] *= alpha[nt][1];
          }
      }

      // ---- O^T[128 dim x rows] += V^T_page . P^T
#pragma unroll
      for (int md = 0; md < 8; ++md) {
        uint32_t a[4];
        const int chunk = (((md & 3) << 1) | v_cb) ^ (v_row & 7);
        ldsm_x4_trans(a, v_base + (md >> 2) * 2048 + v_row * 128 + chunk * 16);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816<BF>(o[md][nt], a, pb[nt][0], pb[nt][1]);
      }

      if (tail) fence_proxy_async_smem();  // generic writes above vs the next TMA into this stage
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(empty + my_slot));
    }

    // ---- piece epilogue: combine the token groups through shared memory
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float l = l_run[nt][c];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][c] = l;
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int row = wr * ROWS_W + nt * 8 + 2 * t + c;
          mbuf[tg * ROWS_PAD + row] = m_run[nt][c];
          lbuf[tg * ROWS_PAD + row] = l_run[nt][c];
        }
    }
#pragma unroll
    for (int md = 0; md < 8; ++md)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = wr * ROWS_W + nt * 8 + 2 * t + (e & 1);
          const int d = md * 16 + g + ((e >> 1) << 3);
          cbuf[(tg * ROWS_PAD + row) * kCombineStride + d] = o[md][nt][e];
        }
    named_bar_sync(1, kConsumerWarps * 32);

    const int piece = (int)blockIdx.x + s;
    const bool piece_ok = whole || SQA_CHECK(piece < p.num_pieces, p.status, 5, piece);
    for (int item = tid; piece_ok && item < rows * 32; item += kConsumerWarps * 32) {
      const int row = item >> 5;
      const int c4 = (item & 31) * 4;
      float mmax = -INFINITY;
#pragma unroll
      for (int x = 0; x < WT; ++x) mmax = fmaxf(mmax, mbuf[x * ROWS_PAD + row]);
      const float base = (mmax == -INFINITY) ? 0.f : mmax;
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int x = 0; x < WT; ++x) {
        const float wgt = ex2(mbuf[x * ROWS_PAD + row] - base);
        L += wgt * lbuf[x * ROWS_PAD + row];
        const float4 v = *reinterpret_cast<const float4*>(cbuf + (x * ROWS_PAD + row) * kCombineStride + c4);
        acc.x += wgt * v.x;
        acc.y += wgt * v.y;
        acc.z += wgt * v.z;
        acc.w += wgt * v.w;
      }
      const float inv = (L > 0.f) ? p.out_scale / L : 0.f;
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
      const float lse = (L > 0.f) ? (mmax + __log2f(L)) * kLn2 : -INFINITY;
      const size_t out_row = (size_t)(w.b * p.q_len + (row >> 2)) * p.hq + w.h * kGroup + (row & 3);
      if (!SQA_CHECK(out_row < (size_t)p.batch * p.q_len * p.hq, p.status, 6, (long long)out_row)) continue;
      if (whole) {
        if (p.out != nullptr) {
          uint2 h;
          h.x = pack2<BF>(acc.x, acc.y);
          h.y = pack2<BF>(acc.z, acc.w);
          *reinterpret_cast<uint2*>(p.out + out_row * kHeadDim + c4) = h;
        } else {
          *reinterpret_cast<float4*>(p.out_o + out_row * kHeadDim + c4) = acc;
          if (c4 == 0) p.out_lse[out_row] = lse;
        }
      } else {
        *reinterpret_cast<float4*>(p.ws_o + ((size_t)piece * ROWS_PAD + row) * kHeadDim + c4) = acc;
        if (c4 == 0) p.ws_lse[(size_t)piece * ROWS_PAD + row] = lse;
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);

    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
}

template <int NT, int WR, bool BF>
__global__ void __launch_bounds__(kThreads, 2)
    sqa_split_kv_kernel(const SplitKvParams p, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v) {
  constexpr int WT = kConsumerWarps / WR;
  constexpr int ROWS_PAD = 8 * NT * WR;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled TMA destinations want 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* cbuf = reinterpret_cast<float*>(smem + (size_t)p.num_stages * kStageBytes);
  float* mbuf = cbuf + WT * ROWS_PAD * kCombineStride;
  float* lbuf = mbuf + WT * ROWS_PAD;
  uint64_t* full = reinterpret_cast<uint64_t*>(lbuf + WT * ROWS_PAD);  // 2S barriers
  uint64_t* empty = full + 2 * p.num_stages;                           // S barriers
  Schedule* sch = reinterpret_cast<Schedule*>(empty + p.num_stages);

  const int warp = threadIdx.x >> 5;
  unsigned long long* tl = p.timeline ? p.timeline + (size_t)blockIdx.x * 32 : nullptr;
  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 0);  // entry
    for (int i = 0; i < 2 * p.num_stages; ++i) mbar_init(smem_u32(full + i), 1);
    for (int i = 0; i < p.num_stages; ++i) mbar_init(smem_u32(empty + i), WR);
    fence_mbar_init();
  }
  if (warp == kConsumerWarps) {
    if ((threadIdx.x & 31) == 0) {
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
    }
    __syncwarp();
    prefetch_start<false>(p, &tm_k, &tm_v, p.num_stages);
  }
  // Everything above writes only shared memory and reads the inputs only as
  // prefetch hints; the inputs and the workspace may still be in use by the
  // previous kernel.
  grid_dependency_wait();
  allow_dependent_launch();  // the merge kernel may be scheduled now; it waits for this grid
  if (threadIdx.x == 0) SQA_STAMP(tl, 1);  // after the dependency wait
  if (warp == 0) build_schedule(p, sch);
  __syncthreads();
  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 2);  // schedule ready
#ifdef SQA_DEBUG_TIMELINE
    if (tl) {
      unsigned int smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      tl[7] = smid;
    }
#endif
  }

  const Schedule s = *sch;
  volatile int* abort = &sch->abort;
  if (warp == kConsumerWarps) {
    producer_loop(p, s, &tm_k, &tm_v, stages, full, empty, abort);
    if ((threadIdx.x & 31) == 0) SQA_STAMP(tl, 5);  // producer done (all loads issued and landed)
  } else {
    consumer_loop<NT, WR, BF>(p, s, stages, full, empty, cbuf, mbuf, lbuf, abort);
    if (threadIdx.x == 0) SQA_STAMP(tl, 4);  // consumers done (last epilogue written)
#ifdef SQA_DEBUG_TIMELINE
    if (threadIdx.x == 0 && tl) {
      unsigned int smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      tl[7] = smid;
    }
#endif
  }
}

template <int NT, int WR, bool BF>
cudaError_t launch_shape(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                         int grid, int smem_bytes, cudaStream_t stream) {
  auto kernel = sqa_split_kv_kernel<NT, WR, BF>;
  // Raise the dynamic shared-memory limit once per device (the size is fixed
  // per warp shape), outside any stream capture that may follow.
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64 || configured[dev] < smem_bytes) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev] = smem_bytes;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kernel, p, tm_k, tm_v);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

int split_kv_smem_bytes(const WarpShape& ws, int num_stages) {
  const int rows = ws.wt() * ws.rows_pad;
  return 1024                                   // alignment slack
         + num_stages * kStageBytes             // K/V ring
         + rows * kCombineStride * 4            // combine buffer
         + 2 * rows * 4                         // m, l
         + 3 * num_stages * 8                   // 2S full + S empty barriers
         + 64;                                  // schedule
}

cudaError_t launch_split_kv(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                            int grid, int smem_bytes, cudaStream_t stream) {
  const WarpShape ws = warp_shape_for(p.q_len);
  if (p.bf16) {
    if (ws.nt == 1) return launch_shape<1, 1, true>(p, tm_k, tm_v, grid, smem_bytes, stream);
    if (ws.wr == 1) return launch_shape<2, 1, true>(p, tm_k, tm_v, grid, smem_bytes, stream);
    if (ws.wr == 2) return launch_shape<2, 2, true>(p, tm_k, tm_v, grid, smem_bytes, stream);
    return launch_shape<2, 4, true>(p, tm_k, tm_v, grid, smem_bytes, stream);
  }
  if (ws.nt == 1) return launch_shape<1, 1, false>(p, tm_k, tm_v, grid, smem_bytes, stream);
  if (ws.wr == 1) return launch_shape<2, 1, false>(p, tm_k, tm_v, grid, smem_bytes, stream);
  if (ws.wr == 2) return launch_shape<2, 2, false>(p, tm_k, tm_v, grid, smem_bytes, stream);
  return launch_shape<2, 4, false>(p, tm_k, tm_v, grid, smem_bytes, stream);
}

}  // namespace sqa
