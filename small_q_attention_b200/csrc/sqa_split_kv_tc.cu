// sqa_split_kv_tc.cu -- split-KV paged attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory).
//
// Same schedule, page table walk, TMA page loads, partial/merge outputs and
// status handling as sqa_split_kv.cu.  The difference is the math engine:
//
// * Pages are staged in blocks of kBP = 4: a ring slot holds the K low/high
//   and V low/high 64-dim halves of 4 pages, each half-region contiguous, so
//   the 64 tokens of a block form one K-major operand (rows 128 B apart, 8-row
//   groups 1 KB apart) and one MN-major operand for V.
// * Q lives in tensor memory for a whole piece, replicated R times down the
//   128 lanes (R = 4 for q_len <= 8, 2 for q_len <= 16): lane 128/R * r + i
//   holds packed query row i (row i = draft token i/4, head i%4 of the group).
//   Per block the MMA warp issues eight M128 x N64 x K16 MMAs for
//   S = Q K_block^T (A = Q from TMEM, B = K from shared memory) into one of
//   four S slots, and kBP M128 x N128 x K16 MMAs for O += P V_page with P read
//   back from TMEM.  Replica r owns pages [4/R r, 4/R (r+1)) of every block:
//   the PV MMA of a page writes only the lanes of its replica (the MMA's
//   output-lane mask), so every replica keeps its own running (O, max, sum)
//   and the replicas are merged once per piece through shared memory.
// * Four softmax warps, one per TMEM lane quadrant; each thread owns one row
//   of one replica and reads only its replica's 64/R S columns of a block, so
//   the exponentials of a block are spread over all four warps.  The max used
//   for the exponentials is raised only when a block's max exceeds it by more
//   than 2^8; then the warp's O rows are rescaled in TMEM.  P (fp16) is written
//   over the block's S columns.
// * Two MMA warps, one issuing the QK products and one the PV products, each
//   converged and issuing through elect.sync: a PV whose P is ready never
//   waits behind a QK whose pages are still in flight.
// * fp8 caches (template mode KV = 2): 16 KB blocks of 128-byte swizzled fp8
//   rows read by kind::f8f6f4 products; Q and P enter as two e4m3 parts each
//   (high + low), so eight QK and four PV products per block as for fp16.
//
// Pipelines (mbarriers; every wait bounded):
//   ring   full[NB] / empty[NB]   producer -> QK issuer; released by the commit after PV
//   S/P    s_full[4] / p_full[4]  QK issuer (commit) -> softmax -> PV issuer
//   pv_done[4]                    PV issuer (commit) -> S/P slot reuse, O rescale, epilogue
//   q_ready[2]                    softmax (Q of a piece in TMEM, one piece ahead) -> QK issuer
// The QK issuer runs up to four blocks ahead of the softmax (one per S slot).
#include <cuda_fp8.h>

#include <mutex>

#include "sqa_internal.h"
#include "sqa_ptx.cuh"
#include "sqa_schedule.cuh"

namespace sqa {
namespace {

constexpr int kBP = 4;                          // pages per block
constexpr int kBlockTokens = kBP * kPageSize;   // 64
constexpr int kRegionBytes = kBP * 2048;        // one 64-dim half of K or V for a block
constexpr int kBlockBytes = 4 * kRegionBytes;   // K lo | K hi | V lo | V hi
constexpr int kTmemCols = 512;                  // O | Q x2 | S/P slots 0..3
constexpr int kColO = 0;
constexpr int kColQ = 128;                      // two Q slots (pieces alternate), 64 columns each
constexpr int kColS = 256;
#ifndef SQA_TC_NUM_S
#define SQA_TC_NUM_S 4
#endif
constexpr int kNumS = SQA_TC_NUM_S;             // S/P slots (64 columns each)
static_assert(kColS + kNumS * 64 <= 512, "S slots must fit in TMEM");
constexpr int kSlotCols = kBlockTokens;         // fp32 S of a block; its fp16 P takes the first half
constexpr int kSoftmaxWarps = 4;
constexpr int kThreadsTc = (kSoftmaxWarps + 3) * 32;  // softmax x4, QK issuer, PV issuer, producer

// Block shape per cache mode.  KV 0 (16-bit): 4 pages (64 tokens) per 32 KB ring
// block (K lo | K hi | V lo | V hi), four 64-column S slots.  fp8 caches, K pages
// then V pages, 2 KB each: KV 2, 4 pages per 16 KB block and four 64-column S
// slots; KV 3, 8 pages per 32 KB block and two 128-column S slots (the same TMEM
// and tokens in flight; the QK products run at N = 128, where the tensor core is
// most efficient, and the softmax's per-block overheads cover twice the tokens:
// the better shape for long per-CTA ranges, the 4-page one for short calls).
template <int KV>
struct TcShape {
  static constexpr bool kFp8 = KV >= 2;
  static constexpr int kPages = KV == 3 ? 8 : kBP;
  static constexpr int kTokens = kPages * kPageSize;
  static constexpr int kSlots = KV == 3 ? 2 : kNumS;
  static constexpr int kSlotCols = kTokens;
  static constexpr int kRing = kFp8 ? kPages * 4096 : kBlockBytes;  // bytes per ring block
  static constexpr int kVOffset = kFp8 ? kPages * 2048 : 2 * kRegionBytes;  // V within a block
  static_assert(kColS + kSlots * kSlotCols <= 512, "S slots must fit in TMEM");
};
constexpr int kMergeCols = 64;                  // dims merged per pass
constexpr int kMergeStride = kMergeCols + 1;    // floats per merge row (conflict-free columns)
constexpr int kMergeBytes = 128 * kMergeStride * 4;  // one row per TMEM lane
constexpr int kMlBytes = 128 * 8;               // (max, sum) per lane
constexpr float kRescaleLog2 = 8.f;
// Cluster mode: a CTA's normalised part [rows <= 64, 128] fp32 and its LSEs sit at
// the start of the operand ring (idle once the CTA's one piece is done).
constexpr int kClusterRows = 64;
constexpr int kMaxCluster = 16;
constexpr float kLn2 = 0.6931471805599453f;

struct TcSmem {
  uint8_t* ring;    // operand blocks, the TMA target
  float* merge;
  float2* ml;
  uint64_t *full, *empty, *s_full, *p_full, *pv_done, *q_ready, *mma_done;
  uint32_t* tmem_base;
  Schedule* sch;
};

// KV: 0 = 16-bit caches; 2, 3 = fp8 caches read by the tensor core as fp8
// (kind::f8f6f4) in 4- or 8-page blocks.

__device__ __forceinline__ TcSmem carve(uint8_t* smem, int nb, int ring_bytes) {
  TcSmem t;
  t.ring = smem;
  t.merge = reinterpret_cast<float*>(smem + (size_t)nb * ring_bytes);
  t.ml = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(t.merge) + kMergeBytes);
  uint64_t* b = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(t.ml) + kMlBytes);
  t.full = b;
  t.empty = t.full + nb;
  t.s_full = t.empty + nb;
  t.p_full = t.s_full + kNumS;
  t.pv_done = t.p_full + kNumS;
  t.q_ready = t.pv_done + kNumS;
  t.mma_done = t.q_ready + 2;
  t.tmem_base = reinterpret_cast<uint32_t*>(t.mma_done + 1);
  t.sch = reinterpret_cast<Schedule*>(t.tmem_base + 2);
  return t;
}

template <int KV>
__device__ __forceinline__ int blocks_of(int n) { return (n + TcShape<KV>::kPages - 1) / TcShape<KV>::kPages; }

// ------------------------------------------------------------------ producer (whole warp)
// KV 2: fp8 boxes (128 dims = 128 bytes, swizzled), one per page per tensor;
// KV 0: two 64-dim fp16 halves per page per tensor; both into the operand ring.
template <int KV>
__device__ void tc_producer(const SplitKvParams& p, const Schedule& sch, const CUtensorMap* tm_k,
                            const CUtensorMap* tm_v, const TcSmem& sm, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_policy_evict_first();
  const int NB = p.num_stages;
  uint64_t* const full = sm.full;
  uint64_t* const empty = sm.empty;
  SegWalk w = first_segment(p, sch);
  int slot = 0;
  uint32_t phase = 0;
  unsigned int bad_page = 0;
  int issued = 0;  // blocks whose loads were issued (a prefix)
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
    for (int c0 = 0; c0 < n; c0 += 32) {  // 32 is a multiple of the block: blocks never straddle chunks
      const int cnt = min(32, n - c0);
      int ids_next = 0;
      if (c0 + 32 < n) {
        ids_next = (c0 + 32 + lane < n) ? __ldg(row + c0 + 32 + lane) : 0;
      } else if (unit_next < sch.end) {
        const int n2 = min(sch.end, wn.seg_start + wn.pages) - unit_next;
        ids_next = (lane < n2) ? __ldg(p.block_tables + (size_t)wn.b * p.max_pages + wn.pg + lane) : 0;
      }
      constexpr int kPg = TcShape<KV>::kPages;
      for (int jb = 0; jb < cnt; jb += kPg) {
        const int np = min(kPg, cnt - jb);
        int pages[kPg];
#pragma unroll
        for (int j = 0; j < kPg; ++j) {
          pages[j] = __shfl_sync(0xffffffffu, ids, min(jb + j, 31));
          if (j < np && (pages[j] < 0 || pages[j] >= p.num_pages)) {
            bad_page = 1;
            pages[j] = 0;
          }
        }
        bool ok = mbar_wait_bounded(smem_u32(empty + slot), phase ^ 1u, abort, p.status, 1, issued);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok) {
          if (elect_one()) {
            const uint32_t f = smem_u32(full + slot);
            // NHD map: (dim, head, token, page); HND map: (dim, token, head, page)
            const int c1 = p.hnd ? 0 : w.h;
            const int c2 = p.hnd ? w.h : 0;
            if constexpr (TcShape<KV>::kFp8) {
              mbar_arrive_expect_tx(f, np * 4096);
              const uint32_t base = smem_u32(sm.ring + (size_t)slot * TcShape<KV>::kRing);
              for (int j = 0; j < np; ++j) {  // 128 fp8 dims x 16 tokens = 2 KB per tensor
                tma_load_4d(base + j * 2048, tm_k, f, 0, c1, c2, pages[j], policy);
                tma_load_4d(base + TcShape<KV>::kVOffset + j * 2048, tm_v, f, 0, c1, c2, pages[j], policy);
              }
            } else {
              mbar_arrive_expect_tx(f, np * kStageBytes);
              const uint32_t base = smem_u32(sm.ring + (size_t)slot * kBlockBytes);
              for (int j = 0; j < np; ++j) {
                const uint32_t dst = base + j * 2048;
                tma_load_4d(dst, tm_k, f, 0, c1, c2, pages[j], policy);
                tma_load_4d(dst + kRegionBytes, tm_k, f, 64, c1, c2, pages[j], policy);
                tma_load_4d(dst + 2 * kRegionBytes, tm_v, f, 0, c1, c2, pages[j], policy);
                tma_load_4d(dst + 3 * kRegionBytes, tm_v, f, 64, c1, c2, pages[j], policy);
              }
            }
          }
          __syncwarp();
          ++issued;
        }
        if (++slot == NB) {
          slot = 0;
          phase ^= 1u;
        }
      }
      ids = ids_next;
    }
    unit = unit_next;
    w = wn;
  }
  if (__any_sync(0xffffffffu, bad_page) && lane == 0) atomicOr(p.status, 8u);  // SQA_DEV_BAD_PAGE
  if (lane == 0 && *abort) {  // only an abort can leave loads in flight
    for (int k = 0; k < min(issued, NB); ++k) {
      const int last = k + NB * ((issued - 1 - k) / NB);
      if (!mbar_drain(smem_u32(full + k), (uint32_t)(last / NB) & 1u, 100000000ull)) atomicOr(p.status, 1u);
    }
  }
}

// ------------------------------------------------------------------ MMA issuers (whole warps, one elected lane)
// Two warps issue to the tensor core: one the QK products, one the PV products,
// so that a PV whose P is ready never waits behind a QK whose pages are still
// in flight (and the other way round).  Ordering between their MMAs comes only
// from the barriers: s_full / p_full / pv_done.

// Both issuers: every MMA this warp issued must finish before TMEM is released.
__device__ __forceinline__ void tc_mma_drain(const SplitKvParams& p, const TcSmem& sm) {
  if (elect_one()) tc_commit(smem_u32(sm.mma_done));
  __syncwarp();
  if (!mbar_drain(smem_u32(sm.mma_done), 0u, 2000000000ull) && (threadIdx.x & 31) == 0) atomicOr(p.status, 1u);
}

// S(h) = Q K_h^T into slot h % kNumS, once the block's pages are in and PV(h - kNumS)
// has released the slot; Q of a piece is in TMEM once q_ready completes.
// KV 2: Q is in TMEM as two e4m3 parts (high: columns 0-31, low: 32-63 of its
// slot, 4 dims per column); S = Q_hi K^T + Q_lo K^T, eight K32 products.
template <bool BF, int KV>
__device__ void tc_mma_qk(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                          volatile int* abort) {
  // Q (TMEM) x K_block (K-major).  Format field 0 is fp16 for kind::f16 and e4m3 for
  // kind::f8f6f4 (where 1 would be e5m2): KV 2 is e4m3 whatever the query type.
  using Sh = TcShape<KV>;
  constexpr uint32_t kIdescQK = mma_idesc_f16(128, Sh::kTokens, false, false, BF && !Sh::kFp8);
  const int NB = p.num_stages;
  SegWalk w = first_segment(p, sch);
  int h = 0;   // CTA block counter
  int pc = 0;  // piece counter
  int unit = sch.start;
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int nblk = blocks_of<KV>(n);
    // Q of piece pc is in Q slot pc % 2 (written one piece ahead by the softmax warps)
    mbar_wait_bounded(smem_u32(sm.q_ready + (pc & 1)), (uint32_t)(pc >> 1) & 1u, abort, p.status, 4, pc);
    const uint32_t q_col = tmem + kColQ + (pc & 1) * 64;
    for (int k = 0; k < nblk; ++k, ++h) {
      if (h >= Sh::kSlots)
        mbar_wait_bounded(smem_u32(sm.pv_done + (h % Sh::kSlots)), (uint32_t)((h - Sh::kSlots) / Sh::kSlots) & 1u, abort,
                          p.status, 11, h);
      const int slot = h % NB;
      mbar_wait_bounded(smem_u32(sm.full + slot), (uint32_t)(h / NB) & 1u, abort, p.status, 5, h);
      __syncwarp();
      tc_fence_after();
      if (h == 0 && (threadIdx.x & 31) == 0 && p.timeline) {
        SQA_STAMP(p.timeline + (size_t)blockIdx.x * 32, 3);
        SQA_CLK(p.timeline + (size_t)blockIdx.x * 32, 12);
      }
      const uint64_t t_qk = SQA_T0();
      if (elect_one()) {
        const uint32_t d = tmem + kColS + (h % Sh::kSlots) * Sh::kSlotCols;
        if constexpr (Sh::kFp8) {
          // K: 64 or 128 token rows of 128 fp8 dims (128 B, swizzled), 8-row groups 1 KB apart
          const uint32_t k_base = smem_u32(sm.ring + (size_t)slot * Sh::kRing);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // high part, then low part; 32 dims (32 B) per step
            const uint64_t b = smem_desc_sw128(k_base + (kk & 3) * 32u, 16, 1024);
            tc_mma_ts_f8(d, q_col + (kk >> 2) * 32 + (kk & 3) * 8, b, kIdescQK, kk > 0 ? 1u : 0u);
          }
        } else {
          const uint32_t k_base = smem_u32(sm.ring + (size_t)slot * kBlockBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t b = smem_desc_sw128(k_base + (kk >> 2) * kRegionBytes + (kk & 3) * 32u, 16, 1024);
            tc_mma_ts(d, q_col + kk * 8, b, kIdescQK, kk > 0 ? 1u : 0u);
          }
        }
        tc_commit(smem_u32(sm.s_full + (h % Sh::kSlots)));
      }
      __syncwarp();
      SQA_WAIT_ACCOUNT(12, t_qk);
      (void)t_qk;
    }
    ++pc;
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
  tc_mma_drain(p, sm);
}

// O += P V_g once the softmax has written P(g); then the block's ring slot and
// S/P slot are released by commits.
// KV 2: P is in TMEM as two e4m3 parts over all 64 tokens of the block (high:
// columns 0-15, low: 16-31 of the S/P slot; zero outside the row's replica), so
// four K32 products with no lane mask cover every replica at once.
template <int R, bool BF, int KV>
__device__ void tc_mma_pv(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                          volatile int* abort) {
  // P (TMEM) x V (MN-major); KV 2: e4m3 whatever the query type (format field 0)
  constexpr uint32_t kIdescPV = mma_idesc_f16(128, 128, false, true, BF && !TcShape<KV>::kFp8);
  using Sh = TcShape<KV>;
  constexpr int kPPR = kBP / R;       // KV 0: pages of a block per replica
  constexpr int kLanesPR = 128 / R;   // TMEM lanes per replica
  const int NB = p.num_stages;
  SegWalk w = first_segment(p, sch);
  int g = 0;  // CTA block counter
  int unit = sch.start;
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int nblk = blocks_of<KV>(n);
    for (int k = 0; k < nblk; ++k, ++g) {
      const int slot = g % NB;
      const int np = min(Sh::kPages, n - k * Sh::kPages);
      mbar_wait_bounded(smem_u32(sm.p_full + (g % Sh::kSlots)), (uint32_t)(g / Sh::kSlots) & 1u, abort, p.status, 6,
                        g);
      __syncwarp();
      tc_fence_after();
      const uint64_t t_pv = SQA_T0();
      if (elect_one()) {
        const uint32_t p_col = tmem + kColS + (g % Sh::kSlots) * Sh::kSlotCols;
        if constexpr (Sh::kFp8) {
          // V: the block's token rows of 128 fp8 dims, one 128-byte MN atom wide; 8-row groups
          // 1 KB apart; P high part in the slot's first kTokens / 4 columns, low part next
          const uint32_t v_base = smem_u32(sm.ring + (size_t)slot * Sh::kRing + Sh::kVOffset);
          const int quarters = (np + 1) / 2;  // 32 tokens per product; absent pages hold zero V
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            for (int qt = 0; qt < quarters; ++qt) {
              const uint64_t b = smem_desc_sw128(v_base + qt * 4096, Sh::kRing, 1024);
              // the piece's first product overwrites O
              tc_mma_ts_f8(tmem + kColO, p_col + part * (Sh::kTokens / 4) + qt * 8, b, kIdescPV,
                           (k > 0 || part > 0 || qt > 0) ? 1u : 0u);
            }
          }
        } else {
          const uint32_t v_base = smem_u32(sm.ring + (size_t)slot * kBlockBytes + 2 * kRegionBytes);
          for (int kk = 0; kk < np; ++kk) {  // 16 tokens (one page) per step
            const int rep = kk / kPPR;
            uint32_t off[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) off[e] = (e * 32 >= rep * kLanesPR && e * 32 < (rep + 1) * kLanesPR) ? 0u : ~0u;
            // MN atoms (64 dims) kRegionBytes apart: V lo -> V hi; K atoms (8 tokens) 1 KB apart
            const uint64_t b = smem_desc_sw128(v_base + kk * 2048, kRegionBytes, 1024);
            // a replica's first page of the piece overwrites its O rows
            tc_mma_ts_lanes(tmem + kColO, p_col + kk * 8, b, kIdescPV, (k > 0 || (kk % kPPR) != 0) ? 1u : 0u, off);
          }
        }
        tc_commit(smem_u32(sm.empty + slot));              // the block's ring slot may be refilled
        tc_commit(smem_u32(sm.pv_done + (g % Sh::kSlots)));  // S/P slot free, O up to date
      }
      __syncwarp();
      SQA_WAIT_ACCOUNT(13, t_pv);
      (void)t_pv;
    }
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
  tc_mma_drain(p, sm);
}

// ------------------------------------------------------------------ softmax + epilogue (4 warps)
// KV 2 (fp8 caches read as fp8): each Q row is scaled by a power of two 2^e
// that brings its largest magnitude into [128, 256) and split into two e4m3
// parts, hi = e4m3(2^e q) and lo = e4m3(2^e q - hi), so S = (Q_hi + Q_lo) K^T
// carries about 8 significant bits of q (the 2^-e is folded into the exponent's
// scale).  P is split the same way (P <= 2^8 < 448 by the rescale rule).
template <int R, bool BF, int KV>
__device__ void tc_softmax(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                           volatile int* abort) {
  constexpr int kLanesPR = 128 / R;          // lanes (rows) per replica
  using Sh = TcShape<KV>;
  constexpr int kTok = Sh::kTokens / R;      // tokens of a block per replica
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;               // 0 .. 127
  const int rows = kGroup * p.q_len;         // <= kLanesPR
  const int rep = (warp * 32) / kLanesPR;    // replica of this warp
  const int lrow = warp * 32 + lane - rep * kLanesPR;  // packed query row of this thread
  const bool active = lrow < rows;
  const int tok_lo = rep * kTok;             // first block column of this replica
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  const int NB = p.num_stages;

  // This thread's lane of Q slot `qs` gets packed row lrow of (b, h) (zeros past the rows).
  auto write_q = [&](int b, int h, int qs) {
    const __half* src = p.q + ((size_t)(b * p.q_len + (lrow >> 2)) * p.hq + h * kGroup + (lrow & 3)) * kHeadDim;
    uint32_t qv[2][32];  // the whole row first: one memory round trip
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = active ? __ldg(reinterpret_cast<const uint4*>(src) + c) : make_uint4(0u, 0u, 0u, 0u);
      qv[c >> 3][4 * (c & 7)] = v.x;
      qv[c >> 3][4 * (c & 7) + 1] = v.y;
      qv[c >> 3][4 * (c & 7) + 2] = v.z;
      qv[c >> 3][4 * (c & 7) + 3] = v.w;
    }
    float qinv = 1.f;  // KV 2: 2^-e of this row
    if constexpr (Sh::kFp8) {
      float mx = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float2 f = unpack2<BF>(qv[i >> 5][i & 31]);
        mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      // mx in [2^(x-127), 2^(x-126)) for biased exponent x: 2^e mx in [128, 256) for e = 134 - x
      const int e = (mx > 0.f) ? max(-100, min(100, 134 - (int)((__float_as_uint(mx) >> 23) & 0xffu))) : 0;
      const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
      qinv = __uint_as_float((uint32_t)(127 - e) << 23);
      uint32_t hi[32], lo[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {  // 4 dims per column: words 2i, 2i + 1 of the row
        const float2 a = unpack2<BF>(qv[(2 * i) >> 5][(2 * i) & 31]);
        const float2 c = unpack2<BF>(qv[(2 * i + 1) >> 5][(2 * i + 1) & 31]);
        const float x0 = a.x * sc, x1 = a.y * sc, x2 = c.x * sc, x3 = c.y * sc;
        const uint32_t h01 = pack_e4m3x2(x0, x1), h23 = pack_e4m3x2(x2, x3);
        const float2 d01 = unpack_e4m3x2(h01), d23 = unpack_e4m3x2(h23);
        hi[i] = h01 | (h23 << 16);
        lo[i] = pack_e4m3x2(x0 - d01.x, x1 - d01.y) | (pack_e4m3x2(x2 - d23.x, x3 - d23.y) << 16);
      }
      tmem_st32(tl + kColQ + qs * 64, hi);
      tmem_st32(tl + kColQ + qs * 64 + 32, lo);
    } else {
      tmem_st32(tl + kColQ + qs * 64, qv[0]);
      tmem_st32(tl + kColQ + qs * 64 + 32, qv[1]);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(sm.q_ready + qs));
    return qinv;
  };
  float qinv_slot[2] = {1.f, 1.f};  // KV 2: 2^-e of this thread's row in each Q slot

  SegWalk w = first_segment(p, sch);
  int gb0 = 0;
  int pc = 0;  // piece counter
  int unit = sch.start;
  while (unit < sch.end) {
    const int s = w.b * p.hkv + w.h;
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int nblk = blocks_of<KV>(n);
    const bool whole = (unit == w.seg_start) && (seg_end <= sch.end);
    const int len_raw = __ldg(p.seq_lens + w.b);
    const int len = min(len_raw, w.pages * kPageSize);
    const int mlen = p.mask_lens ? __ldg(p.mask_lens + w.b) : len_raw;
    const int thr = min(len, mlen - p.q_len + (lrow >> 2) + 1);
    const int thr_min = min(len, mlen - p.q_len + 1);  // visible tokens of draft row 0

    // Q into TMEM one piece ahead: piece pc uses Q slot pc % 2, so the QK products
    // of the next piece can run while this piece's epilogue is still merging.
    // Slot (pc + 1) % 2 is free: every QK product of piece pc - 1 is complete
    // (all its S blocks were consumed).
    if (pc == 0) {
      qinv_slot[0] = write_q(w.b, w.h, 0);
      if (tid == 0 && p.timeline) SQA_CLK(p.timeline + (size_t)blockIdx.x * 32, 13);
    }
    // this piece's score scale (KV 2: with the row's 2^-e)
    const float cs = p.scale_log2 * ((pc & 1) ? qinv_slot[1] : qinv_slot[0]);
    if (seg_end < sch.end) {  // the next piece starts the next segment
      SegWalk nw = w;
      next_segment(p, nw);
      const float qi = write_q(nw.b, nw.h, (pc + 1) & 1);
      if ((pc + 1) & 1) qinv_slot[1] = qi;
      else qinv_slot[0] = qi;
    }

    float m_used = -INFINITY, l = 0.f;
    for (int k = 0; k < nblk; ++k) {
      const int g = gb0 + k;
      const int np = min(Sh::kPages, n - k * Sh::kPages);
      const int tok0 = (w.pg + k * Sh::kPages) * kPageSize + tok_lo;  // first token of this replica's columns
      const int valid = np * kPageSize - tok_lo;                 // valid columns of this replica (may be <= 0)
      mbar_wait_bounded(smem_u32(sm.s_full + (g % Sh::kSlots)), (uint32_t)(g / Sh::kSlots) & 1u, abort, p.status, 7,
                        g);
      tc_fence_after();
      if (g == 0 && tid == 0 && p.timeline) SQA_CLK(p.timeline + (size_t)blockIdx.x * 32, 14);
      const uint64_t t_sm = SQA_T0();
      const uint32_t slot_col = tl + kColS + (g % Sh::kSlots) * Sh::kSlotCols;
      uint32_t sraw[kTok];
      if constexpr (kTok == 16) {
        tmem_ld16(slot_col + tok_lo, sraw);
      } else {
#pragma unroll
        for (int c = 0; c < kTok; c += 32)
          tmem_ld32(slot_col + tok_lo + c, *reinterpret_cast<uint32_t(*)[32]>(sraw + c));
      }
      tmem_wait_ld();
      // Scores stay unscaled until the exponent: max(c * s) = c * max(s) for c > 0.
      // mask columns past the piece (stale data), the causal tail and the sequence end
      if (valid < kTok || tok0 + kTok > thr_min) {
#pragma unroll
        for (int t = 0; t < kTok; ++t)
          if (t >= valid || tok0 + t >= thr) sraw[t] = 0xff800000u;  // -inf
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < kTok; t += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(sraw[t]));
        mx1 = fmaxf(mx1, __uint_as_float(sraw[t + 1]));
      }
      const float m_new = fmaxf(m_used, fmaxf(mx0, mx1) * cs);
      const bool need = active && (m_new > m_used + kRescaleLog2);
      if (k == 0) {
        m_used = m_new;  // the piece's first PV of this replica overwrites its O rows
      } else if (__any_sync(0xffffffffu, need)) {
        // O must be stable: wait for PV(g - 1), then rescale this warp's rows in TMEM
        mbar_wait_bounded(smem_u32(sm.pv_done + ((g - 1) % Sh::kSlots)), (uint32_t)((g - 1) / Sh::kSlots) & 1u, abort,
                          p.status, 8, g);
        tc_fence_after();
        const float alpha = need ? ex2(m_used - m_new) : 1.f;
        if (need) {
          m_used = m_new;
          l *= alpha;
        }
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t o[16];
          tmem_ld16(tl + kColO + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st16(tl + kColO + c, o);
        }
        tmem_wait_st();
      }
      // p = 2^(c*s - m): one FFMA and one ex2 per score
      const float nbase = active ? -((m_used == -INFINITY) ? 0.f : m_used) : -INFINITY;
      float ls[2] = {0.f, 0.f};
      if constexpr (Sh::kFp8) {
        // P as e4m3 high and low parts over all tokens of the block (the slot's first
        // kTokens / 4 columns and the next, 4 tokens per column), zero outside this
        // replica's tokens so that the PV products need no lane mask
        constexpr int kW = kTok / 4;  // columns of this replica per part
        uint32_t ph[kW], pl[kW];
#pragma unroll
        for (int t = 0; t < kW; ++t) {
          const float p0 = ex2(fmaf(__uint_as_float(sraw[4 * t]), cs, nbase));
          const float p1 = ex2(fmaf(__uint_as_float(sraw[4 * t + 1]), cs, nbase));
          const float p2 = ex2(fmaf(__uint_as_float(sraw[4 * t + 2]), cs, nbase));
          const float p3 = ex2(fmaf(__uint_as_float(sraw[4 * t + 3]), cs, nbase));
          ls[t & 1] += (p0 + p1) + (p2 + p3);
          // high part e4m3(p), low part e4m3(p - high) (the high part read back exactly)
          const uint32_t h01 = pack_e4m3x2(p0, p1), h23 = pack_e4m3x2(p2, p3);
          const float2 d01 = unpack_e4m3x2(h01), d23 = unpack_e4m3x2(h23);
          ph[t] = h01 | (h23 << 16);
          pl[t] = pack_e4m3x2(p0 - d01.x, p1 - d01.y) | (pack_e4m3x2(p2 - d23.x, p3 - d23.y) << 16);
        }
        constexpr int kPartCols = Sh::kTokens / 4;  // 16 or 32
        if constexpr (kPartCols == 16) {
          uint32_t pw[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pw[i] = (i / kW == rep) ? ph[i % kW] : 0u;
            pw[16 + i] = (i / kW == rep) ? pl[i % kW] : 0u;
          }
          tmem_st32(slot_col, pw);
        } else {
          uint32_t pw[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pw[i] = (i / kW == rep) ? ph[i % kW] : 0u;
          tmem_st32(slot_col, pw);
#pragma unroll
          for (int i = 0; i < 32; ++i) pw[i] = (i / kW == rep) ? pl[i % kW] : 0u;
          tmem_st32(slot_col + 32, pw);
        }
      } else {
        // P as fp16 / bf16 pairs over this replica's columns in the first half of the S slot
        uint32_t pk[kTok / 2];
#pragma unroll
        for (int t = 0; t < kTok / 2; ++t) {
          const float p0 = ex2(fmaf(__uint_as_float(sraw[2 * t]), cs, nbase));
          const float p1 = ex2(fmaf(__uint_as_float(sraw[2 * t + 1]), cs, nbase));
          ls[t & 1] += p0 + p1;
          pk[t] = pack2<BF>(p0, p1);
        }
        if constexpr (kTok == 16) tmem_st8(slot_col + tok_lo / 2, pk);
        else tmem_st16(slot_col + tok_lo / 2, pk);
      }
      l += ls[0] + ls[1];
      tmem_wait_st();
      const int btok = (w.pg + k * Sh::kPages) * kPageSize;
      if (Sh::kFp8 && (btok + np * kPageSize > len || np < Sh::kPages) && warp == 0) {
        // fp8 V rows (128 B, swizzled within the row only) of tokens at or past the
        // sequence end, and of the absent pages a 32-token product still reads: zero
        uint8_t* vreg = sm.ring + (size_t)(g % NB) * Sh::kRing + Sh::kVOffset;
        const int pages_read = (np + 1) / 2 * 2;  // whole 32-token quarters
        for (int j = 0; j < pages_read; ++j) {
          const int first = (j < np) ? max(len - (btok + j * kPageSize), 0) : 0;
          if (first >= kPageSize) continue;
          for (int c = lane; c < (kPageSize - first) * 8; c += 32)
            *reinterpret_cast<uint4*>(vreg + j * 2048 + (first + (c >> 3)) * 128 + (c & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      if (!Sh::kFp8 && btok + np * kPageSize > len && warp == 0) {
        // tokens at or past the sequence end: zero their V rows (the pool may hold NaN there)
        uint8_t* vreg = sm.ring + (size_t)(g % NB) * kBlockBytes + 2 * kRegionBytes;
        for (int j = 0; j < np; ++j) {
          const int first = max(len - (btok + j * kPageSize), 0);
          if (first >= kPageSize) continue;
          for (int c = lane; c < (kPageSize - first) * 16; c += 32) {
            const int r = first + (c >> 4);
            *reinterpret_cast<uint4*>(vreg + ((c >> 3) & 1) * kRegionBytes + j * 2048 + r * 128 + (c & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(sm.p_full + (g % Sh::kSlots)));
      SQA_WAIT_ACCOUNT(14, t_sm);
      (void)t_sm;
    }

    // ---- epilogue: merge the R replicas of every row, then write the piece's rows
    const uint64_t t_ep = SQA_T0();
    const int gl = gb0 + nblk - 1;
    sm.ml[rep * kLanesPR + lrow] = make_float2(m_used, l);
    mbar_wait_bounded(smem_u32(sm.pv_done + (gl % Sh::kSlots)), (uint32_t)(gl / Sh::kSlots) & 1u, abort, p.status, 10,
                      gl);
    tc_fence_after();
    named_bar_sync(1, kSoftmaxWarps * 32);
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float2 v = sm.ml[r * kLanesPR + lrow];
      if (v.y > 0.f) mx = fmaxf(mx, v.x);
    }
    float L = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float2 v = sm.ml[r * kLanesPR + lrow];
      if (v.y > 0.f) L += v.y * ex2(v.x - mx);
    }
    // this replica's weight (L > 0 when l > 0), with the output scale folded in
    const float f = (l > 0.f) ? ex2(m_used - mx) * p.out_scale / L : 0.f;
    const float lse = (L > 0.f) ? (mx + __log2f(L)) * kLn2 : -INFINITY;
    // Two chunks of 64 dims: every warp stores its rows' weighted chunk (a
    // uniform branch: tcgen05.ld needs the whole warp), then the 128 threads sum
    // the replicas in a fixed order (deterministic) and write coalesced rows.
    const int piece = (int)blockIdx.x + s;
    float* mrow = sm.merge + (rep * kLanesPR + lrow) * kMergeStride;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += kMergeCols) {
#pragma unroll
      for (int c = 0; c < kMergeCols; c += 16) {
        uint32_t o[16];
        tmem_ld16(tl + kColO + c0 + c, o);
        tmem_wait_ld();
        // a replica without tokens (f == 0) may hold stale O: never multiply it in
#pragma unroll
        for (int t = 0; t < 16; ++t) mrow[c + t] = (f != 0.f) ? __uint_as_float(o[t]) * f : 0.f;
      }
      named_bar_sync(1, kSoftmaxWarps * 32);
      for (int idx = tid; idx < rows * (kMergeCols / 8); idx += kSoftmaxWarps * 32) {
        const int r = idx / (kMergeCols / 8), ch = idx % (kMergeCols / 8);
        float v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = 0.f;
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          const float* src = sm.merge + (rr * kLanesPR + r) * kMergeStride + ch * 8;
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] += src[t];
        }
        const size_t out_row = (size_t)(w.b * p.q_len + (r >> 2)) * p.hq + w.h * kGroup + (r & 3);
        const int col = c0 + ch * 8;
        if (p.cluster) {  // cluster mode: this CTA's part, for the reduction across the cluster
          float* dst = reinterpret_cast<float*>(sm.ring) + r * kHeadDim + col;
          *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
        } else if (whole && p.out != nullptr) {
          uint4 h;
          h.x = pack2<BF>(v[0], v[1]);
          h.y = pack2<BF>(v[2], v[3]);
          h.z = pack2<BF>(v[4], v[5]);
          h.w = pack2<BF>(v[6], v[7]);
          *reinterpret_cast<uint4*>(p.out + out_row * kHeadDim + col) = h;
        } else {
          float* dst = whole ? p.out_o + out_row * kHeadDim + col
                             : p.ws_o + ((size_t)piece * p.rows_pad + r) * kHeadDim + col;
          *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
      named_bar_sync(1, kSoftmaxWarps * 32);
    }
    tc_fence_before();  // O reads are done before the next piece's first PV overwrites it
    SQA_WAIT_ACCOUNT(15, t_ep);
    (void)t_ep;
    if (rep == 0 && active) {
      const size_t out_row = (size_t)(w.b * p.q_len + (lrow >> 2)) * p.hq + w.h * kGroup + (lrow & 3);
      if (p.cluster) reinterpret_cast<float*>(sm.ring)[kClusterRows * kHeadDim + lrow] = lse;
      else if (whole && p.out == nullptr) p.out_lse[out_row] = lse;
      else if (!whole) p.ws_lse[(size_t)piece * p.rows_pad + lrow] = lse;
    }

    gb0 += nblk;
    ++pc;
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
#ifdef SQA_DEBUG_TIMELINE
  if (tid == 0 && p.timeline) p.timeline[(size_t)blockIdx.x * 32 + 15] = (unsigned long long)gb0 * 100 + pc;
#endif
}

// ------------------------------------------------------------------ cluster reduction (all threads)
// Cluster mode: each CTA of the cluster left its part of the segment (normalised
// rows and natural-log LSEs, -inf for a part without keys) in its shared memory;
// after a cluster barrier, the cluster's rank-0 CTA reads every part through
// distributed shared memory and writes the segment's rows with the arithmetic of
// the split-KV merge (max, weights exp(lse - max), sum, divide; 0 for a row that
// sees no key).  A second barrier keeps every CTA's shared memory alive until
// rank 0 has read it.  Every thread of every CTA reaches both barriers.
template <bool BF>
__device__ void tc_cluster_reduce(const SplitKvParams& p, const TcSmem& sm, const Schedule& s) {
  float* cl = reinterpret_cast<float*>(sm.ring);
  float* cl_lse = cl + kClusterRows * kHeadDim;
  const int rows = kGroup * p.q_len;
  if (s.start >= s.end)  // no page here: this part carries no weight
    for (int r = threadIdx.x; r < rows; r += blockDim.x) cl_lse[r] = -INFINITY;
  cluster_sync_all();
  const int C = p.cluster;
  if ((int)blockIdx.x % C == 0) {
    const int seg = (int)blockIdx.x / C;
    const int b = seg / p.hkv;
    const int h = seg - b * p.hkv;
    const uint32_t o_base = smem_u32(cl), l_base = smem_u32(cl_lse);
    for (int idx = threadIdx.x; idx < rows * (kHeadDim / 4); idx += blockDim.x) {
      const int r = idx / (kHeadDim / 4);
      const int c4 = idx - r * (kHeadDim / 4);
      // parts 8 at a time, every load of a batch in flight at once; a running max
      // rescales what earlier batches summed (one round trip for C <= 8)
      constexpr int kBatch = 8;
      float mx = -INFINITY, total = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j0 = 0; j0 < C; j0 += kBatch) {
        float l[kBatch];
        float4 v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          if (j0 + j < C) {
            l[j] = ld_cluster_f32(cluster_map(l_base + r * 4, j0 + j));
            v[j] = ld_cluster_v4(cluster_map(o_base + (r * kHeadDim + c4 * 4) * 4, j0 + j));
          } else {
            l[j] = -INFINITY;
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        float bmx = mx;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) bmx = fmaxf(bmx, l[j]);
        if (bmx == -INFINITY) continue;  // nothing visible so far
        if (bmx > mx && mx != -INFINITY) {
          const float scale = ex2((mx - bmx) * 1.4426950408889634f);
          total *= scale;
          acc.x *= scale;
          acc.y *= scale;
          acc.z *= scale;
          acc.w *= scale;
        }
        mx = bmx;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const float wgt = ex2((l[j] - mx) * 1.4426950408889634f);  // -inf -> 0
          total += wgt;
          acc.x += wgt * v[j].x;
          acc.y += wgt * v[j].y;
          acc.z += wgt * v[j].z;
          acc.w += wgt * v[j].w;
        }
      }
      const float inv = total > 0.f ? 1.f / total : 0.f;
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
      const size_t out_row = (size_t)(b * p.q_len + (r >> 2)) * p.hq + h * kGroup + (r & 3);
      if (p.out != nullptr) {
        uint2 o;
        o.x = pack2<BF>(acc.x, acc.y);
        o.y = pack2<BF>(acc.z, acc.w);
        *reinterpret_cast<uint2*>(p.out + out_row * kHeadDim + c4 * 4) = o;
      } else {
        *reinterpret_cast<float4*>(p.out_o + out_row * kHeadDim + c4 * 4) = acc;
        if (c4 == 0) p.out_lse[out_row] = total > 0.f ? (mx + __log2f(total) * kLn2) : -INFINITY;
      }
    }
  }
  cluster_sync_all();
}

template <int R, bool BF, int KV>
__global__ void __launch_bounds__(kThreadsTc, 1)
    sqa_split_kv_tc_kernel(const SplitKvParams p, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcSmem sm = carve(smem, p.num_stages, TcShape<KV>::kRing);
  const int warp = threadIdx.x >> 5;
  constexpr int kMmaWarp = kSoftmaxWarps;         // QK issuer; owns the TMEM allocation
  constexpr int kPvWarp = kSoftmaxWarps + 1;
  constexpr int kProducerWarp = kSoftmaxWarps + 2;
  unsigned long long* tl = p.timeline ? p.timeline + (size_t)blockIdx.x * 32 : nullptr;
#ifdef SQA_DEBUG_TIMELINE
  if (threadIdx.x < 16) sqa_wait_ns[threadIdx.x] = 0;
#endif

  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 0);
#ifdef SQA_DEBUG_TIMELINE
    if (tl) tl[5] = clock64();
#endif
    for (int i = 0; i < p.num_stages; ++i) {
      mbar_init(smem_u32(sm.full + i), 1);  // the producer's arrival + the TMA bytes
      mbar_init(smem_u32(sm.empty + i), 1);
    }
    for (int i = 0; i < kNumS; ++i) {
      mbar_init(smem_u32(sm.s_full + i), 1);
      mbar_init(smem_u32(sm.p_full + i), kSoftmaxWarps);
      mbar_init(smem_u32(sm.pv_done + i), 1);
    }
    mbar_init(smem_u32(sm.q_ready), kSoftmaxWarps);
    mbar_init(smem_u32(sm.q_ready + 1), kSoftmaxWarps);
    mbar_init(smem_u32(sm.mma_done), 2);  // one commit from each issuer
    fence_mbar_init();
  }
  if (warp == kProducerWarp && (threadIdx.x & 31) == 0) {
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  // The PV issuer has nothing to do before the first P: it prefetches this
  // CTA's first pages into L2 before the dependency wait (hints only), off the
  // start-up path of the other warps.
  if (warp == kPvWarp) prefetch_start<KV != 0>(p, &tm_k, &tm_v, p.num_stages * TcShape<KV>::kPages);
  grid_dependency_wait();
  allow_dependent_launch();
  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 1);
    SQA_CLK(tl, 8);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(sm.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0) build_schedule(p, sm.sch);
  tc_fence_before();
  // Start-up barrier: the TMEM address, the schedule and the mbarriers are
  // ready.  Every warp but the PV issuer syncs on barrier 3 and arrives on
  // barrier 2; the PV issuer waits on barrier 2 only, so its prefetches never
  // hold up the others.
  const uint32_t nthreads = blockDim.x;
  if (warp == kPvWarp) {
    named_bar_sync(2, nthreads);
  } else {
    named_bar_sync(3, nthreads - 32);
    named_bar_arrive(2, nthreads);
  }
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  const Schedule s = *sm.sch;
  volatile int* abort = &sm.sch->abort;
  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 2);
    SQA_CLK(tl, 9);
  }

  if (warp == kProducerWarp) {
    tc_producer<KV>(p, s, &tm_k, &tm_v, sm, abort);
  } else if (warp == kMmaWarp) {
    tc_mma_qk<BF, KV>(p, s, sm, tmem, abort);
  } else if (warp == kPvWarp) {
    tc_mma_pv<R, BF, KV>(p, s, sm, tmem, abort);
  } else {
    tc_softmax<R, BF, KV>(p, s, sm, tmem, abort);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (p.cluster) tc_cluster_reduce<BF>(p, sm, s);
#ifdef SQA_DEBUG_TIMELINE
  if (tl && threadIdx.x == 0) {
    tl[4] = global_timer_ns();
    tl[6] = clock64();
    unsigned int smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    tl[7] = smid;
    for (int k = 1; k < 16; ++k) tl[16 + k] = sqa_wait_ns[k];
  }
#endif
}

template <int R, bool BF, int KV>
cudaError_t launch_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid,
                      int smem_bytes, cudaStream_t stream) {
  auto kernel = sqa_split_kv_tc_kernel<R, BF, KV>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64 || configured[dev] < smem_bytes) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev] = smem_bytes;
  }
  if (p.cluster > 8) {  // 16-CTA clusters are outside the portable size
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return err;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.cluster > 1 ? p.cluster : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.cluster > 1 ? 2 : 1;
  err = cudaLaunchKernelEx(&cfg, kernel, p, tm_k, tm_v);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

int split_kv_tc_block_bytes(int kv_fp8) { return kv_fp8 == 3 ? 8 * 4096 : kv_fp8 ? 4 * 4096 : kBlockBytes; }

int split_kv_tc_max_clusters(int cluster, int smem_bytes) {
  if (cluster < 2 || cluster > kMaxCluster) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  static std::mutex mu;
  static int cache[64][kMaxCluster + 1] = {};
  static int cache_smem[64][kMaxCluster + 1] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (cache_smem[dev][cluster] == smem_bytes) return cache[dev][cluster];
  auto kernel = sqa_split_kv_tc_kernel<4, false, 0>;  // every instantiation: same threads, 1 CTA per SM
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess ||
      (cluster > 8 && cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster);
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  cache[dev][cluster] = n;
  cache_smem[dev][cluster] = smem_bytes;
  return n;
}

int split_kv_tc_smem_bytes(int num_blocks, int kv_fp8) {
  return 1024 + num_blocks * split_kv_tc_block_bytes(kv_fp8) + kMergeBytes + kMlBytes +
         (2 * num_blocks + 3 * kNumS + 3) * 8 + 8 + 64;
}

cudaError_t launch_split_kv_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               int grid, int smem_bytes, cudaStream_t stream) {
  const bool r4 = kGroup * p.q_len <= 32;
  if (p.kv_fp8 == 3) {  // fp8 caches read as fp8, 8-page blocks; fp16 or bf16 queries
    if (p.bf16)
      return r4 ? launch_tc<4, true, 3>(p, tm_k, tm_v, grid, smem_bytes, stream)
                : launch_tc<2, true, 3>(p, tm_k, tm_v, grid, smem_bytes, stream);
    return r4 ? launch_tc<4, false, 3>(p, tm_k, tm_v, grid, smem_bytes, stream)
              : launch_tc<2, false, 3>(p, tm_k, tm_v, grid, smem_bytes, stream);
  }
  if (p.kv_fp8) {  // fp8 caches read as fp8, 4-page blocks
    if (p.bf16)
      return r4 ? launch_tc<4, true, 2>(p, tm_k, tm_v, grid, smem_bytes, stream)
                : launch_tc<2, true, 2>(p, tm_k, tm_v, grid, smem_bytes, stream);
    return r4 ? launch_tc<4, false, 2>(p, tm_k, tm_v, grid, smem_bytes, stream)
              : launch_tc<2, false, 2>(p, tm_k, tm_v, grid, smem_bytes, stream);
  }
  if (p.bf16)
    return r4 ? launch_tc<4, true, 0>(p, tm_k, tm_v, grid, smem_bytes, stream)
              : launch_tc<2, true, 0>(p, tm_k, tm_v, grid, smem_bytes, stream);
  return r4 ? launch_tc<4, false, 0>(p, tm_k, tm_v, grid, smem_bytes, stream)
            : launch_tc<2, false, 0>(p, tm_k, tm_v, grid, smem_bytes, stream);
}

}  // namespace sqa
