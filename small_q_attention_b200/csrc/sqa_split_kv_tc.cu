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
// * One thread (the MMA warp) issues, per block, eight tcgen05.mma
//   M128 x N64 x K16 for S = Q K_block^T into a TMEM slot, and kBP
//   M128 x N128 x K16 for O += P V_block with P read back from TMEM.  Q (the
//   4 * q_len packed query rows of one KV head, zero-padded to 128) is a
//   128-byte-swizzled K-major tile in shared memory.  O (128 fp32 columns)
//   stays in TMEM for a whole piece.  Per-page MMAs (N = 16) were measured
//   first and were issue-bound at ~100 cycles per instruction.
// * 32 * SW softmax threads each own one packed query row = one TMEM lane, so
//   row max and sum need no shuffles.  The max used for the exponentials is
//   raised only when a block's max exceeds it by more than 2^8; then this
//   warp's O rows are rescaled in TMEM (rare after the first blocks; the final
//   1/l keeps the result exact).  P is written as fp16 over the block's S.
//
// Pipelines (mbarriers; every wait bounded):
//   ring   full[NB] / empty[NB]   producer -> MMA; released by the commit after PV
//   S/P    s_full[2] / p_full[2]  MMA (QK commit) -> softmax -> MMA (PV)
//   pv_done[2]                    MMA (PV commit) -> S/P slot reuse, O rescale, epilogue
//   q_ready                       softmax (Q tile of the piece written) -> MMA
// QK of block g+1 is issued before PV of block g.
#include "sqa_internal.h"
#include "sqa_ptx.cuh"
#include "sqa_schedule.cuh"

namespace sqa {
namespace {

constexpr int kBP = 4;                          // pages per block
constexpr int kBlockTokens = kBP * kPageSize;   // 64
constexpr int kRegionBytes = kBP * 2048;        // one 64-dim half of K or V for a block
constexpr int kBlockBytes = 4 * kRegionBytes;   // K lo | K hi | V lo | V hi
constexpr int kTmemCols = 256;                  // O | S/P slot 0 | S/P slot 1
constexpr int kColO = 0;
constexpr int kColS = 128;
constexpr int kSlotCols = kBlockTokens;         // fp32 S of a block; its fp16 P takes the first half
constexpr int kQBytes = 128 * 128 * 2;          // Q tile: 128 rows x 128 dims fp16, two 64-dim halves
constexpr float kRescaleLog2 = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

struct TcSmem {
  uint8_t* q;
  uint8_t* ring;
  uint64_t *full, *empty, *s_full, *p_full, *pv_done, *q_ready, *mma_done;
  uint32_t* tmem_base;
  Schedule* sch;
};

__device__ __forceinline__ TcSmem carve(uint8_t* smem, int nb) {
  TcSmem t;
  t.q = smem;
  t.ring = smem + kQBytes;
  uint64_t* b = reinterpret_cast<uint64_t*>(t.ring + (size_t)nb * kBlockBytes);
  t.full = b;
  t.empty = t.full + nb;
  t.s_full = t.empty + nb;
  t.p_full = t.s_full + 2;
  t.pv_done = t.p_full + 2;
  t.q_ready = t.pv_done + 2;
  t.mma_done = t.q_ready + 1;
  t.tmem_base = reinterpret_cast<uint32_t*>(t.mma_done + 1);
  t.sch = reinterpret_cast<Schedule*>(t.tmem_base + 2);
  return t;
}

__device__ __forceinline__ int blocks_of(int n) { return (n + kBP - 1) / kBP; }

// ------------------------------------------------------------------ producer
__device__ void tc_producer(const SplitKvParams& p, const Schedule& sch, const CUtensorMap* tm_k,
                            const CUtensorMap* tm_v, const TcSmem& sm, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_policy_evict_first();
  const int NB = p.num_stages;
  SegWalk w = first_segment(p, sch);
  int slot = 0;
  uint32_t phase = 0;
  unsigned int bad_page = 0;
  int issued = 0;  // blocks whose loads were issued (a prefix)
  int unit = sch.start;
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int32_t* row = p.block_tables + (size_t)w.b * p.max_pages + w.pg;
    int ids = (lane < n) ? __ldg(row + lane) : 0;
    for (int c0 = 0; c0 < n; c0 += 32) {  // 32 is a multiple of kBP: blocks never straddle chunks
      const int cnt = min(32, n - c0);
      const int nxt = c0 + 32 + lane;
      const int ids_next = (nxt < n) ? __ldg(row + nxt) : 0;
      for (int jb = 0; jb < cnt; jb += kBP) {
        const int np = min(kBP, cnt - jb);
        int pages[kBP];
#pragma unroll
        for (int j = 0; j < kBP; ++j) {
          pages[j] = __shfl_sync(0xffffffffu, ids, min(jb + j, 31));
          if (j < np && (pages[j] < 0 || pages[j] >= p.num_pages)) {
            bad_page = 1;
            pages[j] = 0;
          }
        }
        if (lane == 0) {
          if (mbar_wait_bounded(smem_u32(sm.empty + slot), phase ^ 1u, abort, p.status, 1, issued)) {
            const uint32_t f = smem_u32(sm.full + slot);
            mbar_arrive_expect_tx(f, np * kStageBytes);
            const uint32_t base = smem_u32(sm.ring + (size_t)slot * kBlockBytes);
            for (int j = 0; j < np; ++j) {
              const int tok = pages[j] * kPageSize;
              const uint32_t dst = base + j * 2048;
              tma_load_3d(dst, tm_k, f, 0, w.h, tok, policy);
              tma_load_3d(dst + kRegionBytes, tm_k, f, 64, w.h, tok, policy);
              tma_load_3d(dst + 2 * kRegionBytes, tm_v, f, 0, w.h, tok, policy);
              tma_load_3d(dst + 3 * kRegionBytes, tm_v, f, 64, w.h, tok, policy);
            }
            ++issued;
          }
        }
        if (++slot == NB) {
          slot = 0;
          phase ^= 1u;
        }
      }
      ids = ids_next;
    }
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
  if (__any_sync(0xffffffffu, bad_page) && lane == 0) atomicOr(p.status, 8u);  // SQA_DEV_BAD_PAGE
  if (lane == 0 && *abort) {  // only an abort can leave loads in flight
    for (int k = 0; k < min(issued, NB); ++k) {
      const int last = k + NB * ((issued - 1 - k) / NB);
      if (!mbar_drain(smem_u32(sm.full + k), (uint32_t)(last / NB) & 1u, 100000000ull)) atomicOr(p.status, 1u);
    }
  }
}

// ------------------------------------------------------------------ MMA issuer (one thread)
__device__ void tc_mma(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                       volatile int* abort) {
  constexpr uint32_t kIdescQK = mma_idesc_f16(128, kBlockTokens, false, false);  // Q x K_block, both K-major
  constexpr uint32_t kIdescPV = mma_idesc_f16(128, 128, false, true);           // P (TMEM) x V (MN-major)
  const int NB = p.num_stages;
  const uint32_t q_base = smem_u32(sm.q);
  SegWalk w = first_segment(p, sch);
  int gb0 = 0;  // CTA block counter at the start of the piece
  int pc = 0;   // piece counter
  int unit = sch.start;

  // S(h) = Q K_h^T into slot h & 1, once PV(h - 2) has released that slot.
  auto issue_qk = [&](int h) {
    if (h >= 2)
      mbar_wait_bounded(smem_u32(sm.pv_done + (h & 1)), (uint32_t)((h - 2) >> 1) & 1u, abort, p.status, 11, h);
    const int slot = h % NB;
    mbar_wait_bounded(smem_u32(sm.full + slot), (uint32_t)(h / NB) & 1u, abort, p.status, 5, h);
    tc_fence_after();
    const uint32_t k_base = smem_u32(sm.ring + (size_t)slot * kBlockBytes);
    const uint32_t d = tmem + kColS + (h & 1) * kSlotCols;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t off = (kk & 3) * 32u;
      const uint64_t a = smem_desc_sw128(q_base + (kk >> 2) * (kQBytes / 2) + off, 16, 1024);
      const uint64_t b = smem_desc_sw128(k_base + (kk >> 2) * kRegionBytes + off, 16, 1024);
      tc_mma_ss(d, a, b, kIdescQK, kk > 0 ? 1u : 0u);
    }
    tc_commit(smem_u32(sm.s_full + (h & 1)));
  };

  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int nblk = blocks_of(n);
    mbar_wait_bounded(smem_u32(sm.q_ready), (uint32_t)(pc & 1), abort, p.status, 4, pc);
    tc_fence_after();
    issue_qk(gb0);
    for (int k = 0; k < nblk; ++k) {
      const int g = gb0 + k;
      if (k + 1 < nblk) issue_qk(g + 1);
      const int slot = g % NB;
      const int np = min(kBP, n - k * kBP);
      mbar_wait_bounded(smem_u32(sm.p_full + (g & 1)), (uint32_t)(g >> 1) & 1u, abort, p.status, 6, g);
      tc_fence_after();
      const uint32_t v_base = smem_u32(sm.ring + (size_t)slot * kBlockBytes + 2 * kRegionBytes);
      const uint32_t p_col = tmem + kColS + (g & 1) * kSlotCols;
      for (int kk = 0; kk < np; ++kk) {  // 16 tokens (one page) per step
        // MN atoms (64 dims) kRegionBytes apart: V lo -> V hi; K atoms (8 tokens) 1 KB apart
        const uint64_t b = smem_desc_sw128(v_base + kk * 2048, kRegionBytes, 1024);
        tc_mma_ts(tmem + kColO, p_col + kk * 8, b, kIdescPV, (k > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(smem_u32(sm.empty + slot));       // the block's ring slot may be refilled
      tc_commit(smem_u32(sm.pv_done + (g & 1)));  // S/P slot free, O up to date
    }
    gb0 += nblk;
    ++pc;
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
  // every MMA this thread issued must finish before TMEM is released
  tc_commit(smem_u32(sm.mma_done));
  if (!mbar_drain(smem_u32(sm.mma_done), 0u, 2000000000ull)) atomicOr(p.status, 1u);
}

// ------------------------------------------------------------------ softmax + epilogue
template <int SW>
__device__ void tc_softmax(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                           volatile int* abort) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;  // 0 .. 32*SW-1
  const int rows = kGroup * p.q_len;
  const int row = warp * 32 + lane;  // = TMEM lane
  const bool active = row < rows;
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  const int NB = p.num_stages;

  SegWalk w = first_segment(p, sch);
  int gb0 = 0;
  int unit = sch.start;
  while (unit < sch.end) {
    const int s = w.b * p.hkv + w.h;
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int nblk = blocks_of(n);
    const bool whole = (unit == w.seg_start) && (seg_end <= sch.end);
    if (tid == 0 && unit == w.seg_start) {
      const int last_cta = (seg_end - 1) / sch.per_cta;
      p.seg_info[s] = make_int2((int)blockIdx.x + s, last_cta - (int)blockIdx.x + 1);
    }
    const int len_raw = __ldg(p.seq_lens + w.b);
    const int len = min(len_raw, w.pages * kPageSize);
    const int mlen = p.mask_lens ? __ldg(p.mask_lens + w.b) : len_raw;
    const int thr = min(len, mlen - p.q_len + (row >> 2) + 1);
    const int thr_min = min(len, mlen - p.q_len + 1);  // visible tokens of draft row 0

    // Q tile of this piece: rows < 4*q_len, 128-byte swizzled, two 64-dim halves.
    // (Every QK product of the previous piece is complete: all its S blocks were consumed.)
    for (int c = tid; c < rows * 16; c += SW * 32) {
      const int r = c >> 4, ch = c & 15;
      const __half* src =
          p.q + ((size_t)(w.b * p.q_len + (r >> 2)) * p.hq + w.h * kGroup + (r & 3)) * kHeadDim + ch * 8;
      uint8_t* dst = sm.q + (ch >> 3) * (kQBytes / 2) + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
    }
    fence_proxy_async_smem();  // make the tile visible to the tensor core
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(sm.q_ready));

    float m_used = -INFINITY, l = 0.f;
    for (int k = 0; k < nblk; ++k) {
      const int g = gb0 + k;
      const int np = min(kBP, n - k * kBP);
      const int tok0 = (w.pg + k * kBP) * kPageSize;  // first token of the block
      const int valid_cols = np * kPageSize;
      mbar_wait_bounded(smem_u32(sm.s_full + (g & 1)), (uint32_t)(g >> 1) & 1u, abort, p.status, 7, g);
      tc_fence_after();
      const uint32_t slot_col = tl + kColS + (g & 1) * kSlotCols;
      uint32_t sraw[kBlockTokens];
      tmem_ld64(slot_col, sraw);
      tmem_wait_ld();
      // Scores stay unscaled until the exponent: max(c * s) = c * max(s) for c > 0.
      // mask a block that is partial (pages past the piece hold stale data) or
      // that reaches the causal tail / the sequence end
      if (valid_cols < kBlockTokens || tok0 + kBlockTokens > thr_min) {
#pragma unroll
        for (int t = 0; t < kBlockTokens; ++t)
          if (t >= valid_cols || tok0 + t >= thr) sraw[t] = 0xff800000u;  // -inf
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < kBlockTokens; t += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(sraw[t]));
        mx1 = fmaxf(mx1, __uint_as_float(sraw[t + 1]));
      }
      const float m_new = fmaxf(m_used, fmaxf(mx0, mx1) * p.scale_log2);
      const bool need = active && (m_new > m_used + kRescaleLog2);
      if (k == 0) {
        m_used = m_new;  // the piece's first PV overwrites O
      } else if (__any_sync(0xffffffffu, need)) {
        // O must be stable: wait for PV(g - 1), then rescale this warp's rows in TMEM
        mbar_wait_bounded(smem_u32(sm.pv_done + ((g - 1) & 1)), (uint32_t)((g - 1) >> 1) & 1u, abort, p.status, 8,
                          g);
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
      // p = 2^(c*s - m): one FFMA and one ex2 per score; P as fp16 over the
      // first half of the block's S columns (already read above)
      const float nbase = active ? -((m_used == -INFINITY) ? 0.f : m_used) : -INFINITY;
      const float cs = p.scale_log2;
      uint32_t pk[kBlockTokens / 2];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int t = 0; t < kBlockTokens / 2; ++t) {
        const float p0 = ex2(fmaf(__uint_as_float(sraw[2 * t]), cs, nbase));
        const float p1 = ex2(fmaf(__uint_as_float(sraw[2 * t + 1]), cs, nbase));
        ls[t & 3] += p0 + p1;
        pk[t] = pack_half2(p0, p1);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_st32(slot_col, pk);
      tmem_wait_st();
      if (tok0 + valid_cols > len && warp == 0) {
        // tokens at or past the sequence end: zero their V rows (the pool may hold NaN there)
        uint8_t* vreg = sm.ring + (size_t)(g % NB) * kBlockBytes + 2 * kRegionBytes;
        for (int j = 0; j < np; ++j) {
          const int first = max(len - (tok0 + j * kPageSize), 0);
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
      if (lane == 0) mbar_arrive(smem_u32(sm.p_full + (g & 1)));
    }

    // ---- epilogue: O is complete once the piece's last PV has finished
    const int gl = gb0 + nblk - 1;
    mbar_wait_bounded(smem_u32(sm.pv_done + (gl & 1)), (uint32_t)(gl >> 1) & 1u, abort, p.status, 10, gl);
    tc_fence_after();
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    const float lse = (l > 0.f) ? (m_used + __log2f(l)) * kLn2 : -INFINITY;
    const size_t out_row = (size_t)(w.b * p.q_len + (row >> 2)) * p.hq + w.h * kGroup + (row & 3);
    const int piece = (int)blockIdx.x + s;
#pragma unroll 1
    for (int c = 0; c < 128; c += 16) {
      uint32_t o[16];
      tmem_ld16(tl + kColO + c, o);
      tmem_wait_ld();
      if (!active) continue;
      float v[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) v[t] = __uint_as_float(o[t]) * inv;
      if (whole && p.out != nullptr) {
        uint4 h0, h1;
        h0.x = pack_half2(v[0], v[1]);
        h0.y = pack_half2(v[2], v[3]);
        h0.z = pack_half2(v[4], v[5]);
        h0.w = pack_half2(v[6], v[7]);
        h1.x = pack_half2(v[8], v[9]);
        h1.y = pack_half2(v[10], v[11]);
        h1.z = pack_half2(v[12], v[13]);
        h1.w = pack_half2(v[14], v[15]);
        uint4* dst = reinterpret_cast<uint4*>(p.out + out_row * kHeadDim + c);
        dst[0] = h0;
        dst[1] = h1;
      } else {
        float* dst = whole ? p.out_o + out_row * kHeadDim + c
                           : p.ws_o + ((size_t)piece * p.rows_pad + row) * kHeadDim + c;
#pragma unroll
        for (int t = 0; t < 16; t += 4)
          *reinterpret_cast<float4*>(dst + t) = make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
      }
    }
    if (active) {
      if (whole && p.out == nullptr) p.out_lse[out_row] = lse;
      if (!whole) p.ws_lse[(size_t)piece * p.rows_pad + row] = lse;
    }
    tc_fence_before();  // O reads are done before the next piece's first PV overwrites it

    gb0 += nblk;
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
}

template <int SW>
__global__ void __launch_bounds__((SW + 2) * 32, 1)
    sqa_split_kv_tc_kernel(const SplitKvParams p, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcSmem sm = carve(smem, p.num_stages);
  const int warp = threadIdx.x >> 5;
  constexpr int kMmaWarp = SW;
  constexpr int kProducerWarp = SW + 1;
  unsigned long long* tl = p.timeline ? p.timeline + (size_t)blockIdx.x * 32 : nullptr;
#ifdef SQA_DEBUG_TIMELINE
  if (threadIdx.x < 16) sqa_wait_ns[threadIdx.x] = 0;
#endif

  if (threadIdx.x == 0) {
    SQA_STAMP(tl, 0);
    for (int i = 0; i < p.num_stages; ++i) {
      mbar_init(smem_u32(sm.full + i), 1);
      mbar_init(smem_u32(sm.empty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(sm.s_full + i), 1);
      mbar_init(smem_u32(sm.p_full + i), SW);
      mbar_init(smem_u32(sm.pv_done + i), 1);
    }
    mbar_init(smem_u32(sm.q_ready), SW);
    mbar_init(smem_u32(sm.mma_done), 1);
    fence_mbar_init();
  }
  // rows of the Q tile past 4 * q_len stay zero for the whole kernel
  for (int i = threadIdx.x; i < kQBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sm.q)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();  // these generic writes are read by the tensor core
  if (warp == kProducerWarp && (threadIdx.x & 31) == 0) {
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  grid_dependency_wait();
  allow_dependent_launch();
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(sm.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0) build_schedule(p, sm.sch);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  const Schedule s = *sm.sch;
  volatile int* abort = &sm.sch->abort;

  if (warp == kProducerWarp) {
    tc_producer(p, s, &tm_k, &tm_v, sm, abort);
  } else if (warp == kMmaWarp) {
    if ((threadIdx.x & 31) == 0) tc_mma(p, s, sm, tmem, abort);
    __syncwarp();
  } else {
    tc_softmax<SW>(p, s, sm, tmem, abort);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
#ifdef SQA_DEBUG_TIMELINE
  if (tl && threadIdx.x == 0) {
    tl[4] = global_timer_ns();
    for (int k = 0; k < 16; ++k) tl[16 + k] = sqa_wait_ns[k];
  }
#endif
}

template <int SW>
cudaError_t launch_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid,
                      int smem_bytes, cudaStream_t stream) {
  auto kernel = sqa_split_kv_tc_kernel<SW>;
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
  cfg.blockDim = dim3((SW + 2) * 32);
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

int split_kv_tc_block_bytes() { return kBlockBytes; }

int split_kv_tc_smem_bytes(int num_blocks) {
  return 1024 + kQBytes + num_blocks * kBlockBytes + (2 * num_blocks + 8) * 8 + 8 + 64;
}

cudaError_t launch_split_kv_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               int grid, int smem_bytes, cudaStream_t stream) {
  if (kGroup * p.q_len <= 32) return launch_tc<1>(p, tm_k, tm_v, grid, smem_bytes, stream);
  return launch_tc<2>(p, tm_k, tm_v, grid, smem_bytes, stream);
}

}  // namespace sqa
