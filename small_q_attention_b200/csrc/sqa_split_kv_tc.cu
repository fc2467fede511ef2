// sqa_split_kv_tc.cu -- split-KV paged attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), for the larger draft lengths.
//
// Same schedule, TMA page staging, partial/merge outputs and status handling
// as sqa_split_kv.cu; what changes is who does the math:
//
// * one thread (the MMA warp) issues, per page, eight tcgen05.mma
//   M128 x N16 x K16 for S = Q K_page^T into a TMEM slot, and later one
//   M128 x N128 x K16 for O += P V_page with P read from TMEM.  Q (the 4 * q_len
//   packed rows, zero-padded to 128) is a 128-byte-swizzled K-major tile in
//   shared memory; K pages are K-major and V pages MN-major operands, both
//   straight from the TMA ring.  O (128 fp32 columns) lives in TMEM for a
//   whole piece;
// * 32 * SW softmax threads each own one packed query row = one TMEM lane:
//   the row max and sum need no shuffles.  The running max used for the
//   exponentials is only raised when a page's max exceeds it by more than
//   2^8, so O in TMEM is rescaled on few pages (the final 1/l keeps the
//   result exact); probabilities go back to TMEM as fp16 for the PV product.
//
// Pipelines (all mbarriers, all waits bounded):
//   TMA ring  full[S]/empty[S]      producer -> MMA, released by the MMA commit after PV
//   S slots   s_full[NS]            MMA (QK commit) -> softmax
//   P slots   p_full[NS]            softmax -> MMA (PV)
//   pv_done[NS]                     MMA (PV commit) -> softmax (P slot reuse, O rescale, epilogue)
//   q_ready                         softmax (Q tile written for the piece) -> MMA
// The MMA thread keeps QK kNS pages ahead of the softmax: after PV(i) it
// issues QK(i + kNS) into the slot the softmax has just released, so the
// softmax never waits for a QK product in the steady state.
#include "sqa_internal.h"
#include "sqa_ptx.cuh"
#include "sqa_schedule.cuh"

namespace sqa {
namespace {

constexpr int kNS = 5;          // S/P slots in TMEM: QK runs up to kNS pages ahead of the softmax
constexpr int kTmemCols = 256;  // O | S slots | P slots
constexpr int kColO = 0;
constexpr int kColS = 128;
constexpr int kColP = kColS + 16 * kNS;
constexpr int kQBytes = 128 * 128 * 2;  // Q tile: 128 rows x 128 dims fp16, two 64-dim halves
constexpr float kRescaleLog2 = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

struct TcSmem {
  uint8_t* q;
  uint8_t* stages;
  uint64_t *full, *empty, *s_full, *p_full, *pv_done, *q_ready, *mma_done;
  uint32_t* tmem_base;
  Schedule* sch;
};

__device__ __forceinline__ TcSmem carve(uint8_t* smem, int S) {
  TcSmem t;
  t.q = smem;
  t.stages = smem + kQBytes;
  uint64_t* b = reinterpret_cast<uint64_t*>(t.stages + (size_t)S * kStageBytes);
  t.full = b;
  t.empty = t.full + S;
  t.s_full = t.empty + S;
  t.p_full = t.s_full + kNS;
  t.pv_done = t.p_full + kNS;
  t.q_ready = t.pv_done + kNS;
  t.mma_done = t.q_ready + 1;
  t.tmem_base = reinterpret_cast<uint32_t*>(t.mma_done + 1);
  t.sch = reinterpret_cast<Schedule*>(t.tmem_base + 2);
  return t;
}

// ------------------------------------------------------------------ producer (in-order ring)
__device__ void tc_producer(const SplitKvParams& p, const Schedule& sch, const CUtensorMap* tm_k,
                            const CUtensorMap* tm_v, const TcSmem& sm, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_policy_evict_first();
  const int S = p.num_stages;
  SegWalk w = first_segment(p, sch);
  int slot = 0;
  uint32_t phase = 0;
  unsigned int bad_page = 0;
  int issued = 0;
  int unit = sch.start;
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const int32_t* row = p.block_tables + (size_t)w.b * p.max_pages + w.pg;
    int ids = (lane < n) ? __ldg(row + lane) : 0;
    for (int c0 = 0; c0 < n; c0 += 32) {
      const int cnt = min(32, n - c0);
      const int nxt = c0 + 32 + lane;
      const int ids_next = (nxt < n) ? __ldg(row + nxt) : 0;
      for (int j = 0; j < cnt; ++j) {
        int page = __shfl_sync(0xffffffffu, ids, j);
        if (page < 0 || page >= p.num_pages) {
          bad_page = 1;
          page = 0;
        }
        if (lane == 0) {
          if (mbar_wait_bounded(smem_u32(sm.empty + slot), phase ^ 1u, abort, p.status, 1, issued)) {
            const uint32_t f = smem_u32(sm.full + slot);
            mbar_arrive_expect_tx(f, kStageBytes);
            const uint32_t dst = smem_u32(sm.stages + (size_t)slot * kStageBytes);
            const int tok = page * kPageSize;
            tma_load_3d(dst, tm_k, f, 0, w.h, tok, policy);
            tma_load_3d(dst + 2048, tm_k, f, 64, w.h, tok, policy);
            tma_load_3d(dst + 4096, tm_v, f, 0, w.h, tok, policy);
            tma_load_3d(dst + 6144, tm_v, f, 64, w.h, tok, policy);
            ++issued;
          }
        }
        if (++slot == S) {
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
    for (int k = 0; k < min(issued, S); ++k) {
      const int last = k + S * ((issued - 1 - k) / S);
      if (!mbar_drain(smem_u32(sm.full + k), (uint32_t)(last / S) & 1u, 100000000ull)) atomicOr(p.status, 1u);
    }
  }
}

// ------------------------------------------------------------------ MMA issuer (one thread)
__device__ void tc_mma(const SplitKvParams& p, const Schedule& sch, const TcSmem& sm, uint32_t tmem,
                       volatile int* abort) {
  constexpr uint32_t kIdescQK = mma_idesc_f16(128, 16, false, false);  // Q (K-major) x K page (K-major)
  constexpr uint32_t kIdescPV = mma_idesc_f16(128, 128, false, true);  // P (TMEM) x V page (MN-major)
  const int S = p.num_stages;
  const uint32_t q_base = smem_u32(sm.q);
  SegWalk w = first_segment(p, sch);
  int i0 = 0;  // CTA page counter at the start of the piece
  int pc = 0;  // piece counter
  int unit = sch.start;
  while (unit < sch.end) {
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    mbar_wait_bounded(smem_u32(sm.q_ready), (uint32_t)(pc & 1), abort, p.status, 4, pc);
    tc_fence_after();
    // S(g) = Q K_g^T into slot g % kNS
    auto issue_qk = [&](int g) {
      const int st = g % S;
      mbar_wait_bounded(smem_u32(sm.full + st), (uint32_t)(g / S) & 1u, abort, p.status, 5, g);
      tc_fence_after();
      const uint32_t k_base = smem_u32(sm.stages + (size_t)st * kStageBytes);
      const uint32_t d = tmem + kColS + (g % kNS) * 16;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk & 3) * 32u;
        const uint64_t a = smem_desc_sw128(q_base + (kk >> 2) * (kQBytes / 2) + off, 16, 1024);
        const uint64_t b = smem_desc_sw128(k_base + (kk >> 2) * 2048 + off, 16, 1024);
        tc_mma_ss(d, a, b, kIdescQK, kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(sm.s_full + (g % kNS)));
    };
    for (int j = 0; j < min(n, kNS); ++j) issue_qk(i0 + j);
    for (int j = 0; j < n; ++j) {  // O += P(g) V_g, then refill the freed slot
      const int g = i0 + j;
      const int st = g % S;
      mbar_wait_bounded(smem_u32(sm.p_full + (g % kNS)), (uint32_t)(g / kNS) & 1u, abort, p.status, 6, g);
      tc_fence_after();
      const uint32_t v_base = smem_u32(sm.stages + (size_t)st * kStageBytes + 4096);
      const uint64_t b = smem_desc_sw128(v_base, 2048, 1024);  // MN atoms: V lo -> V hi; K atoms: 8 tokens
      tc_mma_ts(tmem + kColO, tmem + kColP + (g % kNS) * 8, b, kIdescPV, j > 0 ? 1u : 0u);
      tc_commit(smem_u32(sm.empty + st));           // the page's stage may be refilled
      tc_commit(smem_u32(sm.pv_done + (g % kNS)));  // P slot free, O up to date
      if (j + kNS < n) issue_qk(g + kNS);           // the softmax has read S(g): reuse its slot
    }
    i0 += n;
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

  SegWalk w = first_segment(p, sch);
  int i0 = 0;
  int unit = sch.start;
  while (unit < sch.end) {
    const int s = w.b * p.hkv + w.h;
    const int seg_end = w.seg_start + w.pages;
    const int n = min(sch.end, seg_end) - unit;
    const bool whole = (unit == w.seg_start) && (seg_end <= sch.end);
    if (tid == 0 && unit == w.seg_start) {
      const int last_cta = (seg_end - 1) / sch.per_cta;
      p.seg_info[s] = make_int2((int)blockIdx.x + s, last_cta - (int)blockIdx.x + 1);
    }
    const int len_raw = __ldg(p.seq_lens + w.b);
    const int len = min(len_raw, w.pages * kPageSize);
    const int mlen = p.mask_lens ? __ldg(p.mask_lens + w.b) : len_raw;
    const int thr_min = min(len, mlen - p.q_len + 1);
    const int thr = min(len, mlen - p.q_len + (row >> 2) + 1);

    // Q tile of this piece: rows < 4*q_len, 128-byte swizzled, two 64-dim halves.
    // (All QK products of the previous piece are complete: every S slot was consumed.)
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
    for (int j = 0; j < n; ++j) {
      const int g = i0 + j;
      const int sl = g % kNS;
      const int tok0 = (w.pg + j) * kPageSize;
      mbar_wait_bounded(smem_u32(sm.s_full + sl), (uint32_t)(g / kNS) & 1u, abort, p.status, 7, g);
      tc_fence_after();
      uint32_t raw[16];
      tmem_ld16(tl + kColS + sl * 16, raw);
      tmem_wait_ld();
      float x[16];
      const bool masked = tok0 + kPageSize > thr_min;
      float mx = -INFINITY;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        x[t] = __uint_as_float(raw[t]) * p.scale_log2;
        if (masked && tok0 + t >= thr) x[t] = -INFINITY;
        mx = fmaxf(mx, x[t]);
      }
      const float m_new = fmaxf(m_used, mx);
      const bool need = active && (m_new > m_used + kRescaleLog2);
      if (j == 0) {
        m_used = m_new;  // the piece's first PV overwrites O
      } else if (__any_sync(0xffffffffu, need)) {
        // O must be stable: wait for PV(g - 1), then rescale this warp's rows in TMEM
        mbar_wait_bounded(smem_u32(sm.pv_done + ((g - 1) % kNS)), (uint32_t)((g - 1) / kNS) & 1u, abort,
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
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
      uint32_t pk[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float p0 = active ? ex2(x[2 * t] - base) : 0.f;
        const float p1 = active ? ex2(x[2 * t + 1] - base) : 0.f;
        l += p0 + p1;
        pk[t] = pack_half2(p0, p1);
      }
      if (g >= kNS)  // PV(g - kNS) has read this P slot
        mbar_wait_bounded(smem_u32(sm.pv_done + sl), (uint32_t)((g - kNS) / kNS) & 1u, abort, p.status, 9, g);
      tc_fence_after();
      tmem_st8(tl + kColP + sl * 8, pk);
      tmem_wait_st();
      if (tok0 + kPageSize > len && warp == 0) {
        // tokens at or past the sequence end: zero their V rows (the pool may hold NaN there)
        uint8_t* vst = sm.stages + (size_t)(g % p.num_stages) * kStageBytes + 4096;
        const int first = max(len - tok0, 0);
        for (int c = lane; c < (kPageSize - first) * 16; c += 32) {
          const int r = first + (c >> 4);
          *reinterpret_cast<uint4*>(vst + ((c >> 3) & 1) * 2048 + r * 128 + (c & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(sm.p_full + sl));
    }

    // ---- epilogue: O is complete once the piece's last PV has finished
    const int gl = i0 + n - 1;
    mbar_wait_bounded(smem_u32(sm.pv_done + (gl % kNS)), (uint32_t)(gl / kNS) & 1u, abort, p.status, 10, gl);
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

    i0 += n;
    unit += n;
    if (unit >= seg_end) next_segment(p, w);
    else w.pg += n;
  }
}

template <int SW>
__global__ void __launch_bounds__((SW + 2) * 32, 2)
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
    for (int i = 0; i < kNS; ++i) {
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

int split_kv_tc_smem_bytes(int num_stages) {
  return 1024 + kQBytes + num_stages * kStageBytes + (2 * num_stages + 3 * kNS + 2) * 8 + 8 + 64;
}

cudaError_t launch_split_kv_tc(const SplitKvParams& p, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                               int grid, int smem_bytes, cudaStream_t stream) {
  if (kGroup * p.q_len <= 32) return launch_tc<1>(p, tm_k, tm_v, grid, smem_bytes, stream);
  return launch_tc<2>(p, tm_k, tm_v, grid, smem_bytes, stream);
}

}  // namespace sqa
