// sqa_api.cu -- the extern "C" boundary (include/small_q_attention.h).
//
// Validates the contract on the host (no device reads), sizes the split-KV
// launch from the SM count and the shapes, encodes the two TMA tensor maps
// over the paged caches and launches the kernels on the caller's stream.
// Errors are status codes; no exception leaves this file.
#include <cstdio>
#include <cmath>
#include <mutex>

#include "../../include/small_q_attention.h"
#include "sqa_internal.h"

namespace sqa {
namespace {

constexpr int kAbiVersion = 110;
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;
constexpr int kCtasPerSm = 2;
// Shared memory one CTA may use so that kCtasPerSm fit on an SM
// (228 KB per SM on sm_100, 1 KB reserved per CTA).
constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemPerCta = kSmemPerSm / kCtasPerSm - 1024;
constexpr int kMaxSmemPerCta = 227 * 1024;  // dynamic shared memory limit of one CTA on sm_100
// Auto kernel choice thresholds on the launch's upper bound of units (pages x KV
// heads), from the 36-case matrix measured on B200 at 1965 MHz: the tcgen05
// kernel from 12288 units for q_len <= 2, from 2048 for q_len 3..4, above 512
// for q_len 5..8, always for q_len >= 9.
constexpr long long kAutoTcUnitsQ2 = 12288;
constexpr long long kAutoTcUnitsQ4 = 2048;
constexpr long long kAutoTcUnitsQ8 = 512;
constexpr int kDefaultMinPagesPerCta = 4;
// fp8 caches: 8-page blocks when a CTA's range is at least this many pages x KV
// heads (measured on B200: 5-6% faster at q16 x 16 x 32K and on cfg5, 4-6% slower
// on calls of ~100 pages per CTA).
constexpr long long kFp8LongRangeUnits = 400;
// Schedule: a segment start costs a CTA as much as this many pages (one more
// piece epilogue and pipeline refill; measured per kernel on B200).
#ifndef SQA_SEGMENT_COST_TC
#define SQA_SEGMENT_COST_TC 24
#endif
#ifndef SQA_SEGMENT_COST_MMA
#define SQA_SEGMENT_COST_MMA 4
#endif
constexpr int kSegmentCostTc = SQA_SEGMENT_COST_TC;
constexpr int kSegmentCostMma = SQA_SEGMENT_COST_MMA;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int sm_count(int device) {
  static std::mutex mu;
  static int cache[kMaxDevices] = {0};
  if (device < 0 || device >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device] = n;
  }
  return cache[device];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [num_pages * 16 tokens, Hkv, 128] fp16 seen as a 3-D tensor; one box is
// 64 dims x 1 head x 16 tokens (2 KB), 128-byte swizzled.
// One box = 64 dims x 16 tokens of one KV head (2 KB, 128-byte swizzle) in every
// layout.  The map is 4-D, (dim, d1, d2, page): NHD has d1 = head (256 B apart),
// d2 = token (Hkv * 256 B apart); HND has d1 = token (256 B apart), d2 = head
// (4 KB apart); pages are `page_stride` bytes apart (16 * Hkv * 256 when the
// cache is one contiguous tensor).
// fp8 caches: the same map with 1-byte elements and a 128-dim (128-byte) box,
// also 128-byte swizzled (the tensor core reads the rows as K-major K and
// MN-major V operands).
bool encode_cache_map_uncached(CUtensorMap* map, const void* base, int num_pages, int hkv, bool hnd,
                               uint64_t page_stride, bool fp8) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t row = (cuuint64_t)kHeadDim * (fp8 ? 1 : 2);
  const cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, hnd ? (cuuint64_t)kPageSize : (cuuint64_t)hkv,
                              hnd ? (cuuint64_t)hkv : (cuuint64_t)kPageSize, (cuuint64_t)num_pages};
  const cuuint64_t strides[3] = {row, hnd ? row * kPageSize : row * hkv, (cuuint64_t)page_stride};
  const cuuint32_t box[4] = {fp8 ? 128u : 64u, hnd ? (cuuint32_t)kPageSize : 1u, hnd ? 1u : (cuuint32_t)kPageSize, 1u};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B,
            // L2 fills of one head's row: 256 B for 16-bit elements, 128 B for fp8 (a
            // 256-byte fill there would also fetch the neighbouring head's row)
            fp8 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A serving loop passes the same caches on every call: keep the last few
// encoded maps per host thread (a map depends only on base, pages and heads;
// the element type does not matter to a copy of 2-byte elements).
bool encode_cache_map(CUtensorMap* map, const void* base, int num_pages, int hkv, bool hnd, uint64_t page_stride,
                      bool fp8) {
  struct Entry {
    const void* base;
    int num_pages, hkv;
    bool hnd, fp8;
    uint64_t page_stride;
    CUtensorMap map;
  };
  constexpr int kEntries = 8;
  thread_local Entry cache[kEntries] = {};
  thread_local int next = 0;
  for (int i = 0; i < kEntries; ++i) {
    if (cache[i].base == base && cache[i].num_pages == num_pages && cache[i].hkv == hkv && cache[i].hnd == hnd &&
        cache[i].fp8 == fp8 && cache[i].page_stride == page_stride && base != nullptr) {
      *map = cache[i].map;
      return true;
    }
  }
  if (!encode_cache_map_uncached(map, base, num_pages, hkv, hnd, page_stride, fp8)) return false;
  cache[next] = Entry{base, num_pages, hkv, hnd, fp8, page_stride, *map};
  next = (next + 1) % kEntries;
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Elements between consecutive pages (0 = contiguous cache) -> bytes.
uint64_t page_stride_bytes(int64_t page_stride, int hkv, int elem_bytes) {
  return (uint64_t)(page_stride > 0 ? page_stride : (int64_t)kPageSize * hkv * kHeadDim) * elem_bytes;
}

// Debug builds synchronise after each launch (outside stream capture) and
// report which kernel failed, so a device fault is tied to one launch.
#ifdef SQA_DEBUG_CHECKS
bool debug_sync(cudaStream_t stream, const char* what, int grid, int smem, const sqa_args* a) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return true;
  const cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    fprintf(stderr, "sqa debug: %s failed: %s (grid %d smem %d batch %d q_len %d hkv %d pages %d max_pages %d)\n",
            what, cudaGetErrorString(e), grid, smem, a->batch, a->q_len, a->num_kv_heads, a->num_pages,
            a->max_pages);
    return false;
  }
  return true;
}
#else
inline bool debug_sync(cudaStream_t, const char*, int, int, const sqa_args*) { return true; }
#endif

struct Plan {
  WarpShape shape;
  bool tc;  // tcgen05 kernel
  int grid;
  int stages;
  int smem;
  int kv_fp8 = 0;  // fp8 caches: 2 = 4-page blocks, 3 = 8-page blocks
  int cluster = 0;  // tcgen05 cluster mode: CTAs per segment (0 = cost-balanced ranges + merge kernel)
  int seg_split = 0;  // tcgen05 segment-aligned split: CTAs per segment (partials merged by the merge kernel)
  int segments;
  int pieces;
  size_t off_lse, off_o, off_timeline = 0, bytes;
};

int validate(const sqa_args* a) {
  if (!a) return SQA_ERR_INVALID_ARGUMENT;
  if (a->batch < 0 || a->q_len <= 0 || a->num_kv_heads <= 0 || a->num_pages <= 0 || a->max_pages <= 0)
    return SQA_ERR_INVALID_ARGUMENT;
  if (a->head_dim != kHeadDim || a->page_size != kPageSize) return SQA_ERR_UNSUPPORTED;
  if (a->num_q_heads != kGroup * a->num_kv_heads) return SQA_ERR_UNSUPPORTED;
  if (a->q_len > SQA_MAX_Q_LEN) return SQA_ERR_UNSUPPORTED;
  if (a->max_seq_len < 0 || a->num_ctas < 0 || a->min_pages_per_cta < 0) return SQA_ERR_INVALID_ARGUMENT;
  if (a->kernel < 0 || a->kernel > 2) return SQA_ERR_INVALID_ARGUMENT;
  if (a->dtype != SQA_DTYPE_F16 && a->dtype != SQA_DTYPE_BF16) return SQA_ERR_UNSUPPORTED;
  if (a->kv_layout != SQA_KV_NHD && a->kv_layout != SQA_KV_HND) return SQA_ERR_UNSUPPORTED;
  if (a->kv_dtype != SQA_KV_SAME && a->kv_dtype != SQA_KV_FP8_E4M3) return SQA_ERR_UNSUPPORTED;
  // The device schedule counts cost in 32 bits: every page x KV head plus the
  // charge of every segment start (at most the larger kernel's), so that the
  // total, a CTA's range ends and their sums stay below 2^31.
  const int max_seg_cost = kSegmentCostTc > kSegmentCostMma ? kSegmentCostTc : kSegmentCostMma;
  if ((long long)a->batch * a->num_kv_heads * ((long long)a->max_pages + max_seg_cost) > (1LL << 30))
    return SQA_ERR_UNSUPPORTED;
  // fp8 caches run on the tcgen05 kernel (fp16 or bf16 queries)
  if (a->kv_dtype == SQA_KV_FP8_E4M3 && a->kernel == 1) return SQA_ERR_UNSUPPORTED;
  // a page must hold 16 x Hkv x 128 elements and start 16-byte aligned (TMA strides)
  const int64_t align_elems = a->kv_dtype == SQA_KV_FP8_E4M3 ? 16 : 8;
  if (a->page_stride < 0 || (a->page_stride > 0 && (a->page_stride < (int64_t)kPageSize * a->num_kv_heads * kHeadDim ||
                                                    a->page_stride % align_elems != 0)))
    return SQA_ERR_INVALID_ARGUMENT;
  if (!(a->sm_scale >= 0.f) || !std::isfinite(a->sm_scale) || !std::isfinite(a->out_scale))
    return SQA_ERR_INVALID_ARGUMENT;
  if (a->min_seq_len < 0) return SQA_ERR_INVALID_ARGUMENT;
  if (a->cluster != 0 && a->cluster != 1 && a->cluster != 2 && a->cluster != 4 && a->cluster != 8 &&
      a->cluster != 16)
    return SQA_ERR_INVALID_ARGUMENT;
  if (a->cluster >= 2 && a->kernel == 1) return SQA_ERR_UNSUPPORTED;  // clusters are a tcgen05-kernel mode
  // unit indices are 32-bit on the device
  if ((long long)a->batch * a->num_kv_heads * a->max_pages >= (1ll << 31)) return SQA_ERR_UNSUPPORTED;
  if ((long long)a->num_pages * kPageSize >= (1ll << 31)) return SQA_ERR_UNSUPPORTED;
  return SQA_OK;
}

int validate_pointers(const sqa_args* a) {
  if (!a->query || !a->key_cache || !a->value_cache || !a->block_tables || !a->seq_lens)
    return SQA_ERR_INVALID_ARGUMENT;
  const bool full = a->out != nullptr;
  const bool partial = a->out_partial != nullptr && a->out_lse != nullptr;
  if (full == partial) return SQA_ERR_INVALID_ARGUMENT;  // exactly one output mode
  if (!aligned16(a->query) || !aligned16(a->key_cache) || !aligned16(a->value_cache)) return SQA_ERR_INVALID_ARGUMENT;
  if (full && !aligned16(a->out)) return SQA_ERR_INVALID_ARGUMENT;
  if (partial && !aligned16(a->out_partial)) return SQA_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a->block_tables) & 3u) || (reinterpret_cast<uintptr_t>(a->seq_lens) & 3u))
    return SQA_ERR_INVALID_ARGUMENT;
  return SQA_OK;
}

int make_plan(const sqa_args* a, int device, Plan* plan) {
  const int sms = sm_count(device);
  if (sms <= 0) return SQA_ERR_CUDA;
  Plan pl;
  pl.shape = warp_shape_for(a->q_len);
  pl.segments = a->batch * a->num_kv_heads;
  long long pages_upper = a->max_pages;
  if (a->max_seq_len > 0) {
    const long long need = (a->max_seq_len + kPageSize - 1) / kPageSize;
    if (need < pages_upper) pages_upper = need;
  }
  const long long units_upper = (long long)pl.segments * pages_upper;
  // Auto (measured on B200): the tcgen05 kernel streams at the HBM roofline for
  // every q_len but has the longer per-CTA latency chain (TMEM, asynchronous MMA
  // completions, replica merge); the warp-level kernel wins small launches.
  if (a->kv_dtype == SQA_KV_FP8_E4M3) {
    pl.tc = true;  // the fp8 products live in the tcgen05 kernel
  } else if (a->kernel == 0) {
    if (a->q_len >= 9) pl.tc = true;
    else if (a->q_len >= 5) pl.tc = units_upper > kAutoTcUnitsQ8;
    else if (a->q_len >= 3) pl.tc = units_upper >= kAutoTcUnitsQ4;
    else pl.tc = units_upper >= kAutoTcUnitsQ2;
  } else {
    pl.tc = a->kernel == 2;
  }
  if (a->cluster >= 2) pl.tc = true;  // a requested cluster size runs the tcgen05 kernel
  const int ctas_per_sm = pl.tc ? 1 : kCtasPerSm;  // tcgen05: one CTA per SM (all of TMEM)
  const int min_pages = a->min_pages_per_cta > 0 ? a->min_pages_per_cta : kDefaultMinPagesPerCta;
  long long grid = a->num_ctas > 0 ? a->num_ctas : (long long)sms * ctas_per_sm;
  if (a->num_ctas <= 0) {
    const long long by_work = (units_upper + min_pages - 1) / min_pages;
    if (by_work < grid) grid = by_work;
  }
  if (grid < 1) grid = 1;
  pl.grid = (int)grid;
  const int grid_default = pl.grid;
  if (pl.tc && a->num_ctas == 0 && a->cluster != 1) {
    // Cluster mode: every (sequence, KV head) segment split evenly over C CTAs of one
    // thread-block cluster, parts reduced through distributed shared memory.  Measured
    // on B200: it removes the merge launch but runs on segments x C <= SMs CTAs, and
    // one CTA streams at most ~55 GB/s, so long segments need all the SMs of the
    // cost-balanced schedule (cfg2: 27.0 us in 4-CTA clusters against 26.4 us); it wins
    // on short near-uniform segments (q4 x 1K x 4: 11.4 against 13.2 us).  Auto: both
    // length hints within 15%, q_len <= 8, 16..32 pages per CTA, clusters of 4 or 2,
    // every cluster resident at once.
    const long long segs = pl.segments;
    if (a->cluster >= 2) {
      pl.cluster = a->cluster;
    } else if (a->max_seq_len > 0 && a->min_seq_len > 0 && 100LL * a->min_seq_len >= 85LL * a->max_seq_len &&
               a->q_len <= 8) {
      const int cands[2] = {4, 2};
      for (int c : cands) {
        if (segs * c <= sms && pages_upper / c >= 16 && pages_upper / c <= 32) {
          pl.cluster = c;
          break;
        }
      }
    }
    if (pl.cluster) pl.grid = (int)(segs * pl.cluster);
  }
  // Segment-aligned split: with near-uniform length hints and fewer segments than
  // CTAs, every segment split evenly over k = grid / segments CTAs, so that no CTA
  // crosses a segment boundary.  In the cost-balanced schedule a CTA that does (a
  // batch-1 call has 8 segments over 148 CTAs) ends ~2 us after the others: a second
  // piece epilogue and pipeline refill on the same page count.  Only where the split
  // keeps >= 90% of the CTAs busy and gives each >= 16 pages; a wrong hint costs
  // time, not correctness.
  if (pl.tc && a->num_ctas == 0 && !pl.cluster && a->max_seq_len > 0 && a->min_seq_len > 0 &&
      100LL * a->min_seq_len >= 85LL * a->max_seq_len) {
    const long long segs = pl.segments;
    const long long k = segs > 0 ? grid_default / segs : 0;
    if (k >= 2 && 10 * segs * k >= 9LL * grid_default && pages_upper >= 16 * k) {
      pl.seg_split = (int)k;
      pl.grid = (int)(segs * k);
    }
  }
  if (pl.tc) {
    // a ring of blocks in up to 227 KB of shared memory: 32 KB (16-bit caches, 4
    // pages), fp8 caches 16 KB (4 pages) or, for long per-CTA ranges, 32 KB (8 pages)
    if (a->kv_dtype == SQA_KV_FP8_E4M3)
      pl.kv_fp8 = units_upper >= (long long)kFp8LongRangeUnits * pl.grid ? 3 : 2;
    const int fixed = split_kv_tc_smem_bytes(0, pl.kv_fp8);
    pl.stages = (kMaxSmemPerCta - fixed) / (split_kv_tc_block_bytes(pl.kv_fp8) + 16);
    if (pl.stages > kMaxStages) pl.stages = kMaxStages;
    pl.smem = split_kv_tc_smem_bytes(pl.stages, pl.kv_fp8);
    if (pl.cluster) {
      // every cluster must be resident at once for the auto choice; a requested size
      // only needs the device to launch it (more clusters run in waves)
      const int fit = split_kv_tc_max_clusters(pl.cluster, pl.smem);
      if (fit < 1) {
        if (a->cluster >= 2) return SQA_ERR_UNSUPPORTED;
        pl.cluster = 0;
      } else if (a->cluster == 0 && fit < pl.segments) {
        pl.cluster = 0;
      }
      if (!pl.cluster && !pl.seg_split) pl.grid = grid_default;
    }
  } else {
    const int fixed = split_kv_smem_bytes(pl.shape, 0);
    pl.stages = (kSmemPerCta - fixed) / (kStageBytes + 24);
    if (pl.stages > kMaxStages) pl.stages = kMaxStages;
    pl.smem = split_kv_smem_bytes(pl.shape, pl.stages);
  }
  pl.pieces = pl.grid + pl.segments;  // piece index = cta + segment < grid + segments - 1

  pl.off_lse = kAlign;  // [0, 256): device status word
  pl.off_o = align_up(pl.off_lse + (size_t)pl.pieces * pl.shape.rows_pad * sizeof(float));
  pl.bytes = align_up(pl.off_o + (size_t)pl.pieces * pl.shape.rows_pad * kHeadDim * sizeof(float));
#ifdef SQA_DEBUG_TIMELINE
  // trace buffer at the end: 8 stamps per split CTA, 4 per merge CTA
  pl.off_timeline = pl.bytes;
  pl.bytes = align_up(pl.bytes + ((size_t)pl.grid * 32 + (size_t)pl.segments * 16 * 4) * 8);
#endif
  *plan = pl;
  return SQA_OK;
}

int current_device(int device) {
  if (device >= 0) return device;
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

}  // namespace
}  // namespace sqa

using namespace sqa;

extern "C" {

int sqa_abi_version(void) { return kAbiVersion; }

const char* sqa_status_string(int status) {
  switch (status) {
    case SQA_OK: return "ok";
    case SQA_ERR_INVALID_ARGUMENT: return "invalid argument (null/misaligned pointer or bad shape)";
    case SQA_ERR_UNSUPPORTED: return "unsupported shape (needs head_dim 128, page_size 16, Hq = 4*Hkv, 1 <= q_len <= 16)";
    case SQA_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case SQA_ERR_CUDA: return "CUDA call failed";
    case SQA_ERR_DEVICE: return "device reported an error (see the SQA_DEV_* bits)";
    default: return "unknown status";
  }
}

size_t sqa_workspace_bytes(const sqa_args* args, int device, int* status) {
  int st = validate(args);
  Plan pl;
  if (st == SQA_OK) {
    const int dev = current_device(device);
    st = dev < 0 ? SQA_ERR_CUDA : make_plan(args, dev, &pl);
  }
  if (status) *status = st;
  return st == SQA_OK ? pl.bytes : 0;
}

int sqa_selected_kernel(const sqa_args* args, int device) {
  int st = validate(args);
  if (st != SQA_OK) return -st;
  const int dev = current_device(device);
  if (dev < 0) return -SQA_ERR_CUDA;
  Plan pl;
  st = make_plan(args, dev, &pl);
  if (st != SQA_OK) return -st;
  return pl.tc ? 2 + 100 * pl.cluster + 10000 * pl.seg_split : 1;
}

int sqa_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < kAlign) return SQA_ERR_INVALID_ARGUMENT;
  return cudaMemsetAsync(workspace, 0, workspace_bytes, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? SQA_OK
             : SQA_ERR_CUDA;
}

namespace {
// Under stream capture: an event-record node that depends on the stream's current
// capture dependencies without joining them, so the next captured kernel keeps its
// programmatic (early-launch) edge to the previous one.  The event then fires when
// the work captured so far has completed: before a split-KV launch, when the previous
// call's merge ends (the moment the split kernel's dependency wait returns); after
// it, when the split kernel ends.  The graph keeps such unjoined nodes.
cudaError_t record_side_branch(cudaEvent_t ev, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  const cudaGraphEdgeData* edges = nullptr;
  size_t n = 0;
  cudaError_t e = cudaStreamGetCaptureInfo_v3(stream, &cs, nullptr, &graph, &deps, &edges, &n);
  if (e != cudaSuccess) return e;
  if (cs != cudaStreamCaptureStatusActive || graph == nullptr) return cudaErrorStreamCaptureInvalidated;
  cudaGraphNode_t node = nullptr;
  return cudaGraphAddEventRecordNode(&node, graph, deps, n, ev);
}

int forward_impl(const sqa_args* a, void* workspace, size_t workspace_bytes, void* stream_ptr,
                 void* ev_before, void* ev_after) {
  int st = validate(a);
  if (st != SQA_OK) return st;
  st = validate_pointers(a);
  if (st != SQA_OK) return st;
  if (a->batch == 0) return SQA_OK;
  const int dev = current_device(-1);
  if (dev < 0) return SQA_ERR_CUDA;
  Plan pl;
  st = make_plan(a, dev, &pl);
  if (st != SQA_OK) return st;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1))) return SQA_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < pl.bytes) return SQA_ERR_WORKSPACE_TOO_SMALL;

  CUtensorMap tm_k, tm_v;
  const bool hnd = a->kv_layout == SQA_KV_HND;
  const bool fp8 = a->kv_dtype == SQA_KV_FP8_E4M3;
  const uint64_t page_stride = page_stride_bytes(a->page_stride, a->num_kv_heads, fp8 ? 1 : 2);
  if (!encode_cache_map(&tm_k, a->key_cache, a->num_pages, a->num_kv_heads, hnd, page_stride, fp8) ||
      !encode_cache_map(&tm_v, a->value_cache, a->num_pages, a->num_kv_heads, hnd, page_stride, fp8))
    return SQA_ERR_CUDA;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  SplitKvParams p = {};
  p.q = static_cast<const __half*>(a->query);
  p.block_tables = a->block_tables;
  p.seq_lens = a->seq_lens;
  p.mask_lens = a->mask_lens;
  p.out = static_cast<__half*>(a->out);
  p.out_o = a->out_partial;
  p.out_lse = a->out_lse;
  p.ws_o = reinterpret_cast<float*>(ws + pl.off_o);
  p.ws_lse = reinterpret_cast<float*>(ws + pl.off_lse);
  p.status = reinterpret_cast<unsigned int*>(ws);
  p.batch = a->batch;
  p.q_len = a->q_len;
  p.hq = a->num_q_heads;
  p.hkv = a->num_kv_heads;
  p.max_pages = a->max_pages;
  p.num_pages = a->num_pages;
  p.num_stages = pl.stages;
  p.num_pieces = pl.pieces;
  p.rows_pad = pl.shape.rows_pad;
  p.timeline = pl.off_timeline ? reinterpret_cast<unsigned long long*>(ws + pl.off_timeline) : nullptr;
  p.scale_log2 = 1.4426950408889634f * (a->sm_scale > 0.f ? a->sm_scale : 1.f / sqrtf((float)kHeadDim));
  p.bf16 = a->dtype == SQA_DTYPE_BF16;
  p.hnd = hnd;
  p.out_scale = a->out_scale != 0.f ? a->out_scale : 1.f;
  p.kv_fp8 = pl.kv_fp8;
  p.seg_cost = pl.tc ? kSegmentCostTc : kSegmentCostMma;
  p.cluster = pl.cluster;
  p.seg_split = pl.seg_split;

  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  // Timing events.  Eagerly: records on the stream before and after the split-KV
  // launch.  Under stream capture: event-record nodes on side branches of the graph
  // (record_side_branch), so the launches keep their programmatic edges.
  bool capturing = false;
  if (ev_before || ev_after) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return SQA_ERR_CUDA;
    capturing = cs == cudaStreamCaptureStatusActive;
  }
  auto record = [&](void* ev) {
    if (!ev) return true;
    const cudaEvent_t e = reinterpret_cast<cudaEvent_t>(ev);
    return (capturing ? record_side_branch(e, stream) : cudaEventRecord(e, stream)) == cudaSuccess;
  };
  if (!record(ev_before)) return SQA_ERR_CUDA;
  const cudaError_t launched = pl.tc ? launch_split_kv_tc(p, tm_k, tm_v, pl.grid, pl.smem, stream)
                                    : launch_split_kv(p, tm_k, tm_v, pl.grid, pl.smem, stream);
  if (launched != cudaSuccess) return SQA_ERR_CUDA;
  if (!debug_sync(stream, "split-KV kernel", pl.grid, pl.smem, a)) return SQA_ERR_CUDA;
  if (!record(ev_after)) return SQA_ERR_CUDA;

  MergeParams m = {};
  m.parts_o = p.ws_o;
  m.parts_lse = p.ws_lse;
  m.seq_lens = a->seq_lens;
  m.out = p.out;
  m.out_o = p.out_o;
  m.out_lse = p.out_lse;
  m.status = p.status;
  m.timeline = p.timeline ? p.timeline + (size_t)pl.grid * 32 : nullptr;
  m.rows = 0;
  m.num_parts = pl.pieces;
  m.piece_rows = pl.shape.rows_pad;
  m.batch = a->batch;
  m.q_len = a->q_len;
  m.hq = a->num_q_heads;
  m.hkv = a->num_kv_heads;
  m.max_pages = a->max_pages;
  m.bf16 = p.bf16;
  m.split_grid = pl.grid;
  m.seg_cost = p.seg_cost;
  m.seg_split = pl.seg_split;
  if (pl.cluster) return SQA_OK;  // the clusters reduced every segment themselves
  if (launch_segment_merge(m, pl.shape.rows_pad, stream) != cudaSuccess) return SQA_ERR_CUDA;
  if (!debug_sync(stream, "merge kernel", pl.segments, 0, a)) return SQA_ERR_CUDA;
  return SQA_OK;
}
}  // namespace

int sqa_forward(const sqa_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(a, workspace, workspace_bytes, stream, nullptr, nullptr);
}

int sqa_forward_timed(const sqa_args* a, void* workspace, size_t workspace_bytes, void* stream,
                      void* event_before, void* event_after) {
  return forward_impl(a, workspace, workspace_bytes, stream, event_before, event_after);
}

int sqa_merge_partials(const float* parts_o, const float* parts_lse, int32_t num_parts, int64_t rows,
                       void* out, float* out_o, float* out_lse, void* stream) {
  if (!parts_o || !parts_lse || num_parts <= 0 || rows < 0) return SQA_ERR_INVALID_ARGUMENT;
  if (!out && !out_o && !out_lse) return SQA_ERR_INVALID_ARGUMENT;
  if (!aligned16(parts_o) || (out && !aligned16(out)) || (out_o && !aligned16(out_o)))
    return SQA_ERR_INVALID_ARGUMENT;
  if (rows == 0) return SQA_OK;
  if ((rows + 3) / 4 >= (1ll << 31)) return SQA_ERR_UNSUPPORTED;
  MergeParams m = {};
  m.parts_o = parts_o;
  m.parts_lse = parts_lse;
  m.out = static_cast<__half*>(out);
  m.out_o = out_o;
  m.out_lse = out_lse;
  m.rows = rows;
  m.bf16 = 0;
  m.num_parts = num_parts;
  return launch_partials_merge(m, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? SQA_OK : SQA_ERR_CUDA;
}

int sqa_read_device_status(void* workspace, uint32_t* device_bits, int clear, void* stream_ptr) {
  if (!workspace) return SQA_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  uint32_t bits = 0;
  if (cudaMemcpyAsync(&bits, workspace, sizeof(bits), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return SQA_ERR_CUDA;
  if (clear && cudaMemsetAsync(workspace, 0, sizeof(bits), stream) != cudaSuccess) return SQA_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return SQA_ERR_CUDA;
  if (device_bits) *device_bits = bits;
  return bits ? SQA_ERR_DEVICE : SQA_OK;
}

}  // extern "C"
