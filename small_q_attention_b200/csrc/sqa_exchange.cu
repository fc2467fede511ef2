// sqa_exchange.cu -- long-context split across the GPUs of one node: every
// rank's partial (O, LSE) goes to rank 0 with peer stores over NVLink, and
// rank 0 merges them.
//
// The upstream has no multi-GPU code; this is the exchange step of splitting
// one sequence's KV range over GPUs (each rank runs the shard form of the
// operator over the pages it holds, mask_lens in whole-sequence coordinates).
// It replaces an all-gather to every rank plus a merge on every rank: one
// copy of each partial crosses NVLink, once, straight from the sending kernel.
//
// Memory: each rank allocates one block (cudaMalloc, at set-up) and exports an
// IPC handle; every rank maps the others' blocks.  Block layout:
//   [0, 256)   header: status word (u32, offset 0), epoch (u64, 8), ack (u64,
//              16), send arrivals (u32, 24), merge arrivals (u32, 28),
//              flags[world] (u64 each, from 64)
//   [256, ..)  slots: O [world, rows, 128] fp32, then LSE [world, rows] fp32
// Only rank 0's slots and flags are written (by every rank, slot r by rank r);
// rank 0 writes every rank's ack.
//
// Protocol per step, epoch e (a device-resident counter, so CUDA-graph replays
// keep counting):
//   every rank (send kernel): wait until its ack >= e - 1 (rank 0 has consumed
//     the previous step's slot), store its (O, LSE) into slot r on rank 0,
//     fence at system scope, and the last CTA to finish sets the local epoch to
//     e and stores flag[r] = e on rank 0 with release semantics;
//   rank 0 (merge kernel): wait until flag[r] >= e for every r, merge the
//     slots into the output, and the last CTA stores ack = e on every rank.
// Every wait is bounded (about a second of %globaltimer); a wait that gives up
// sets SQA_DEV_TIMEOUT in the local status word and the kernel carries on (the
// output is then not valid).  No load here is a TMA or bulk copy: plain
// loads and stores only, and no multicast of any kind.
#include <algorithm>
#include <new>

#include "../../include/small_q_attention.h"
#include "sqa_internal.h"
#include "sqa_merge_row.cuh"
#include "sqa_ptx.cuh"

namespace sqa {
namespace {

constexpr int kMaxWorld = 8;
constexpr size_t kHeader = 256;
constexpr size_t kOffEpoch = 8, kOffAck = 16, kOffArriveSend = 24, kOffArriveMerge = 28, kOffFlags = 64;
constexpr uint64_t kWaitLimitNs = 1000000000ull;

struct LcSendParams {
  const float* o;        // this rank's partial [rows, 128]
  const float* lse;      // [rows]
  float* slot_o;         // rank 0's slot for this rank [rows, 128]
  float* slot_lse;       // [rows]
  unsigned long long* flag;   // rank 0's flag for this rank
  uint8_t* local;        // this rank's header
  long long rows;
};

struct LcMergeParams {
  const float* slots_o;  // rank 0's slots [world, rows, 128]
  const float* slots_lse;
  uint8_t* local;        // rank 0's header (flags live here)
  unsigned long long* acks[kMaxWorld];  // every rank's ack word
  __half* out;           // [rows, 128] fp16 or bf16
  long long rows;
  int world;
  int bf16;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait until *p >= target; false (and the timeout bit set) when it gives up.
__device__ bool wait_at_least(const unsigned long long* p, unsigned long long target, unsigned int* status) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  unsigned int backoff = 32;
  while (ld_acquire_sys(p) < target) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, SQA_DEV_TIMEOUT);
      return false;
    }
    __nanosleep(backoff);
    if (backoff < 1024) backoff <<= 1;
  }
  return true;
}

__global__ void __launch_bounds__(256) sqa_lc_send_kernel(const LcSendParams p) {
  allow_dependent_launch();
  grid_dependency_wait();  // the partial (O, LSE) of this step is complete
  unsigned int* status = reinterpret_cast<unsigned int*>(p.local);
  auto* epoch = reinterpret_cast<unsigned long long*>(p.local + kOffEpoch);
  auto* ack = reinterpret_cast<unsigned long long*>(p.local + kOffAck);
  auto* arrive = reinterpret_cast<unsigned int*>(p.local + kOffArriveSend);
  // The epoch only moves when every CTA of this grid has finished (last CTA below).
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(epoch) + 1;
  __shared__ int go;
  if (threadIdx.x == 0) go = wait_at_least(ack, e - 1, status) ? 1 : 0;
  __syncthreads();
  if (go) {
    const long long n4 = p.rows * (kHeadDim / 4);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
      reinterpret_cast<float4*>(p.slot_o)[i] = __ldg(reinterpret_cast<const float4*>(p.o) + i);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < p.rows; i += stride)
      p.slot_lse[i] = __ldg(p.lse + i);
  }
  // The CTA's peer stores precede the barrier; one system-scope fence by thread 0
  // after it orders all of them before the arrival (and, through the last CTA's
  // fence, before the flag).  A fence in every thread cost ~16 us per launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const bool last = atomicAdd(arrive, 1u) == gridDim.x - 1;
    if (last) {
      __threadfence_system();
      *arrive = 0u;
      *reinterpret_cast<volatile unsigned long long*>(epoch) = e;
      st_release_sys(p.flag, e);
    }
  }
}

__global__ void __launch_bounds__(256) sqa_lc_merge_kernel(const LcMergeParams p) {
  allow_dependent_launch();
  grid_dependency_wait();  // this rank's own send of the step is complete (the epoch moved)
  unsigned int* status = reinterpret_cast<unsigned int*>(p.local);
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(p.local + kOffEpoch);
  auto* flags = reinterpret_cast<unsigned long long*>(p.local + kOffFlags);
  auto* arrive = reinterpret_cast<unsigned int*>(p.local + kOffArriveMerge);
  if (threadIdx.x == 0) {
    for (int r = 0; r < p.world; ++r) wait_at_least(flags + r, e, status);
  }
  __syncthreads();
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row < p.rows)  // the slots were written by other GPUs: read through L2
    merge_row<true>(p.slots_o + row * kHeadDim, (size_t)p.rows * kHeadDim, p.slots_lse + row, (size_t)p.rows,
                    p.world, p.out + row * kHeadDim, nullptr, nullptr, p.bf16 != 0);
  __syncthreads();  // every read of the slots in this CTA is done before the acks below
  if (threadIdx.x == 0) {
    __threadfence_system();
    const bool last = atomicAdd(arrive, 1u) == gridDim.x - 1;
    if (last) {
      __threadfence_system();
      *arrive = 0u;
      for (int r = 0; r < p.world; ++r) st_release_sys(p.acks[r], e);
    }
  }
}

template <typename P>
cudaError_t launch_pdl256(void (*kernel)(const P), int grid, const P& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, p);
  return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace
}  // namespace sqa

using namespace sqa;

struct sqa_lc_group {
  int rank = 0, world = 0, device = -1;
  long long rows = 0;
  size_t bytes = 0;
  uint8_t* local = nullptr;                // this rank's block
  uint8_t* blocks[kMaxWorld] = {nullptr};  // every rank's block as mapped here (own block included)
  bool opened[kMaxWorld] = {false};
};

namespace {
size_t block_bytes(int world, long long rows) {
  const size_t o = (size_t)world * rows * kHeadDim * sizeof(float);
  const size_t l = ((size_t)world * rows * sizeof(float) + 255) / 256 * 256;
  return kHeader + o + l;
}
float* slots_o(uint8_t* block) { return reinterpret_cast<float*>(block + kHeader); }
float* slots_lse(uint8_t* block, int world, long long rows) {
  return reinterpret_cast<float*>(block + kHeader + (size_t)world * rows * kHeadDim * sizeof(float));
}
}  // namespace

extern "C" {

size_t sqa_lc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int sqa_lc_create(int32_t rank, int32_t world, int64_t rows, sqa_lc_group** group, void* handle_out) {
  if (!group || !handle_out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || rows <= 0)
    return SQA_ERR_INVALID_ARGUMENT;
  if (rows > (1ll << 24)) return SQA_ERR_UNSUPPORTED;
  *group = nullptr;
  auto* g = new (std::nothrow) sqa_lc_group();
  if (!g) return SQA_ERR_CUDA;
  g->rank = rank;
  g->world = world;
  g->rows = rows;
  g->bytes = block_bytes(world, rows);
  if (cudaGetDevice(&g->device) != cudaSuccess || cudaMalloc(&g->local, g->bytes) != cudaSuccess ||
      cudaMemset(g->local, 0, g->bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), g->local) != cudaSuccess) {
    if (g->local) cudaFree(g->local);
    delete g;
    return SQA_ERR_CUDA;
  }
  g->blocks[rank] = g->local;
  *group = g;
  return SQA_OK;
}

int sqa_lc_connect(sqa_lc_group* g, const void* handles) {
  if (!g || !handles) return SQA_ERR_INVALID_ARGUMENT;
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < g->world; ++r) {
    if (r == g->rank || g->blocks[r]) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SQA_ERR_CUDA;
    g->blocks[r] = static_cast<uint8_t*>(p);
    g->opened[r] = true;
  }
  return SQA_OK;
}

int sqa_lc_exchange(sqa_lc_group* g, const float* o, const float* lse, void* out, int32_t out_bf16,
                    void* stream_ptr) {
  if (!g || !o || !lse) return SQA_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < g->world; ++r)
    if (!g->blocks[r]) return SQA_ERR_INVALID_ARGUMENT;  // not connected
  if (g->rank == 0 && !out) return SQA_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(o) & 15u) || (out && (reinterpret_cast<uintptr_t>(out) & 15u)))
    return SQA_ERR_INVALID_ARGUMENT;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  uint8_t* root = g->blocks[0];
  LcSendParams s;
  s.o = o;
  s.lse = lse;
  s.slot_o = slots_o(root) + (size_t)g->rank * g->rows * kHeadDim;
  s.slot_lse = slots_lse(root, g->world, g->rows) + (size_t)g->rank * g->rows;
  s.flag = reinterpret_cast<unsigned long long*>(root + kOffFlags) + g->rank;
  s.local = g->local;
  s.rows = g->rows;
  const long long n4 = g->rows * (kHeadDim / 4);
  const int send_grid = (int)std::min<long long>(64, (n4 + 255) / 256);
  if (launch_pdl256(sqa_lc_send_kernel, send_grid, s, stream) != cudaSuccess) return SQA_ERR_CUDA;
  if (g->rank != 0) return SQA_OK;
  LcMergeParams m = {};
  m.slots_o = slots_o(g->local);
  m.slots_lse = slots_lse(g->local, g->world, g->rows);
  m.local = g->local;
  for (int r = 0; r < g->world; ++r) m.acks[r] = reinterpret_cast<unsigned long long*>(g->blocks[r] + kOffAck);
  m.out = static_cast<__half*>(out);
  m.rows = g->rows;
  m.world = g->world;
  m.bf16 = out_bf16 ? 1 : 0;
  const int merge_grid = (int)((g->rows + 7) / 8);  // one warp per row, 8 per CTA
  return launch_pdl256(sqa_lc_merge_kernel, merge_grid, m, stream) == cudaSuccess ? SQA_OK : SQA_ERR_CUDA;
}

int sqa_lc_read_status(sqa_lc_group* g, uint32_t* device_bits, int clear, void* stream) {
  if (!g) return SQA_ERR_INVALID_ARGUMENT;
  return sqa_read_device_status(g->local, device_bits, clear, stream);
}

int sqa_lc_disconnect(sqa_lc_group* g) {
  if (!g) return SQA_OK;
  int st = SQA_OK;
  for (int r = 0; r < g->world; ++r) {
    if (g->opened[r] && cudaIpcCloseMemHandle(g->blocks[r]) != cudaSuccess) st = SQA_ERR_CUDA;
    if (r != g->rank) g->blocks[r] = nullptr;
    g->opened[r] = false;
  }
  return st;
}

int sqa_lc_destroy(sqa_lc_group* g) {
  if (!g) return SQA_OK;
  int st = sqa_lc_disconnect(g);
  if (g->local && cudaFree(g->local) != cudaSuccess) st = SQA_ERR_CUDA;
  delete g;
  return st;
}

}  // extern "C"
