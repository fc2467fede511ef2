// sqa_noalloc.cu -- sqa_forward_noalloc: the operator with built-in scratch.
//
// Some callers cannot allocate device memory for the workspace: a binding
// that calls this C ABI directly from a language with no CUDA allocator of
// its own, or a serving engine that hands almost all of HBM to its KV-cache
// pool up front and forbids allocations during a decode step (cudaMalloc
// there can fail for lack of memory, and cudaMalloc/cudaFree synchronise the
// device).  For them this entry point takes its scratch from a fixed array
// in device memory that is part of this library, so the caller passes only
// inputs and outputs.
//
// The array costs SQA_NOALLOC_SCRATCH_BYTES on every GPU that loads the
// library, for the life of the process.  Its device address is looked up
// once per device with cudaGetSymbolAddress on the first call made with that
// device current (the host-side name of the array is only a stand-in and must
// never be handed to a kernel).  The address belongs to the device's primary
// context: after cudaDeviceReset, or with another context made current, the
// cached address is stale, and neither case is supported.  All calls share
// the array: calls that overlap on the GPU (different streams, or different
// host threads) race on it and must be serialised by the caller.
#include <mutex>

#include "../../include/small_q_attention.h"
#include <cuda_runtime.h>

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kStatusBytes = 256;  // the device status word lives at offset 0

static __device__ __align__(256) unsigned char g_noalloc_scratch[SQA_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device.
int scratch_address(void** out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return SQA_ERR_CUDA;
  if (device < 0 || device >= kMaxDevices) return SQA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return SQA_ERR_CUDA;
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return SQA_OK;
}

}  // namespace

extern "C" SQA_API int sqa_forward_noalloc(const sqa_args* args, void* stream) {
  int st = SQA_OK;
  const size_t need = sqa_workspace_bytes(args, -1, &st);
  if (st != SQA_OK) return st;
  if (need > (size_t)SQA_NOALLOC_SCRATCH_BYTES) return SQA_ERR_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != SQA_OK) return st;
  // The array keeps the previous call's contents; only the sticky status word
  // must start at zero (the split partials are written before they are read
  // within a call).
  if (cudaMemsetAsync(scratch, 0, kStatusBytes, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return SQA_ERR_CUDA;
  return sqa_forward(args, scratch, SQA_NOALLOC_SCRATCH_BYTES, stream);
}

// The status word of the last sqa_forward_noalloc call on the current device:
// the same read as sqa_read_device_status, on the built-in scratch array.
extern "C" SQA_API int sqa_noalloc_read_device_status(uint32_t* device_bits, int clear, void* stream) {
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != SQA_OK) return st;
  return sqa_read_device_status(scratch, device_bits, clear, stream);
}
