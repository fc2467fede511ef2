// sqa_append.cu -- the cache-append step before MTP attention: write the K/V
// of the q_len new (draft) tokens of every sequence into their page slots.
//
// The upstream operator takes seq_lens as the length *after* the draft tokens
// were appended (src/small_q_attention/reference.py:25) and leaves the append
// to the caller; this is that step.  Token qi of sequence b is position
// t = seq_lens[b] - q_len + qi, stored in page block_tables[b, t / 16], slot
// t % 16, at element ((page * 16 + slot) * Hkv + kvh) * 128 + d of each cache
// (the layout of csrc/small_q_attention_ext.cu:466).
//
// One thread moves 16 bytes: a token row of one KV head (256 B; 128 B for fp8) is 16 (8) threads,
// consecutive threads read consecutive bytes of new_keys / new_values and
// write consecutive bytes of one 256-byte cache row.  The step is a pure copy
// (bit-exact).  A sequence shorter than q_len or with more pages than its
// table row is skipped whole, a token whose page id is outside the cache is
// skipped; both are reported in the status word (same bits as the attention).
#include "small_q_attention.h"
#include "sqa_internal.h"
#include "sqa_ptx.cuh"

namespace sqa {
namespace {

struct AppendParams {
  const uint4* new_k;       // [batch, q_len, hkv, 128] fp16, 16 uint4 per row
  const uint4* new_v;
  uint4* k_cache;           // [num_pages, 16, hkv, 128] fp16
  uint4* v_cache;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  unsigned int* status;     // may be null
  long long items;          // batch * q_len * hkv * row16
  int row16;                // 16-byte units per token row of one KV head (16 for 2-byte, 8 for 1-byte elements)
  int q_len, hkv, num_pages, max_pages;
  int hnd;                  // caches are [P, Hkv, 16, 128] (else [P, 16, Hkv, 128])
  long long page_stride16;  // 16-byte units from one page to the next
};

__global__ void __launch_bounds__(256) sqa_cache_append_kernel(const AppendParams p) {
  grid_dependency_wait();    // the previous kernel may have produced the new K/V or the tables
  allow_dependent_launch();  // the attention that follows waits for this grid to finish
  unsigned int bad = 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < p.items; i += stride) {
    const long long row = i / p.row16;  // (b, qi, kvh)
    const int c = (int)(i - row * p.row16);
    const int h = (int)(row % p.hkv);
    const long long bq = row / p.hkv;
    const int qi = (int)(bq % p.q_len);
    const int b = (int)(bq / p.q_len);
    const int len = __ldg(p.seq_lens + b);
    const int t = len - p.q_len + qi;
    unsigned int err = 0;
    int page = 0;
    if (len < p.q_len) {
      err = 4u;  // SQA_DEV_SEQ_TOO_SHORT: the whole sequence is skipped
    } else if ((len + kPageSize - 1) / kPageSize > p.max_pages) {
      err = 2u;  // SQA_DEV_SEQ_TOO_LONG: the whole sequence is skipped
    } else {
      page = __ldg(p.block_tables + (size_t)b * p.max_pages + t / kPageSize);
      if (page < 0 || page >= p.num_pages) err = 8u;  // SQA_DEV_BAD_PAGE: this token is skipped
    }
    if (err) {
      bad |= err;
      continue;
    }
    const size_t in_page = p.hnd ? ((size_t)h * kPageSize + (t % kPageSize)) * p.row16 + c
                                 : ((size_t)(t % kPageSize) * p.hkv + h) * p.row16 + c;
    const size_t dst = (size_t)page * p.page_stride16 + in_page;
    p.k_cache[dst] = __ldg(p.new_k + i);
    p.v_cache[dst] = __ldg(p.new_v + i);
  }
  if (bad && p.status != nullptr) atomicOr(p.status, bad);
}

}  // namespace
}  // namespace sqa

using namespace sqa;

extern "C" SQA_API int sqa_cache_append(const sqa_append_args* a, void* stream) {
  if (a == nullptr) return SQA_ERR_INVALID_ARGUMENT;
  if (a->head_dim != kHeadDim || a->page_size != kPageSize) return SQA_ERR_UNSUPPORTED;
  if (a->batch < 0 || a->q_len <= 0 || a->num_kv_heads <= 0 || a->num_pages <= 0 || a->max_pages <= 0)
    return SQA_ERR_INVALID_ARGUMENT;
  if (a->kv_layout != SQA_KV_NHD && a->kv_layout != SQA_KV_HND) return SQA_ERR_UNSUPPORTED;
  if (a->kv_dtype != SQA_KV_SAME && a->kv_dtype != SQA_KV_FP8_E4M3) return SQA_ERR_UNSUPPORTED;
  if (a->page_stride < 0 || (a->page_stride > 0 && (a->page_stride < (int64_t)kPageSize * a->num_kv_heads * kHeadDim ||
                                                    a->page_stride % (a->kv_dtype == SQA_KV_FP8_E4M3 ? 16 : 8) != 0)))
    return SQA_ERR_INVALID_ARGUMENT;
  if (a->batch == 0) return SQA_OK;
  if (!a->new_keys || !a->new_values || !a->key_cache || !a->value_cache || !a->block_tables || !a->seq_lens)
    return SQA_ERR_INVALID_ARGUMENT;
  const uintptr_t wide = reinterpret_cast<uintptr_t>(a->new_keys) | reinterpret_cast<uintptr_t>(a->new_values) |
                         reinterpret_cast<uintptr_t>(a->key_cache) | reinterpret_cast<uintptr_t>(a->value_cache);
  const uintptr_t narrow = reinterpret_cast<uintptr_t>(a->block_tables) | reinterpret_cast<uintptr_t>(a->seq_lens) |
                           reinterpret_cast<uintptr_t>(a->status);
  if ((wide & 15u) || (narrow & 3u)) return SQA_ERR_INVALID_ARGUMENT;

  AppendParams p;
  p.new_k = static_cast<const uint4*>(a->new_keys);
  p.new_v = static_cast<const uint4*>(a->new_values);
  p.k_cache = static_cast<uint4*>(a->key_cache);
  p.v_cache = static_cast<uint4*>(a->value_cache);
  p.block_tables = a->block_tables;
  p.seq_lens = a->seq_lens;
  p.status = a->status;
  const bool fp8 = a->kv_dtype == SQA_KV_FP8_E4M3;
  p.row16 = fp8 ? 8 : 16;
  p.items = (long long)a->batch * a->q_len * a->num_kv_heads * p.row16;
  p.q_len = a->q_len;
  p.hkv = a->num_kv_heads;
  p.num_pages = a->num_pages;
  p.max_pages = a->max_pages;
  p.hnd = a->kv_layout == SQA_KV_HND;
  p.page_stride16 =
      (a->page_stride > 0 ? a->page_stride : (int64_t)kPageSize * a->num_kv_heads * kHeadDim) / (fp8 ? 16 : 8);

  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                cudaSuccess)
    return SQA_ERR_CUDA;
  long long blocks = (p.items + 255) / 256;
  if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, sqa_cache_append_kernel, p) != cudaSuccess) return SQA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? SQA_OK : SQA_ERR_CUDA;
}
