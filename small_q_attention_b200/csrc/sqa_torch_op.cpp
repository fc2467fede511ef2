// sqa_torch_op.cpp -- the operator as a torch extension over the C ABI.
//
// Two doors into the same code:
// * TORCH_LIBRARY(sqa_b200): torch.ops.sqa_b200.small_q_attention /
//   small_q_attention_partial, with CUDA and Meta kernels, so torch.compile and
//   fake-tensor tracing see a real operator instead of an opaque Python call;
// * a pybind11 module (_sqa_torch.forward / forward_partial) that the Python
//   entry small_q_attention() calls directly: the contract checks, argument
//   packing, workspace lookup and both launches run here in C++, on torch's
//   current stream, in a few microseconds of host time.
//
// The checks and their exception types restate the upstream Python wrapper's
// contract (src/small_q_attention/cuda.py:197-211: ValueError for a tensor
// that is not on CUDA, not contiguous, of the wrong dtype or outside the shape
// contract); the launch is sqa_forward (include/small_q_attention.h), which
// replaces small_q_attention_v3 (csrc/small_q_attention_ext.cu:1132-1210).
// Nothing here computes: every kernel lives in libsqa_b200.so.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/small_q_attention.h"

namespace {

constexpr int64_t kHeadDim = SQA_HEAD_DIM;
constexpr int64_t kPage = SQA_PAGE_SIZE;
constexpr int64_t kGroup = SQA_GQA_GROUP;
constexpr int64_t kMaxQ = SQA_MAX_Q_LEN;

// Elements from one page to the next (0 = contiguous caches); the caches may be
// views of a bigger pool: packed within a page, one 16-byte aligned page
// stride shared by K and V.
int64_t cache_page_stride(const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK_VALUE(k.dim() == 4, "key_cache must be 4-D");
  if (k.is_contiguous() && v.is_contiguous()) return 0;
  const auto st = k.strides();
  const int64_t inner = k.size(1) * k.size(2) * k.size(3);
  const int64_t align = 16 / k.element_size();
  const bool packed = st[1] == k.size(2) * k.size(3) && st[2] == k.size(3) && st[3] == 1;
  TORCH_CHECK_VALUE(v.strides() == st && packed && st[0] >= inner && st[0] % align == 0,
                    "key_cache / value_cache must be packed within a page, with one page stride "
                    "(16-byte aligned) shared by K and V");
  return st[0];
}

void check_inputs(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& bt,
                  const at::Tensor& sl, int64_t page_size, const c10::optional<at::Tensor>& mask_lens,
                  int64_t kv_layout) {
  const at::Tensor* all[6] = {&q, &k, &v, &bt, &sl, mask_lens.has_value() ? &*mask_lens : nullptr};
  const int n = mask_lens.has_value() ? 6 : 5;
  for (int i = 0; i < n; ++i) TORCH_CHECK_VALUE(all[i]->defined(), "all inputs must be CUDA tensors");
  TORCH_CHECK_VALUE(q.is_cuda(), "all inputs must be CUDA tensors");
  const auto dev = q.device();
  for (int i = 0; i < n; ++i) {
    TORCH_CHECK_VALUE(all[i]->device() == dev, "all inputs must be CUDA tensors on the same device");
    if (i != 1 && i != 2) TORCH_CHECK_VALUE(all[i]->is_contiguous(), "all inputs must be contiguous");
  }
  cache_page_stride(k, v);
  const auto qd = q.scalar_type(), kd = k.scalar_type();
  TORCH_CHECK_VALUE((qd == at::kHalf || qd == at::kBFloat16) && v.scalar_type() == kd &&
                        (kd == qd || kd == at::kFloat8_e4m3fn),
                    "the kernel requires FP16 (or BF16) Q/K/V of one type, or FP16/BF16 Q with FP8-E4M3 K/V");
  for (int i = 3; i < n; ++i)
    TORCH_CHECK_VALUE(all[i]->scalar_type() == at::kInt, "block_tables, seq_lens and mask_lens must be int32");
  TORCH_CHECK_VALUE(q.dim() == 4 && k.dim() == 4, "query and key_cache must be 4-D");
  TORCH_CHECK_VALUE(v.sizes() == k.sizes(), "value_cache shape mismatch");
  TORCH_CHECK_VALUE(kv_layout == SQA_KV_NHD || kv_layout == SQA_KV_HND,
                    "kv_layout must be \"NHD\" ([pages, 16, Hkv, 128]) or \"HND\" ([pages, Hkv, 16, 128])");
  const int64_t batch = q.size(0), q_len = q.size(1), hq = q.size(2), head_dim = q.size(3);
  const bool hnd = kv_layout == SQA_KV_HND;
  const int64_t hkv = hnd ? k.size(1) : k.size(2);
  const int64_t cache_page = hnd ? k.size(2) : k.size(1);
  TORCH_CHECK_VALUE(q_len >= 1 && q_len <= kMaxQ, "q_len must be in [1, ", kMaxQ, "]");
  TORCH_CHECK_VALUE(head_dim == kHeadDim && k.size(3) == kHeadDim, "the kernel supports head_dim 128");
  TORCH_CHECK_VALUE(hkv > 0 && hq % hkv == 0 && hq / hkv == kGroup,
                    "the kernel requires a GQA group size of exactly 4 (Hq/Hkv = 32/8)");
  TORCH_CHECK_VALUE(page_size == cache_page && cache_page == kPage,
                    "page_size must be 16 and match the cache's page dimension");
  TORCH_CHECK_VALUE(bt.dim() == 2 && bt.size(0) == batch && sl.numel() == batch,
                    "invalid metadata: block_tables must be [batch, max_pages], seq_lens [batch]");
  TORCH_CHECK_VALUE(!mask_lens.has_value() || mask_lens->numel() == batch,
                    "mask_lens must have one entry per sequence");
  TORCH_CHECK_VALUE(k.size(0) > 0 && bt.size(1) > 0, "empty KV cache is not supported");
}

sqa_args fill_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& bt,
                   const at::Tensor& sl, const c10::optional<at::Tensor>& mask_lens, int64_t max_seq_len,
                   int64_t num_ctas, int64_t min_pages_per_cta, int64_t kernel, int64_t kv_layout, double sm_scale,
                   double out_scale, int64_t min_seq_len = 0, int64_t cluster = 0) {
  sqa_args a = {};
  const bool hnd = kv_layout == SQA_KV_HND;
  a.query = q.data_ptr();
  a.key_cache = k.data_ptr();
  a.value_cache = v.data_ptr();
  a.block_tables = bt.data_ptr<int32_t>();
  a.seq_lens = sl.data_ptr<int32_t>();
  a.mask_lens = mask_lens.has_value() ? mask_lens->data_ptr<int32_t>() : nullptr;
  a.batch = (int32_t)q.size(0);
  a.q_len = (int32_t)q.size(1);
  a.num_q_heads = (int32_t)q.size(2);
  a.num_kv_heads = (int32_t)(hnd ? k.size(1) : k.size(2));
  a.head_dim = (int32_t)q.size(3);
  a.page_size = (int32_t)(hnd ? k.size(2) : k.size(1));
  a.num_pages = (int32_t)k.size(0);
  a.max_pages = (int32_t)bt.size(1);
  a.max_seq_len = (int32_t)max_seq_len;
  a.num_ctas = (int32_t)num_ctas;
  a.min_pages_per_cta = (int32_t)min_pages_per_cta;
  a.kernel = (int32_t)kernel;
  a.dtype = q.scalar_type() == at::kBFloat16 ? SQA_DTYPE_BF16 : SQA_DTYPE_F16;
  a.kv_layout = (int32_t)kv_layout;
  a.sm_scale = (float)sm_scale;
  a.out_scale = (float)out_scale;
  a.page_stride = cache_page_stride(k, v);
  a.kv_dtype = k.scalar_type() == at::kFloat8_e4m3fn ? SQA_KV_FP8_E4M3 : SQA_KV_SAME;
  a.min_seq_len = (int32_t)min_seq_len;
  a.cluster = (int32_t)cluster;
  return a;
}

void check_status(int code, const char* what) {
  if (code == SQA_OK) return;
  const std::string msg = std::string(what) + ": " + sqa_status_string(code) + " (status " + std::to_string(code) + ")";
  TORCH_CHECK_VALUE(code != SQA_ERR_INVALID_ARGUMENT && code != SQA_ERR_UNSUPPORTED, msg);
  TORCH_CHECK(false, msg);
}

// One workspace per (device, stream), grown on demand; the status word of a
// new one starts zeroed.  (A caller's explicit workspace is used as given.)
struct WsEntry {
  int device;
  cudaStream_t stream;
  at::Tensor ws;
};
std::mutex g_ws_mu;
std::vector<WsEntry> g_ws;

std::pair<void*, size_t> workspace_for(const sqa_args& a, const at::Device& dev, cudaStream_t stream,
                                       const c10::optional<at::Tensor>& workspace) {
  if (workspace.has_value()) {
    const at::Tensor& w = *workspace;
    TORCH_CHECK_VALUE(w.device() == dev && w.is_contiguous(),
                      "workspace must be a contiguous tensor on the query's device");
    return {w.data_ptr(), (size_t)w.numel() * w.element_size()};
  }
  int st = SQA_OK;
  const size_t need = sqa_workspace_bytes(&a, dev.index(), &st);
  check_status(st, "sqa_workspace_bytes");
  std::lock_guard<std::mutex> lock(g_ws_mu);
  for (auto& e : g_ws) {
    if (e.device == dev.index() && e.stream == stream) {
      if ((size_t)e.ws.numel() < need) e.ws = at::zeros({(int64_t)std::max<size_t>(need, 1 << 20)},
                                                        at::TensorOptions().dtype(at::kByte).device(dev));
      return {e.ws.data_ptr(), (size_t)e.ws.numel()};
    }
  }
  g_ws.push_back(WsEntry{dev.index(), stream,
                         at::zeros({(int64_t)std::max<size_t>(need, 1 << 20)}, at::TensorOptions().dtype(at::kByte).device(dev))});
  return {g_ws.back().ws.data_ptr(), (size_t)g_ws.back().ws.numel()};
}

// check=True: synchronise and raise what the upstream CPU reference raises
// for bad metadata (reference.py:52-53; index_select on a bad page id).
void raise_device_bits(void* ws, cudaStream_t stream) {
  uint32_t bits = 0;
  const int code = sqa_read_device_status(ws, &bits, 1, stream);
  if (code != SQA_OK && code != SQA_ERR_DEVICE) check_status(code, "sqa_read_device_status");
  TORCH_CHECK_VALUE(!(bits & SQA_DEV_SEQ_TOO_SHORT), "seq_lens must be at least q_len for MTP attention");
  TORCH_CHECK_VALUE(!(bits & SQA_DEV_SEQ_TOO_LONG), "seq_lens exceeds page_size * block_tables.shape[1]");
  TORCH_CHECK_INDEX(!(bits & SQA_DEV_BAD_PAGE), "block_tables holds a page id outside the cache");
  TORCH_CHECK(!(bits & SQA_DEV_TIMEOUT), "a bounded device wait timed out; the output is not valid");
}

void launch(sqa_args& a, const at::Tensor& q, const c10::optional<at::Tensor>& workspace, bool check) {
  const at::Device dev = q.device();
  c10::cuda::OptionalCUDAGuard guard;
  if (c10::cuda::current_device() != dev.index()) guard.set_index(dev.index());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  auto [ws, ws_bytes] = workspace_for(a, dev, stream, workspace);
  const int code = sqa_forward(&a, ws, ws_bytes, stream);
  if (code == SQA_ERR_WORKSPACE_TOO_SMALL && workspace.has_value()) {
    int st = SQA_OK;
    TORCH_CHECK_VALUE(false, "workspace too small: need ", sqa_workspace_bytes(&a, dev.index(), &st), " bytes");
  }
  check_status(code, "sqa_forward");
  if (check) raise_device_bits(ws, stream);
}

at::Tensor forward(const at::Tensor& query, const at::Tensor& key_cache, const at::Tensor& value_cache,
                   const at::Tensor& block_tables, const at::Tensor& seq_lens, int64_t page_size, int64_t max_seq_len,
                   const c10::optional<at::Tensor>& out, const c10::optional<at::Tensor>& workspace, int64_t num_ctas,
                   int64_t min_pages_per_cta, int64_t kernel, bool check, int64_t kv_layout, double sm_scale,
                   double out_scale, int64_t min_seq_len, int64_t cluster) {
  check_inputs(query, key_cache, value_cache, block_tables, seq_lens, page_size, c10::nullopt, kv_layout);
  at::Tensor o;
  if (out.has_value()) {
    o = *out;
    TORCH_CHECK_VALUE(o.sizes() == query.sizes() && o.scalar_type() == query.scalar_type() && o.is_contiguous() &&
                          o.device() == query.device(),
                      "out must be a contiguous tensor shaped and typed like query");
  } else {
    o = at::empty_like(query);
  }
  sqa_args a = fill_args(query, key_cache, value_cache, block_tables, seq_lens, c10::nullopt, max_seq_len, num_ctas,
                         min_pages_per_cta, kernel, kv_layout, sm_scale, out_scale, min_seq_len, cluster);
  a.out = o.data_ptr();
  launch(a, query, workspace, check);
  return o;
}

std::tuple<at::Tensor, at::Tensor> forward_partial(
    const at::Tensor& query, const at::Tensor& key_cache, const at::Tensor& value_cache,
    const at::Tensor& block_tables, const at::Tensor& seq_lens, int64_t page_size,
    const c10::optional<at::Tensor>& mask_lens, int64_t max_seq_len, const c10::optional<at::Tensor>& out,
    const c10::optional<at::Tensor>& out_lse, const c10::optional<at::Tensor>& workspace, int64_t num_ctas,
    int64_t min_pages_per_cta, int64_t kernel, bool check, int64_t kv_layout, double sm_scale, double out_scale,
    int64_t min_seq_len, int64_t cluster) {
  check_inputs(query, key_cache, value_cache, block_tables, seq_lens, page_size, mask_lens, kv_layout);
  const auto f32 = query.options().dtype(at::kFloat);
  at::Tensor o = out.has_value() ? *out : at::empty(query.sizes(), f32);
  at::Tensor l = out_lse.has_value() ? *out_lse : at::empty(query.sizes().slice(0, 3), f32);
  TORCH_CHECK_VALUE(o.scalar_type() == at::kFloat && o.sizes() == query.sizes() && o.is_contiguous() &&
                        o.device() == query.device(),
                    "out must be a contiguous fp32 tensor shaped like query");
  TORCH_CHECK_VALUE(l.scalar_type() == at::kFloat && l.sizes() == query.sizes().slice(0, 3) && l.is_contiguous() &&
                        l.device() == query.device(),
                    "out_lse must be a contiguous fp32 tensor [batch, q_len, Hq]");
  sqa_args a = fill_args(query, key_cache, value_cache, block_tables, seq_lens, mask_lens, max_seq_len, num_ctas,
                         min_pages_per_cta, kernel, kv_layout, sm_scale, out_scale, min_seq_len, cluster);
  a.out_partial = o.data_ptr<float>();
  a.out_lse = l.data_ptr<float>();
  launch(a, query, workspace, check);
  return {o, l};
}

// ---- the registered operators (functional: they allocate their outputs)
at::Tensor op_forward(const at::Tensor& query, const at::Tensor& key_cache, const at::Tensor& value_cache,
                      const at::Tensor& block_tables, const at::Tensor& seq_lens, int64_t page_size,
                      int64_t max_seq_len, int64_t kernel, int64_t kv_layout, double sm_scale, double out_scale) {
  return forward(query, key_cache, value_cache, block_tables, seq_lens, page_size, max_seq_len, c10::nullopt,
                 c10::nullopt, 0, 0, kernel, false, kv_layout, sm_scale, out_scale, 0, 0);
}

std::tuple<at::Tensor, at::Tensor> op_forward_partial(const at::Tensor& query, const at::Tensor& key_cache,
                                                      const at::Tensor& value_cache, const at::Tensor& block_tables,
                                                      const at::Tensor& seq_lens, int64_t page_size,
                                                      const c10::optional<at::Tensor>& mask_lens,
                                                      int64_t max_seq_len, int64_t kernel, int64_t kv_layout,
                                                      double sm_scale, double out_scale) {
  return forward_partial(query, key_cache, value_cache, block_tables, seq_lens, page_size, mask_lens, max_seq_len,
                         c10::nullopt, c10::nullopt, c10::nullopt, 0, 0, kernel, false, kv_layout, sm_scale,
                         out_scale, 0, 0);
}

at::Tensor meta_forward(const at::Tensor& query, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        const at::Tensor&, int64_t, int64_t, int64_t, int64_t, double, double) {
  return at::empty_like(query);
}

std::tuple<at::Tensor, at::Tensor> meta_forward_partial(const at::Tensor& query, const at::Tensor&,
                                                        const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                                        int64_t, const c10::optional<at::Tensor>&, int64_t, int64_t,
                                                        int64_t, double, double) {
  const auto f32 = query.options().dtype(at::kFloat);
  return {at::empty(query.sizes(), f32), at::empty(query.sizes().slice(0, 3), f32)};
}

}  // namespace

TORCH_LIBRARY(sqa_b200, m) {
  m.def(
      "small_q_attention(Tensor query, Tensor key_cache, Tensor value_cache, Tensor block_tables, "
      "Tensor seq_lens, int page_size, int max_seq_len=0, int kernel=0, int kv_layout=0, float sm_scale=0., "
      "float out_scale=1.) -> Tensor");
  m.def(
      "small_q_attention_partial(Tensor query, Tensor key_cache, Tensor value_cache, Tensor block_tables, "
      "Tensor seq_lens, int page_size, Tensor? mask_lens=None, int max_seq_len=0, int kernel=0, int kv_layout=0, "
      "float sm_scale=0., float out_scale=1.) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(sqa_b200, CUDA, m) {
  m.impl("small_q_attention", &op_forward);
  m.impl("small_q_attention_partial", &op_forward_partial);
}

TORCH_LIBRARY_IMPL(sqa_b200, Meta, m) {
  m.impl("small_q_attention", &meta_forward);
  m.impl("small_q_attention_partial", &meta_forward_partial);
}

PYBIND11_MODULE(_sqa_torch, m) {
  m.doc() = "small-q paged MTP attention (B200): direct entry over the C ABI";
  m.def("forward", &forward, "causal paged MTP attention (see small_q_attention_b200.small_q_attention)");
  m.def("forward_partial", &forward_partial, "shard form: normalised fp32 O and natural-log LSE");
  m.def("abi_version", &sqa_abi_version);
}
