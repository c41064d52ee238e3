// The decode path's entry points as PyTorch dispatcher operators, torch.ops.mcb200.*: the same
// libmcb200 C ABI (include/mcb200.h) called from C++, so an eager caller pays the dispatcher's
// cost per call instead of building ctypes argument structs, and torch.compile sees the ops
// (their shape functions are registered in modelcore_b200/torch_ops.py).
//
//   kv_append_rope  rope + QK-norm + x scale of q (and k) and the insert of k, v at each row's
//                   position (modelcore/components/attention.py:147-160 and the insert of
//                   kernels/flash_attn.py:337-346); returns the processed q
//   kv_broadcast    positions [0, n_pos) of one cache row copied into a range of rows, every
//                   slot (KVCache.prefill / prefill_row, modelcore/cache.py:75-119)
//   decode_attn     the attention of flash_attn_with_kvcache over one cache slot
//                   (kernels/flash_attn.py:348-366)
//   append_attn     kv_append_rope then decode_attn, in one launch where the plan allows it
//   kv_advance      cache_seqlens += n (KVCache.advance, modelcore/cache.py:62-73)
//   linear          mcb_linear's plain, residual, gated and norm-out projections (the decode
//                   step's, modelcore/components/linear.py:14 with block.py:57-59, mlp.py:89-90)
//   add_rms_norm    the residual add and the next RMSNorm (block.py:57-59, norm.py:43-44)
//
// Every op runs on the current CUDA stream of its tensors' device, checks dtypes, devices and
// dimensions here (TORCH_CHECK: a RuntimeError in Python) and leaves sizes, strides and
// alignment to the library's own checks, whose message it raises.  The partials workspace and
// the arrival counters of decode_attn come from the caching allocator; the counters, zero on
// allocation and left zero by every completed call, are kept per device and grown on demand
// (earlier arrays stay alive: a captured CUDA graph may hold them).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <limits>
#include <mutex>
#include <vector>

#include "../../include/mcb200.h"

namespace {

void check_status(int rc, const char* what) {
  if (rc == MCB_OK) return;
  char msg[512];
  mcb_last_error(msg, sizeof(msg));
  TORCH_CHECK(false, what, ": ", msg, " (mcb_status ", rc, ")");
}

void need(const at::Tensor& t, const char* name, int64_t dim, at::ScalarType dtype) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == dim, name, " must have ", dim, " dimensions, got ", t.dim());
  TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, ", got ", t.scalar_type());
}

void same_device(const at::Tensor& a, const at::Tensor& b, const char* name) {
  TORCH_CHECK(a.device() == b.device(), name, " must be on ", a.device(), ", got ", b.device());
}

void bthd_strides(const at::Tensor& t, int64_t (&s)[3]) {
  TORCH_CHECK(t.stride(3) == 1, "the head dimension must be contiguous");
  s[0] = t.stride(0);
  s[1] = t.stride(1);
  s[2] = t.stride(2);
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// the fp32 epsilon torch's F.rms_norm uses for a bf16 input when none is given (opmath epsilon)
float norm_eps(std::optional<double> eps) {
  return eps.has_value() ? static_cast<float>(*eps) : std::numeric_limits<float>::epsilon();
}

void check_slot(const at::Tensor& c, const char* name, const at::Tensor& q, int64_t Hkv) {
  need(c, name, 4, at::kBFloat16);
  same_device(q, c, name);
  TORCH_CHECK(c.is_contiguous(), name, " must be a contiguous (B, Tmax, Hkv, D) slot");
  TORCH_CHECK(c.size(0) == q.size(0) && c.size(3) == q.size(3) && (Hkv < 0 || c.size(2) == Hkv), name,
              " must be (", q.size(0), ", Tmax, ", Hkv, ", ", q.size(3), "), got ", c.sizes());
}

void check_seqlens(const at::Tensor& s, const at::Tensor& q) {
  need(s, "cache_seqlens", 1, at::kInt);
  same_device(q, s, "cache_seqlens");
  TORCH_CHECK(s.is_contiguous() && s.size(0) == q.size(0), "cache_seqlens must be a contiguous (",
              q.size(0), ",) int32 tensor");
}

void check_table(const at::Tensor& t, const char* name, const at::Tensor& q) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "rotary ", name,
              " must be a contiguous bf16 CUDA tensor");
  same_device(q, t, name);
  TORCH_CHECK(t.size(-1) == q.size(3) / 2, "rotary ", name, " must have D/2 = ", q.size(3) / 2, " columns");
}

// Per-device arrival counters (zero-filled, grown on demand, never freed while the process runs).
int32_t* counters_for(const at::Device& dev, size_t count) {
  static std::mutex mu;
  static std::vector<std::vector<at::Tensor>> per_dev(64);
  std::lock_guard<std::mutex> lock(mu);
  const int idx = dev.index();
  TORCH_CHECK(idx >= 0 && idx < 64, "device index ", idx);
  auto& bufs = per_dev[idx];
  if (bufs.empty() || static_cast<size_t>(bufs.back().numel()) < count) {
    const int64_t n = std::max<int64_t>(static_cast<int64_t>(count), 1 << 16);
    bufs.push_back(at::zeros({n}, at::TensorOptions().dtype(at::kInt).device(dev)));
  }
  return bufs.back().data_ptr<int32_t>();
}

mcb_attn_args attn_args(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                        const at::Tensor& cache_seqlens, int64_t window, std::optional<double> softmax_scale,
                        int64_t num_ctas, bool ring, const at::Tensor& out) {
  need(q, "q", 4, at::kBFloat16);
  check_slot(k_cache, "k_cache", q, -1);
  check_slot(v_cache, "v_cache", q, k_cache.size(2));
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes(), "k_cache and v_cache shapes differ");
  check_seqlens(cache_seqlens, q);
  mcb_attn_args a = {};
  a.q = q.data_ptr();
  bthd_strides(q, a.q_stride);
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.cache_seqlens = cache_seqlens.data_ptr<int32_t>();
  a.out = out.data_ptr();
  a.B = static_cast<int32_t>(q.size(0));
  a.T = static_cast<int32_t>(q.size(1));
  a.Hq = static_cast<int32_t>(q.size(2));
  a.Hkv = static_cast<int32_t>(k_cache.size(2));
  a.D = static_cast<int32_t>(q.size(3));
  a.Tmax = static_cast<int32_t>(k_cache.size(1));
  a.window = window < 0 ? -1 : static_cast<int32_t>(window);
  a.softmax_scale = softmax_scale.has_value() ? static_cast<float>(*softmax_scale)
                                              : static_cast<float>(1.0 / std::sqrt(static_cast<double>(q.size(3))));
  a.num_ctas = static_cast<int32_t>(num_ctas);
  a.ring = ring ? 1 : 0;
  return a;
}

// Workspace and counters for the planned launch, then the launch.
void run_attn(mcb_attn_args* a, const at::Tensor& q) {
  at::Tensor ws;
  const size_t need_ws = mcb_decode_attn_workspace_size(a);
  if (need_ws > 0) {
    ws = at::empty({static_cast<int64_t>(need_ws)}, q.options().dtype(at::kByte));
    a->workspace = ws.data_ptr();
    a->workspace_bytes = need_ws;
  }
  const size_t ncount = mcb_decode_attn_counter_count(a);
  if (ncount > 0) {
    a->counters = counters_for(q.device(), ncount);
    a->counter_count = ncount;
  }
  check_status(mcb_decode_attn(a, stream_of(q)), "mcb200::decode_attn");
}

at::Tensor kv_append_rope(const at::Tensor& q, const std::optional<at::Tensor>& k,
                          const std::optional<at::Tensor>& v, const std::optional<at::Tensor>& k_cache,
                          const std::optional<at::Tensor>& v_cache, const at::Tensor& cache_seqlens,
                          const at::Tensor& cos, const at::Tensor& sin, std::optional<double> eps, double scale,
                          bool ring) {
  need(q, "q", 4, at::kBFloat16);
  c10::cuda::CUDAGuard guard(q.device());
  check_seqlens(cache_seqlens, q);
  check_table(cos, "cos", q);
  check_table(sin, "sin", q);
  const bool write_kv = k.has_value();
  TORCH_CHECK(write_kv == v.has_value() && write_kv == k_cache.has_value() && write_kv == v_cache.has_value(),
              "k, v, k_cache and v_cache come together (all or none)");
  at::Tensor q_out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  mcb_append_args a = {};
  a.q = q.data_ptr();
  bthd_strides(q, a.q_stride);
  a.q_out = q_out.data_ptr();
  a.B = static_cast<int32_t>(q.size(0));
  a.T = static_cast<int32_t>(q.size(1));
  a.Hq = static_cast<int32_t>(q.size(2));
  a.D = static_cast<int32_t>(q.size(3));
  a.flags = MCB_APPEND_ROTATE_Q;
  if (write_kv) {
    need(*k, "k", 4, at::kBFloat16);
    need(*v, "v", 4, at::kBFloat16);
    same_device(q, *k, "k");
    same_device(q, *v, "v");
    TORCH_CHECK(k->sizes() == v->sizes() && k->size(0) == q.size(0) && k->size(1) == q.size(1) &&
                    k->size(3) == q.size(3),
                "k and v must be (B, T, Hkv, D) like q's B, T and D");
    check_slot(*k_cache, "k_cache", q, k->size(2));
    check_slot(*v_cache, "v_cache", q, k->size(2));
    TORCH_CHECK(v_cache->sizes() == k_cache->sizes(), "k_cache and v_cache shapes differ");
    a.k = k->data_ptr();
    a.v = v->data_ptr();
    bthd_strides(*k, a.k_stride);
    bthd_strides(*v, a.v_stride);
    a.k_cache = k_cache->data_ptr();
    a.v_cache = v_cache->data_ptr();
    a.Hkv = static_cast<int32_t>(k->size(2));
    a.Tmax = static_cast<int32_t>(k_cache->size(1));
    a.flags |= MCB_APPEND_ROTATE_K | MCB_APPEND_WRITE_KV;
  }
  a.cache_seqlens = cache_seqlens.data_ptr<int32_t>();
  a.cos = cos.data_ptr();
  a.sin = sin.data_ptr();
  a.rot_len = static_cast<int32_t>(cos.numel() / (q.size(3) / 2));
  a.eps = norm_eps(eps);
  a.scale = static_cast<float>(scale);
  a.ring = ring ? 1 : 0;
  check_status(mcb_kv_append_rope(&a, stream_of(q)), "mcb200::kv_append_rope");
  return q_out;
}

void kv_broadcast(const at::Tensor& src_k, const at::Tensor& src_v, const at::Tensor& dst_k,
                  const at::Tensor& dst_v, int64_t src_row, int64_t dst_row_begin, int64_t dst_row_count,
                  int64_t n_pos, const std::optional<at::Tensor>& dst_seqlens) {
  for (const at::Tensor* t : {&src_k, &src_v, &dst_k, &dst_v}) {
    need(*t, "cache", 5, at::kBFloat16);
    same_device(dst_k, *t, "cache");
    TORCH_CHECK(t->is_contiguous(), "caches must be contiguous (n_slots, B, Tmax, Hkv, D) tensors");
  }
  TORCH_CHECK(dst_k.sizes() == dst_v.sizes() && src_k.sizes() == src_v.sizes(), "k and v caches must have equal shapes");
  TORCH_CHECK(dst_k.size(0) == src_k.size(0) && dst_k.size(3) == src_k.size(3) && dst_k.size(4) == src_k.size(4),
              "cache layouts differ: dst ", dst_k.sizes(), " vs src ", src_k.sizes());
  c10::cuda::CUDAGuard guard(dst_k.device());
  mcb_copy_args a = {};
  a.dst_k = dst_k.data_ptr();
  a.dst_v = dst_v.data_ptr();
  a.src_k = src_k.data_ptr();
  a.src_v = src_v.data_ptr();
  a.n_slots = static_cast<int32_t>(dst_k.size(0));
  a.src_batch = static_cast<int32_t>(src_k.size(1));
  a.src_row = static_cast<int32_t>(src_row);
  a.src_tmax = static_cast<int32_t>(src_k.size(2));
  a.dst_batch = static_cast<int32_t>(dst_k.size(1));
  a.dst_row_begin = static_cast<int32_t>(dst_row_begin);
  a.dst_row_count = static_cast<int32_t>(dst_row_count);
  a.dst_tmax = static_cast<int32_t>(dst_k.size(2));
  a.n_pos = static_cast<int32_t>(n_pos);
  a.row_elems = static_cast<int32_t>(dst_k.size(3) * dst_k.size(4));
  if (dst_seqlens.has_value()) {
    need(*dst_seqlens, "dst_seqlens", 1, at::kInt);
    same_device(dst_k, *dst_seqlens, "dst_seqlens");
    TORCH_CHECK(dst_seqlens->is_contiguous() && dst_seqlens->size(0) == dst_k.size(1),
                "dst_seqlens must be a contiguous (", dst_k.size(1), ",) int32 tensor");
    a.dst_seqlens = dst_seqlens->data_ptr<int32_t>();
  }
  check_status(mcb_kv_copy_rows(&a, stream_of(dst_k)), "mcb200::kv_broadcast");
}

at::Tensor decode_attn(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                       const at::Tensor& cache_seqlens, int64_t window, std::optional<double> softmax_scale,
                       int64_t num_ctas, bool ring) {
  need(q, "q", 4, at::kBFloat16);
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  mcb_attn_args a = attn_args(q, k_cache, v_cache, cache_seqlens, window, softmax_scale, num_ctas, ring, out);
  run_attn(&a, q);
  return out;
}

at::Tensor append_attn(const at::Tensor& q, const std::optional<at::Tensor>& k, const std::optional<at::Tensor>& v,
                       const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& cache_seqlens,
                       const at::Tensor& cos, const at::Tensor& sin, std::optional<double> eps, double scale,
                       int64_t window, bool ring) {
  need(q, "q", 4, at::kBFloat16);
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(k.has_value() == v.has_value(), "k and v come together");
  check_table(cos, "cos", q);
  check_table(sin, "sin", q);
  at::Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  mcb_attn_args a = attn_args(q, k_cache, v_cache, cache_seqlens, window, std::nullopt, 0, ring, out);
  if (!mcb_decode_attn_fusable(&a)) {  // the two launches, the same bits
    at::Tensor qa = k.has_value()
                        ? kv_append_rope(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin, eps, scale, ring)
                        : kv_append_rope(q, std::nullopt, std::nullopt, std::nullopt, std::nullopt, cache_seqlens,
                                         cos, sin, eps, scale, ring);
    mcb_attn_args b = attn_args(qa, k_cache, v_cache, cache_seqlens, window, std::nullopt, 0, ring, out);
    run_attn(&b, qa);
    return out;
  }
  a.fuse_append = 1;
  if (k.has_value()) {
    need(*k, "k", 4, at::kBFloat16);
    need(*v, "v", 4, at::kBFloat16);
    same_device(q, *k, "k");
    same_device(q, *v, "v");
    TORCH_CHECK(k->sizes() == v->sizes() && k->size(0) == q.size(0) && k->size(1) == 1 &&
                    k->size(2) == k_cache.size(2) && k->size(3) == q.size(3),
                "k and v must be (B, 1, Hkv, D) like the slot");
    a.k_new = k->data_ptr();
    a.v_new = v->data_ptr();
    bthd_strides(*k, a.k_new_stride);
    bthd_strides(*v, a.v_new_stride);
  }
  a.rot_cos = cos.data_ptr();
  a.rot_sin = sin.data_ptr();
  a.rot_len = static_cast<int32_t>(cos.numel() / (q.size(3) / 2));
  a.rotate_k = 1;
  a.norm_eps = norm_eps(eps);
  a.qk_scale = static_cast<float>(scale);
  run_attn(&a, q);
  return out;
}

void kv_advance(const at::Tensor& cache_seqlens, int64_t n) {
  need(cache_seqlens, "cache_seqlens", 1, at::kInt);
  TORCH_CHECK(cache_seqlens.is_contiguous(), "cache_seqlens must be contiguous");
  c10::cuda::CUDAGuard guard(cache_seqlens.device());
  check_status(mcb_kv_advance(cache_seqlens.data_ptr<int32_t>(), static_cast<int32_t>(cache_seqlens.numel()),
                              static_cast<int32_t>(n), stream_of(cache_seqlens)),
               "mcb200::kv_advance");
}

int64_t row_stride(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be a 2-D tensor with unit column stride");
  return t.stride(0);
}

// mcb_linear's plain, residual, gated and norm-out modes (the decode step's projections)
void linear(const at::Tensor& x, const at::Tensor& weight, const at::Tensor& out, const std::optional<at::Tensor>& res,
            const std::optional<at::Tensor>& h_out, std::optional<double> eps, bool gated, bool pdl) {
  for (const at::Tensor* t : {&x, &weight, &out}) {
    need(*t, "x, weight and out", 2, at::kBFloat16);
    same_device(x, *t, "weight and out");
  }
  c10::cuda::CUDAGuard guard(x.device());
  mcb_linear_args a = {};
  a.x = x.data_ptr();
  a.w = weight.data_ptr();
  a.y = out.data_ptr();
  a.x_stride = row_stride(x, "x");
  a.w_stride = row_stride(weight, "weight");
  a.y_stride = row_stride(out, "out");
  a.R = static_cast<int32_t>(x.size(0));
  a.K = static_cast<int32_t>(x.size(1));
  a.N = static_cast<int32_t>(gated ? weight.size(0) / 2 : weight.size(0));
  TORCH_CHECK(weight.size(1) == x.size(1), "weight must be (N, ", x.size(1), "), got ", weight.sizes());
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == a.N, "out must be (", x.size(0), ", ", a.N, ")");
  if (res.has_value()) {
    need(*res, "res", 2, at::kBFloat16);
    same_device(x, *res, "res");
    TORCH_CHECK(res->sizes() == out.sizes(), "res must be shaped like out");
    a.res = res->data_ptr();
    a.res_stride = row_stride(*res, "res");
  }
  a.flags = gated ? MCB_LINEAR_GATED : 0;
  if (h_out.has_value()) {
    need(*h_out, "h_out", 2, at::kBFloat16);
    same_device(x, *h_out, "h_out");
    TORCH_CHECK(h_out->sizes() == out.sizes(), "h_out must be shaped like out");
    a.h_out = h_out->data_ptr();
    a.h_out_stride = row_stride(*h_out, "h_out");
    a.flags |= MCB_LINEAR_NORM_OUT;
  }
  a.eps = norm_eps(eps);
  a.pdl = pdl ? 1 : 0;
  check_status(mcb_linear(&a, stream_of(x)), "mcb200::linear");
}

// x_out = x + delta (when delta is given; x_out may be x), h_out = rms_norm(that)
void add_rms_norm(const at::Tensor& x, const std::optional<at::Tensor>& delta, const std::optional<at::Tensor>& x_out,
                  const at::Tensor& h_out, std::optional<double> eps) {
  need(x, "x", 2, at::kBFloat16);
  need(h_out, "h_out", 2, at::kBFloat16);
  same_device(x, h_out, "h_out");
  TORCH_CHECK(h_out.sizes() == x.sizes(), "h_out must be shaped like x");
  c10::cuda::CUDAGuard guard(x.device());
  mcb_add_norm_args a = {};
  a.x = x.data_ptr();
  a.x_stride = row_stride(x, "x");
  a.h_out = h_out.data_ptr();
  a.h_stride = row_stride(h_out, "h_out");
  a.rows = static_cast<int32_t>(x.size(0));
  a.C = static_cast<int32_t>(x.size(1));
  if (delta.has_value()) {
    TORCH_CHECK(x_out.has_value(), "x_out is needed with delta");
    for (const at::Tensor* t : {&*delta, &*x_out}) {
      need(*t, "delta and x_out", 2, at::kBFloat16);
      same_device(x, *t, "delta and x_out");
      TORCH_CHECK(t->sizes() == x.sizes(), "delta and x_out must be shaped like x");
    }
    a.delta = delta->data_ptr();
    a.delta_stride = row_stride(*delta, "delta");
    a.x_out = x_out->data_ptr();
    a.x_out_stride = row_stride(*x_out, "x_out");
  }
  a.eps = norm_eps(eps);
  check_status(mcb_add_rms_norm(&a, stream_of(x)), "mcb200::add_rms_norm");
}

}  // namespace

TORCH_LIBRARY(mcb200, m) {
  m.def(
      "kv_append_rope(Tensor q, Tensor? k, Tensor? v, Tensor(a!)? k_cache, Tensor(b!)? v_cache, "
      "Tensor cache_seqlens, Tensor cos, Tensor sin, float? eps=None, float scale=1.2, bool ring=False) -> Tensor");
  m.def(
      "kv_broadcast(Tensor src_k, Tensor src_v, Tensor(a!) dst_k, Tensor(b!) dst_v, int src_row, "
      "int dst_row_begin, int dst_row_count, int n_pos, Tensor(c!)? dst_seqlens=None) -> ()");
  m.def(
      "decode_attn(Tensor q, Tensor k_cache, Tensor v_cache, Tensor cache_seqlens, int window=-1, "
      "float? softmax_scale=None, int num_ctas=0, bool ring=False) -> Tensor");
  m.def(
      "append_attn(Tensor q, Tensor? k, Tensor? v, Tensor(a!) k_cache, Tensor(b!) v_cache, "
      "Tensor cache_seqlens, Tensor cos, Tensor sin, float? eps=None, float scale=1.2, int window=-1, "
      "bool ring=False) -> Tensor");
  m.def("kv_advance(Tensor(a!) cache_seqlens, int n) -> ()");
  m.def(
      "linear(Tensor x, Tensor weight, Tensor(a!) out, Tensor? res=None, Tensor(b!)? h_out=None, "
      "float? eps=None, bool gated=False, bool pdl=False) -> ()");
  m.def("add_rms_norm(Tensor x, Tensor? delta, Tensor(a!)? x_out, Tensor(b!) h_out, float? eps=None) -> ()");
}

TORCH_LIBRARY_IMPL(mcb200, CUDA, m) {
  m.impl("kv_append_rope", &kv_append_rope);
  m.impl("kv_broadcast", &kv_broadcast);
  m.impl("decode_attn", &decode_attn);
  m.impl("append_attn", &append_attn);
  m.impl("kv_advance", &kv_advance);
  m.impl("linear", &linear);
  m.impl("add_rms_norm", &add_rms_norm);
}
