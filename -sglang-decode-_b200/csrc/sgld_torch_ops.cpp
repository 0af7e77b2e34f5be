// PyTorch operator library over the C ABI (include/sgld_b200.h): registers
//   torch.ops.sglang_decode.plan_build, .decode and .merge
// so the decode path is visible to torch's operator registry (schemas with mutation
// annotations, Meta kernels for tracing) while every launch still goes through the
// torch-free C entry points of libsgld_sm100.so.  Argument checks, strides, pointers and
// the current CUDA stream are read here, in C++, so a decode step costs Python one
// operator call per launch group.
//
// The ops replace the reference's Triton launches: plan_build <- planning/builder.py:6-28,
// decode <- runtime/engine.py:62-73, merge <- kernels/merge.py:7-30.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>
#include <ATen/ATen.h>

#include <cstring>
#include <string>

#include "sgld_b200.h"

namespace {

void check_status(int rc, const char* what) {
  if (rc == SGLD_OK) return;
  const std::string msg = std::string(what) + ": " + sgld_last_error();
  if (rc == SGLD_ERR_INVALID_ARGUMENT || rc == SGLD_ERR_UNSUPPORTED) TORCH_CHECK_VALUE(false, msg);
  TORCH_CHECK(false, msg);
}

int32_t dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kHalf: return SGLD_DTYPE_F16;
    case at::kBFloat16: return SGLD_DTYPE_BF16;
    case at::kFloat8_e4m3fn: return SGLD_DTYPE_E4M3;
    default: TORCH_CHECK_VALUE(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

sgld_plan_geometry geometry_of(at::IntArrayRef g) {
  TORCH_CHECK_VALUE(g.size() == 5, "geometry is (batch_capacity, max_splits, max_context, groups, workers)");
  return sgld_plan_geometry{static_cast<int32_t>(g[0]), static_cast<int32_t>(g[1]), static_cast<int32_t>(g[2]),
                            static_cast<int32_t>(g[3]), static_cast<int32_t>(g[4])};
}

// The plan is one contiguous int32 storage, laid out as sgld_plan_buffers_in_storage says.
sgld_plan_buffers plan_of(const at::Tensor& storage, const sgld_plan_geometry& g) {
  TORCH_CHECK_VALUE(storage.scalar_type() == at::kInt && storage.is_cuda() && storage.is_contiguous(),
                    "the plan storage must be a contiguous int32 CUDA tensor");
  const size_t words = sgld_plan_storage_words(&g);
  TORCH_CHECK_VALUE(words > 0 && static_cast<size_t>(storage.numel()) >= words, "the plan storage holds ",
                    storage.numel(), " int32 words; the geometry needs ", words);
  sgld_plan_buffers b;
  check_status(sgld_plan_buffers_in_storage(storage.data_ptr<int32_t>(), &g, &b), "sgld_plan_buffers_in_storage");
  return b;
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

bool finite_positive(double x) { return x > 0.0 && x <= 3.0e38; }

void plan_build(const at::Tensor& plan, at::IntArrayRef geometry, int64_t force_mode,
                const std::optional<at::Tensor>& rules, int64_t n_rules, const std::optional<at::Tensor>& counters) {
  const c10::cuda::CUDAGuard guard(plan.device());
  const sgld_plan_geometry g = geometry_of(geometry);
  const sgld_plan_buffers p = plan_of(plan, g);
  const int32_t* r = rules.has_value() && n_rules > 0 ? rules->data_ptr<int32_t>() : nullptr;
  int32_t* c = counters.has_value() ? counters->data_ptr<int32_t>() : nullptr;
  const int32_t nc = counters.has_value() ? static_cast<int32_t>(counters->numel()) : 0;
  check_status(sgld_plan_build(&p, &g, static_cast<int32_t>(force_mode), r, static_cast<int32_t>(n_rules), c, nc,
                               stream_of(plan)),
               "sgld_plan_build");
}

// The engine's argument checks: the reference's runtime/engine.py:35-61, plus the additions
// (fewer Q rows than the capacity, fp8 K/V, logit cap, the fused KV-cache write).  Query
// heads and head_dim come from `out` ([capacity, query_heads, head_dim], the engine's output
// buffer), kv_heads from the geometry.  Every failure raises ValueError in Python.
void check_decode_call(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pages,
                       const std::optional<at::Tensor>& indptr, const at::Tensor& out, const sgld_plan_geometry& g,
                       int64_t page_size, double logit_cap, double k_scale, double v_scale,
                       const std::optional<at::Tensor>& k_new, const std::optional<at::Tensor>& v_new,
                       const std::optional<at::Tensor>& new_loc) {
  const bool kv_fp8 = k.scalar_type() == at::kFloat8_e4m3fn;
  const bool q16 = q.scalar_type() == at::kHalf || q.scalar_type() == at::kBFloat16;
  TORCH_CHECK_VALUE(q16 && v.scalar_type() == k.scalar_type() && (k.scalar_type() == q.scalar_type() || kv_fp8),
                    "BF16/FP16 Q/K/V of identical dtype are required (or fp8 e4m3 K/V)");
  TORCH_CHECK_VALUE(out.dim() == 3 && out.size(0) == g.batch_capacity, "out must be [capacity, query_heads, head_dim]");
  const int64_t hq = out.size(1), d = out.size(2), hkv = g.groups;
  TORCH_CHECK_VALUE(!kv_fp8 || d == 128, "fp8 K/V are supported for head_dim 128");
  TORCH_CHECK_VALUE(q.dim() == 3 && q.size(1) == hq && q.size(2) == d && q.size(0) >= 1 &&
                        q.size(0) <= g.batch_capacity,
                    "Q must be [rows <= capacity, query_heads, head_dim]");
  TORCH_CHECK_VALUE(out.scalar_type() == q.scalar_type(), "Q dtype differs from the engine's output dtype");
  for (const at::Tensor* t : {&q, &k, &v, &pages})
    TORCH_CHECK_VALUE(t->device() == out.device(), "all tensors must live on the engine's device");
  TORCH_CHECK_VALUE(pages.scalar_type() == at::kInt, "page table / kv_indices must be int32");
  if (!indptr.has_value()) {
    TORCH_CHECK_VALUE(k.dim() == 4 && v.dim() == 4 && k.sizes() == v.sizes(),
                      "paged KV must have matching [page,token,head,dim] shapes");
    TORCH_CHECK_VALUE(k.size(1) == page_size && k.size(2) == hkv && k.size(3) == d,
                      "KV geometry differs from the capture configuration");
    const int64_t max_pages = (g.max_context + page_size - 1) / page_size;
    TORCH_CHECK_VALUE(pages.dim() == 2 && pages.size(0) == g.batch_capacity && pages.size(1) == max_pages,
                      "page table capacity mismatch");
  } else {
    TORCH_CHECK_VALUE(k.dim() == 3 && v.sizes() == k.sizes() && k.size(1) == hkv && k.size(2) == d,
                      "CSR KV must be [token,head,dim]");
    TORCH_CHECK_VALUE(page_size == 1 && pages.dim() == 1, "CSR integration uses one-token physical pages");
    TORCH_CHECK_VALUE(indptr->scalar_type() == at::kInt && indptr->dim() == 1 && indptr->device() == out.device(),
                      "kv_indptr must be a 1-D int32 tensor");
  }
  TORCH_CHECK_VALUE(finite_positive(k_scale), "k_scale must be a finite value > 0");
  TORCH_CHECK_VALUE(finite_positive(v_scale), "v_scale must be a finite value > 0");
  TORCH_CHECK_VALUE(logit_cap >= 0.0 && logit_cap <= 3.0e38, "logit_cap must be a finite value >= 0 (0 disables it)");
  if (!new_loc.has_value()) {
    TORCH_CHECK_VALUE(!k_new.has_value() && !v_new.has_value(), "k_new / v_new need new_loc");
    return;
  }
  const int64_t rows = q.size(0);
  for (const std::optional<at::Tensor>* t : {&k_new, &v_new})
    TORCH_CHECK_VALUE(t->has_value() && (*t)->scalar_type() == q.scalar_type() && (*t)->device() == out.device() &&
                          (*t)->dim() == 3 && (*t)->size(0) == rows && (*t)->size(1) == hkv && (*t)->size(2) == d,
                      "k_new / v_new must be [q rows, kv_heads, head_dim] in Q's dtype");
  const at::Tensor& loc = *new_loc;
  TORCH_CHECK_VALUE((loc.scalar_type() == at::kLong || loc.scalar_type() == at::kInt) &&
                        loc.device() == out.device() && loc.dim() == 1 && loc.size(0) == rows && loc.stride(0) == 1,
                    "new_loc must be a contiguous 1-D int64/int32 tensor, one slot per Q row");
}

// K/V: paged [pages, page_size, Hkv, D] or CSR [tokens, Hkv, D] (indptr given).
void decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pages,
            const std::optional<at::Tensor>& indptr, at::Tensor out, at::Tensor partial, at::Tensor lse,
            at::Tensor counter, at::Tensor status, const at::Tensor& plan, at::IntArrayRef geometry, int64_t page_size,
            double scale, double logit_cap, double k_scale, double v_scale, const std::optional<at::Tensor>& k_new,
            const std::optional<at::Tensor>& v_new, const std::optional<at::Tensor>& new_loc) {
  const c10::cuda::CUDAGuard guard(out.device());
  const sgld_plan_geometry g = geometry_of(geometry);
  check_decode_call(q, k, v, pages, indptr, out, g, page_size, logit_cap, k_scale, v_scale, k_new, v_new, new_loc);
  const sgld_plan_buffers p = plan_of(plan, g);
  sgld_decode_args a;
  std::memset(&a, 0, sizeof(a));
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.out = out.data_ptr();
  a.pages = pages.data_ptr<int32_t>();
  for (int i = 0; i < 3; ++i) a.q_stride[i] = q.stride(i);
  if (indptr.has_value()) {
    a.indptr = indptr->data_ptr<int32_t>();
    const int64_t ks[4] = {k.stride(0), 0, k.stride(1), k.stride(2)};
    const int64_t vs[4] = {v.stride(0), 0, v.stride(1), v.stride(2)};
    std::memcpy(a.k_stride, ks, sizeof(ks));
    std::memcpy(a.v_stride, vs, sizeof(vs));
  } else {
    for (int i = 0; i < 4; ++i) a.k_stride[i] = k.stride(i), a.v_stride[i] = v.stride(i);
    a.pt_stride[0] = pages.stride(0);
    a.pt_stride[1] = pages.stride(1);
  }
  a.kv_extent = k.size(0) == v.size(0) ? k.size(0) : 0;
  a.dtype = dtype_code(q);
  a.kv_dtype = dtype_code(k);
  a.query_heads = static_cast<int32_t>(out.size(1));
  a.kv_heads = g.groups;
  a.head_dim = static_cast<int32_t>(out.size(2));
  a.page_size = static_cast<int32_t>(page_size);
  a.scale = static_cast<float>(scale);
  a.logit_cap = static_cast<float>(logit_cap);
  a.k_scale = static_cast<float>(k_scale);
  a.v_scale = static_cast<float>(v_scale);
  a.q_rows = static_cast<int32_t>(q.size(0));
  if (new_loc.has_value()) {
    a.k_new = k_new->data_ptr();
    a.v_new = v_new->data_ptr();
    a.new_loc = new_loc->data_ptr();
    for (int i = 0; i < 3; ++i) a.knew_stride[i] = k_new->stride(i), a.vnew_stride[i] = v_new->stride(i);
    a.new_loc_int32 = new_loc->scalar_type() == at::kInt ? 1 : 0;
  }
  a.counter = counter.data_ptr<int32_t>();
  a.partial = partial.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.status = status.data_ptr<int32_t>();
  check_status(sgld_decode_persistent(&a, &p, &g, stream_of(out)), "sgld_decode_persistent");
}

void merge(const at::Tensor& partial, const at::Tensor& lse, const at::Tensor& counts, const at::Tensor& error,
           at::Tensor out) {
  const c10::cuda::CUDAGuard guard(partial.device());
  TORCH_CHECK_VALUE(partial.dim() == 4, "partial is [batch, heads, splits, head_dim]");
  check_status(sgld_merge_splits(partial.data_ptr<float>(), lse.data_ptr<float>(), counts.data_ptr<int32_t>(),
                                 error.data_ptr<int32_t>(), out.data_ptr(), dtype_code(out),
                                 static_cast<int32_t>(partial.size(0)), static_cast<int32_t>(partial.size(1)),
                                 static_cast<int32_t>(partial.size(3)), static_cast<int32_t>(partial.size(2)),
                                 stream_of(partial)),
               "sgld_merge_splits");
}

void plan_build_meta(const at::Tensor&, at::IntArrayRef, int64_t, const std::optional<at::Tensor>&, int64_t,
                     const std::optional<at::Tensor>&) {}
void decode_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                 const std::optional<at::Tensor>&, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                 const at::Tensor&, at::IntArrayRef, int64_t, double, double, double, double,
                 const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&) {}
void merge_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, at::Tensor) {}

}  // namespace

TORCH_LIBRARY(sglang_decode, m) {
  m.def("plan_build(Tensor(a!) plan, int[] geometry, int force_mode, Tensor? rules, int n_rules, "
        "Tensor(b!)? counters) -> ()");
  m.def("decode(Tensor q, Tensor(a!) k, Tensor(b!) v, Tensor pages, Tensor? indptr, Tensor(c!) out, "
        "Tensor(d!) partial, Tensor(e!) lse, Tensor(f!) counter, Tensor(g!) status, Tensor plan, int[] geometry, "
        "int page_size, float scale, float logit_cap, float k_scale, float v_scale, Tensor? k_new, Tensor? v_new, "
        "Tensor? new_loc) -> ()");
  m.def("merge(Tensor partial, Tensor lse, Tensor counts, Tensor error, Tensor(a!) out) -> ()");
}

TORCH_LIBRARY_IMPL(sglang_decode, CUDA, m) {
  m.impl("plan_build", &plan_build);
  m.impl("decode", &decode);
  m.impl("merge", &merge);
}

TORCH_LIBRARY_IMPL(sglang_decode, Meta, m) {
  m.impl("plan_build", &plan_build_meta);
  m.impl("decode", &decode_meta);
  m.impl("merge", &merge_meta);
}
