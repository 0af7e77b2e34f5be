// PyTorch operator library over the C ABI (include/sgld_b200.h): registers
//   torch.ops.sglang_decode.plan_build, .decode and .merge
// so the decode path is visible to torch's operator registry (schemas with mutation
// annotations, Meta kernels for tracing) while every launch still goes through the
// torch-free C entry points of libsgld_sm100.so.  Strides, pointers and the current CUDA
// stream are read here, in C++, instead of by ctypes in Python.
//
// The ops replace the reference's Triton launches: plan_build <- planning/builder.py:6-28,
// decode <- runtime/engine.py:62-73, merge <- kernels/merge.py:7-30.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>
#include <ATen/ATen.h>

#include <array>
#include <cstring>
#include <string>

#include "sgld_b200.h"

namespace {

constexpr int kPlanFields = 20;   // sgld_plan_buffers, in declaration order

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

sgld_plan_buffers plan_of(const std::vector<at::Tensor>& plan) {
  TORCH_CHECK_VALUE(static_cast<int>(plan.size()) == kPlanFields, "plan must hold ", kPlanFields, " int32 tensors");
  std::array<int32_t*, kPlanFields> p{};
  for (int i = 0; i < kPlanFields; ++i) {
    TORCH_CHECK_VALUE(plan[i].scalar_type() == at::kInt && plan[i].is_cuda(), "plan tensors must be int32 CUDA tensors");
    p[i] = plan[i].data_ptr<int32_t>();
  }
  sgld_plan_buffers b;
  static_assert(sizeof(b) == sizeof(p), "sgld_plan_buffers is 20 pointers");
  std::memcpy(&b, p.data(), sizeof(b));
  return b;
}

sgld_plan_geometry geometry_of(at::IntArrayRef g) {
  TORCH_CHECK_VALUE(g.size() == 5, "geometry is (batch_capacity, max_splits, max_context, groups, workers)");
  return sgld_plan_geometry{static_cast<int32_t>(g[0]), static_cast<int32_t>(g[1]), static_cast<int32_t>(g[2]),
                            static_cast<int32_t>(g[3]), static_cast<int32_t>(g[4])};
}

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void plan_build(std::vector<at::Tensor> plan, at::IntArrayRef geometry, int64_t force_mode,
                const std::optional<at::Tensor>& rules, int64_t n_rules, const std::optional<at::Tensor>& counters) {
  const c10::cuda::CUDAGuard guard(plan.at(0).device());
  const sgld_plan_buffers p = plan_of(plan);
  const sgld_plan_geometry g = geometry_of(geometry);
  const int32_t* r = rules.has_value() && n_rules > 0 ? rules->data_ptr<int32_t>() : nullptr;
  int32_t* c = counters.has_value() ? counters->data_ptr<int32_t>() : nullptr;
  const int32_t nc = counters.has_value() ? static_cast<int32_t>(counters->numel()) : 0;
  check_status(sgld_plan_build(&p, &g, static_cast<int32_t>(force_mode), r, static_cast<int32_t>(n_rules), c, nc,
                               stream_of(plan.at(0))),
               "sgld_plan_build");
}

// K/V: paged [pages, page_size, Hkv, D] or CSR [tokens, Hkv, D] (indptr given).
void decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pages,
            const std::optional<at::Tensor>& indptr, at::Tensor out, at::Tensor partial, at::Tensor lse,
            at::Tensor counter, at::Tensor status, std::vector<at::Tensor> plan, at::IntArrayRef geometry,
            int64_t query_heads, int64_t kv_heads, int64_t head_dim, int64_t page_size, double scale,
            double logit_cap, double k_scale, double v_scale, const std::optional<at::Tensor>& k_new,
            const std::optional<at::Tensor>& v_new, const std::optional<at::Tensor>& new_loc) {
  const c10::cuda::CUDAGuard guard(q.device());
  const sgld_plan_buffers p = plan_of(plan);
  const sgld_plan_geometry g = geometry_of(geometry);
  sgld_decode_args a;
  std::memset(&a, 0, sizeof(a));
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.out = out.data_ptr();
  a.pages = pages.data_ptr<int32_t>();
  for (int i = 0; i < 3; ++i) a.q_stride[i] = q.stride(i);
  const bool csr = indptr.has_value();
  if (csr) {
    TORCH_CHECK_VALUE(k.dim() == 3 && v.dim() == 3, "CSR K/V are [tokens, kv_heads, head_dim]");
    a.indptr = indptr->data_ptr<int32_t>();
    const int64_t ks[4] = {k.stride(0), 0, k.stride(1), k.stride(2)};
    const int64_t vs[4] = {v.stride(0), 0, v.stride(1), v.stride(2)};
    std::memcpy(a.k_stride, ks, sizeof(ks));
    std::memcpy(a.v_stride, vs, sizeof(vs));
  } else {
    TORCH_CHECK_VALUE(k.dim() == 4 && v.dim() == 4 && pages.dim() == 2, "paged K/V are [pages, page_size, kv_heads, head_dim]");
    for (int i = 0; i < 4; ++i) a.k_stride[i] = k.stride(i), a.v_stride[i] = v.stride(i);
    a.pt_stride[0] = pages.stride(0);
    a.pt_stride[1] = pages.stride(1);
  }
  a.kv_extent = k.size(0) == v.size(0) ? k.size(0) : 0;
  a.dtype = dtype_code(q);
  a.kv_dtype = dtype_code(k);
  a.query_heads = static_cast<int32_t>(query_heads);
  a.kv_heads = static_cast<int32_t>(kv_heads);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.page_size = static_cast<int32_t>(page_size);
  a.scale = static_cast<float>(scale);
  a.logit_cap = static_cast<float>(logit_cap);
  a.k_scale = static_cast<float>(k_scale);
  a.v_scale = static_cast<float>(v_scale);
  a.q_rows = static_cast<int32_t>(q.size(0));
  if (new_loc.has_value()) {
    TORCH_CHECK_VALUE(k_new.has_value() && v_new.has_value(), "the KV-cache write needs k_new, v_new and new_loc");
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
  check_status(sgld_decode_persistent(&a, &p, &g, stream_of(q)), "sgld_decode_persistent");
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

void plan_build_meta(std::vector<at::Tensor>, at::IntArrayRef, int64_t, const std::optional<at::Tensor>&, int64_t,
                     const std::optional<at::Tensor>&) {}
void decode_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                 const std::optional<at::Tensor>&, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                 std::vector<at::Tensor>, at::IntArrayRef, int64_t, int64_t, int64_t, int64_t, double, double, double,
                 double, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                 const std::optional<at::Tensor>&) {}
void merge_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, at::Tensor) {}

}  // namespace

TORCH_LIBRARY(sglang_decode, m) {
  m.def("plan_build(Tensor(a!)[] plan, int[] geometry, int force_mode, Tensor? rules, int n_rules, "
        "Tensor(b!)? counters) -> ()");
  m.def("decode(Tensor q, Tensor(a!) k, Tensor(b!) v, Tensor pages, Tensor? indptr, Tensor(c!) out, "
        "Tensor(d!) partial, Tensor(e!) lse, Tensor(f!) counter, Tensor(g!) status, Tensor[] plan, int[] geometry, "
        "int query_heads, int kv_heads, int head_dim, int page_size, float scale, float logit_cap, float k_scale, "
        "float v_scale, Tensor? k_new, Tensor? v_new, Tensor? new_loc) -> ()");
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
