// C ABI entry points (include/sgld_b200.h): host-side argument checks, then one
// asynchronous launch each.  No allocation, no synchronisation, no host readback.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "sgld_internal.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return SGLD_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int bit_length(int64_t x) {
  int n = 0;
  while (x > 0) {
    ++n;
    x >>= 1;
  }
  return n;
}

// Capacity contract of the reference's DecodeConfig (config.py:27-38), minus the
// group-size whitelist (any integer group 1..16 is supported here).
int check_geometry(const sgld_plan_geometry* g) {
  if (g == nullptr) return fail(SGLD_ERR_INVALID_ARGUMENT, "geometry is NULL");
  if (g->batch_capacity <= 0 || g->max_splits <= 0 || g->max_context <= 0 || g->groups <= 0 ||
      g->workers <= 0)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "geometry fields must be positive");
  const int64_t records = static_cast<int64_t>(g->batch_capacity) * g->max_splits;
  if (records > sgld::kMaxRecords)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "record capacity batch_capacity*max_splits exceeds 4096");
  if (records * g->groups >= (int64_t{1} << 31))
    return fail(SGLD_ERR_INVALID_ARGUMENT, "task capacity must stay below 2^31");
  if (g->workers > sgld::kMaxPlanWorkers)
    return fail(SGLD_ERR_UNSUPPORTED, "workers above 4096 are not supported");
  return SGLD_OK;
}

int plan_buckets(const sgld_plan_geometry* g) {
  const int64_t tiles = (static_cast<int64_t>(g->max_context) + sgld::kBlockKV - 1) / sgld::kBlockKV;
  return bit_length(tiles - 1) + 1;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 4D map {D, Hkv, page_size, pages} over a paged K or V tensor with element strides
// (head, token-in-page, page); boxes of {64 dims, 1 head, box_rows tokens, 1 page}
// land in shared memory with the 128-byte swizzle.
bool encode_paged_map(CUtensorMap* map, const void* base, int32_t dtype, int64_t d, int64_t hkv, int64_t ps,
                      int64_t pages, const int64_t* stride, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(hkv), static_cast<cuuint64_t>(ps),
                        static_cast<cuuint64_t>(pages)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(stride[2]) * 2, static_cast<cuuint64_t>(stride[1]) * 2,
                           static_cast<cuuint64_t>(stride[0]) * 2};
  for (cuuint64_t st : strides)
    if (st == 0 || st % 16 != 0 || st >= (cuuint64_t{1} << 40)) return false;
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType type =
      dtype == SGLD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, type, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3D map {D, Hq, rows} over Q with element strides (head, request); boxes of {64 dims,
// 16 heads, 1 request} land in shared memory with the 128-byte swizzle.  Heads past Hq and
// requests past `rows` read as zeros.
bool encode_q_map(CUtensorMap* map, const void* base, int32_t dtype, int64_t d, int64_t hq, int64_t rows,
                  const int64_t* stride) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u) != 0 || stride[2] != 1) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(hq), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride[1]) * 2, static_cast<cuuint64_t>(stride[0]) * 2};
  for (cuuint64_t st : strides)
    if (st == 0 || st % 16 != 0 || st >= (cuuint64_t{1} << 40)) return false;
  cuuint32_t box[3] = {64, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType type =
      dtype == SGLD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, type, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Kernel choice.  SGLD_DECODE_KERNEL=tcgen05 selects the tcgen05 kernel wherever it applies,
// =small the small-batch kernel wherever it applies, =mma the persistent mma.sync kernel
// everywhere; unset, the measured-faster kernel for the geometry: the small-batch kernel when
// the whole task capacity is at most kSmallTaskCapacity, else the persistent mma.sync kernel.
constexpr int64_t kSmallTaskCapacity = 1024;

bool kernel_env_is(const char* name) {
  const char* v = std::getenv("SGLD_DECODE_KERNEL");
  return v != nullptr && std::strcmp(v, name) == 0;
}
bool kernel_env_unset() {
  const char* v = std::getenv("SGLD_DECODE_KERNEL");
  return v == nullptr || v[0] == 0;
}
bool use_tc_kernel() { return kernel_env_is("tcgen05"); }

bool tma_disabled_by_env() {
  const char* v = std::getenv("SGLD_DISABLE_TMA");
  return v != nullptr && v[0] == '1';
}

int check_plan_pointers(const sgld_plan_buffers* p) {
  if (p == nullptr) return fail(SGLD_ERR_INVALID_ARGUMENT, "plan buffers are NULL");
  const void* ptrs[] = {p->lengths, p->splits, p->active, p->counts, p->offsets, p->chunk,
                        p->request, p->split, p->begin, p->end, p->weight, p->order,
                        p->pack_first, p->pack_count, p->record_count, p->num_packs, p->mode,
                        p->error, p->static_head, p->static_next, p->arrivals};
  for (const void* q : ptrs)
    if (q == nullptr) return fail(SGLD_ERR_INVALID_ARGUMENT, "a plan buffer pointer is NULL");
  return SGLD_OK;
}

}  // namespace

namespace sgld {
// Record `msg` as this host thread's sgld_last_error() message and return `code`.
int set_last_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace sgld

extern "C" {

int32_t sgld_abi_version(void) { return SGLD_ABI_VERSION; }

const char* sgld_last_error(void) { return g_last_error.c_str(); }

size_t sgld_layer_workspace_bytes(int32_t batch_capacity, int32_t query_heads, int32_t kv_heads,
                                  int32_t head_dim, int32_t max_splits) {
  if (batch_capacity <= 0 || query_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || max_splits <= 0)
    return 0;
  const size_t slots = static_cast<size_t>(batch_capacity) * query_heads * max_splits;
  return 2 * sizeof(int32_t)                                   /* claim counter + spare */
         + slots * head_dim * sizeof(float)                    /* partial */
         + slots * sizeof(float)                               /* lse */
         + sizeof(int32_t);                                    /* status */
}

size_t sgld_plan_storage_words(const sgld_plan_geometry* g) {
  if (g == nullptr || g->batch_capacity <= 0 || g->max_splits <= 0 || g->groups <= 0 || g->workers <= 0) return 0;
  const size_t b = static_cast<size_t>(g->batch_capacity), e = b * g->max_splits, t = e * g->groups;
  return 5 * b + 2 + 6 * e + 3 * t + 4 + static_cast<size_t>(g->workers) + b * g->groups;   // sizes as listed below
}

int sgld_plan_buffers_in_storage(int32_t* storage, const sgld_plan_geometry* g, sgld_plan_buffers* out) {
  if (storage == nullptr || out == nullptr || sgld_plan_storage_words(g) == 0)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "storage, geometry or output is NULL or empty");
  const size_t b = static_cast<size_t>(g->batch_capacity), e = b * g->max_splits, t = e * g->groups;
  int32_t* cur = storage;
  auto take = [&cur](size_t n) {
    int32_t* p = cur;
    cur += n;
    return p;
  };
  out->lengths = take(b);
  out->splits = take(b);
  out->active = take(1);
  out->counts = take(b);
  out->offsets = take(b + 1);
  out->chunk = take(b);
  out->request = take(e);
  out->split = take(e);
  out->begin = take(e);
  out->end = take(e);
  out->weight = take(e);
  out->order = take(e);
  out->pack_first = take(t);
  out->pack_count = take(t);
  out->record_count = take(1);
  out->num_packs = take(1);
  out->mode = take(1);
  out->error = take(1);
  out->static_head = take(static_cast<size_t>(g->workers));
  out->static_next = take(t);
  out->arrivals = take(b * g->groups);
  return SGLD_OK;
}

int sgld_plan_build(const sgld_plan_buffers* plan, const sgld_plan_geometry* geometry,
                    int32_t force_mode, const int32_t* rules, int32_t n_rules,
                    int32_t* layer_counters, int32_t n_counter_words, void* stream) {
  int rc = check_geometry(geometry);
  if (rc) return rc;
  if ((rc = check_plan_pointers(plan))) return rc;
  if (force_mode < -1 || force_mode > 4) return fail(SGLD_ERR_INVALID_ARGUMENT, "force_mode must be -1..4");
  if (n_rules < 0 || (n_rules > 0 && rules == nullptr))
    return fail(SGLD_ERR_INVALID_ARGUMENT, "rules pointer/count mismatch");
  if (n_counter_words < 0 || (n_counter_words > 0 && layer_counters == nullptr))
    return fail(SGLD_ERR_INVALID_ARGUMENT, "counter pointer/count mismatch");
  sgld::PlanLaunch a;
  a.p = *plan;
  a.bcap = geometry->batch_capacity;
  a.smax = geometry->max_splits;
  a.maxctx = geometry->max_context;
  a.groups = geometry->groups;
  a.workers = geometry->workers;
  a.buckets = plan_buckets(geometry);
  a.force = force_mode;
  a.rules = rules;
  a.n_rules = n_rules;
  a.counters = layer_counters;
  a.n_counters = n_counter_words;
  if (a.buckets > sgld::kMaxBuckets) return fail(SGLD_ERR_UNSUPPORTED, "max_context too large");
  cudaError_t e = sgld::launch_plan(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sgld_plan_build launch");
  return SGLD_OK;
}

}  // extern "C"

namespace sgld {

// Every host-side check of sgld_decode_persistent, with nothing enqueued: shapes, dtypes,
// pointers (scratch included), strides and capacities.  SGLD_OK when a launch may follow.
int validate_decode(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                    const sgld_plan_geometry* geometry) {
  if (args == nullptr) return fail(SGLD_ERR_INVALID_ARGUMENT, "decode args are NULL");
  int rc = check_geometry(geometry);
  if (rc) return rc;
  if ((rc = check_plan_pointers(plan))) return rc;
  const sgld_decode_args& d = *args;
  if (!d.q || !d.k || !d.v || !d.out || !d.pages || !d.counter || !d.partial || !d.lse || !d.status)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "a tensor or scratch pointer is NULL");
  if (!aligned16(d.partial))   // the epilogue and the merge move partial rows as float4
    return fail(SGLD_ERR_INVALID_ARGUMENT, "partial must be 16-byte aligned");
  if (!(d.logit_cap >= 0.f) || d.logit_cap > 3.0e38f)   // rejects NaN, negatives and infinity
    return fail(SGLD_ERR_INVALID_ARGUMENT, "logit_cap must be a finite value >= 0 (0 disables it)");
  if (!(d.k_scale >= 0.f) || d.k_scale > 3.0e38f || !(d.v_scale >= 0.f) || d.v_scale > 3.0e38f)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "k_scale / v_scale must be finite values >= 0 (0 reads as 1)");
  const bool kv_fp8 = d.kv_dtype == SGLD_DTYPE_E4M3;
  if (!kv_fp8 && d.kv_dtype != d.dtype)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "kv_dtype must equal dtype or be SGLD_DTYPE_E4M3");
  if (d.dtype != SGLD_DTYPE_F16 && d.dtype != SGLD_DTYPE_BF16)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "dtype must be fp16 or bf16");
  if (d.head_dim != 64 && d.head_dim != 128 && d.head_dim != 256)
    return fail(SGLD_ERR_UNSUPPORTED, "supported head dimensions: 64, 128, 256");
  if (kv_fp8 && d.head_dim != 128) return fail(SGLD_ERR_UNSUPPORTED, "fp8 K/V: head_dim 128 only");
  if (d.kv_heads <= 0 || d.query_heads <= 0 || d.query_heads % d.kv_heads)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "query heads must be a positive multiple of KV heads");
  const int group = d.query_heads / d.kv_heads;
  if (group > 16) return fail(SGLD_ERR_UNSUPPORTED, "GQA group sizes above 16 are not supported");
  if (d.kv_heads != geometry->groups)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "kv_heads must equal the plan's groups");
  if (d.page_size <= 0) return fail(SGLD_ERR_INVALID_ARGUMENT, "page_size must be positive");
  const bool csr = d.indptr != nullptr;
  if (csr && d.page_size != 1) return fail(SGLD_ERR_INVALID_ARGUMENT, "CSR indexing uses page_size 1");
  if (!(d.scale == d.scale)) return fail(SGLD_ERR_INVALID_ARGUMENT, "scale is NaN");
  const int32_t q_rows = d.q_rows == 0 ? geometry->batch_capacity : d.q_rows;
  if (q_rows < 0 || q_rows > geometry->batch_capacity)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "q_rows must be 0 (capacity) or 1..batch_capacity");
  const bool kv_write = d.new_loc != nullptr;
  if (!kv_write && (d.k_new != nullptr || d.v_new != nullptr))
    return fail(SGLD_ERR_INVALID_ARGUMENT, "k_new / v_new need new_loc");
  if (kv_write && (d.k_new == nullptr || d.v_new == nullptr))
    return fail(SGLD_ERR_INVALID_ARGUMENT, "the KV-cache write needs k_new, v_new and new_loc");

  return SGLD_OK;
}

// The calling thread's current CUDA context (a CUcontext), or nullptr when the driver
// entry point is unavailable.  Caches keyed by device ordinal compare it to notice a
// device reset (a new primary context reuses the ordinal but not the old addresses).
void* current_context() {
  using GetCurrent = CUresult (*)(CUcontext*);
  static GetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<GetCurrent>(nullptr);
    return reinterpret_cast<GetCurrent>(p);
  }();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

}  // namespace sgld

extern "C" {

}  // extern "C"

namespace {

// Fill the kernel parameter block of a validated call and choose the kernel; returns an
// SGLD_KERNEL_* value.
int prepare_launch(const sgld_decode_args& d, const sgld_plan_buffers* plan, const sgld_plan_geometry* geometry,
                   sgld::DecodeLaunch& a) {
  const bool kv_fp8 = d.kv_dtype == SGLD_DTYPE_E4M3;
  const int group = d.query_heads / d.kv_heads;
  const bool csr = d.indptr != nullptr;
  const int32_t q_rows = d.q_rows == 0 ? geometry->batch_capacity : d.q_rows;
  std::memset(&a, 0, sizeof(a));
  a.d = d;
  a.p = *plan;
  a.bcap = geometry->batch_capacity;
  a.smax = geometry->max_splits;
  a.workers = geometry->workers;
  a.group_size = group;
  a.csr = csr ? 1 : 0;
  if (csr) a.d.k_stride[1] = 0, a.d.v_stride[1] = 0;
  // 16-byte copies need 16-byte aligned rows: strides in whole 16-byte chunks of elements.
  const int64_t per_chunk = kv_fp8 ? 16 : 8;
  bool fast_kv = aligned16(d.k) && aligned16(d.v) && d.k_stride[3] == 1 && d.v_stride[3] == 1;
  for (int i = 0; i < 3; ++i)
    fast_kv = fast_kv && (a.d.k_stride[i] % per_chunk == 0) && (a.d.v_stride[i] % per_chunk == 0);
  a.kv_fp8 = kv_fp8 ? 1 : 0;
  if (a.d.k_scale == 0.f) a.d.k_scale = 1.f;
  if (a.d.v_scale == 0.f) a.d.v_scale = 1.f;
  a.q_rows = q_rows;
  a.fast_kv = fast_kv ? 1 : 0;
  a.fast_q = (aligned16(d.q) && d.q_stride[2] == 1 && d.q_stride[0] % 8 == 0 && d.q_stride[1] % 8 == 0) ? 1 : 0;
  const int ps = d.page_size;
  const bool pageable_tma = !csr && fast_kv && ps % 32 == 0 && d.kv_extent > 0 &&
                            d.kv_extent < (int64_t{1} << 31) && !tma_disabled_by_env();
  // The tcgen05 kernel: head_dim 128, 16-bit K/V in 16-byte rows, Q loadable by a TMA box.
  if (!kv_fp8 && d.head_dim == 128 && fast_kv && a.fast_q && use_tc_kernel() &&
      encode_q_map(&a.qmap, d.q, d.dtype, d.head_dim, d.query_heads, q_rows, d.q_stride)) {
    if (pageable_tma &&
        encode_paged_map(&a.kmap, d.k, d.dtype, d.head_dim, d.kv_heads, ps, d.kv_extent, d.k_stride, 32) &&
        encode_paged_map(&a.vmap, d.v, d.dtype, d.head_dim, d.kv_heads, ps, d.kv_extent, d.v_stride, 32)) {
      a.tma_kv = 1;
      a.box_rows = 32;
      return SGLD_KERNEL_TCGEN05_TMA;
    }
    return SGLD_KERNEL_TCGEN05;
  }
  // Small-batch kernel: one CTA per task of the capacity (head_dim 128, 16-bit K/V, group <= 8).
  const int64_t task_capacity = static_cast<int64_t>(geometry->batch_capacity) * geometry->max_splits * d.kv_heads;
  if (!kv_fp8 && d.head_dim == 128 && group <= 8 && fast_kv && a.fast_q && task_capacity <= (int64_t{1} << 20) &&
      (kernel_env_is("small") || (kernel_env_unset() && task_capacity <= kSmallTaskCapacity)))
    return SGLD_KERNEL_SMALL;
  // mma.sync kernel.  Paged KV by tensor-map TMA: a box of 32 tokens never crosses a page
  // because stages start 32-token aligned and 32 divides the page size.  Smaller pages stay
  // on the multi-warp cp.async path, which measured faster than 8- or 16-row boxes.  So do
  // D <= 128 kernels with a group of at most 8: they carry 10 cp.async producer warps,
  // which outrun a single thread issuing boxes (C4, page 64: 982 vs 1080 us).
  const bool wide_cp_async = d.head_dim <= 128 && group <= 8;
  if (!kv_fp8 && pageable_tma && !wide_cp_async) {
    const int box_rows = 32;
    if (encode_paged_map(&a.kmap, d.k, d.dtype, d.head_dim, d.kv_heads, ps, d.kv_extent, d.k_stride, box_rows) &&
        encode_paged_map(&a.vmap, d.v, d.dtype, d.head_dim, d.kv_heads, ps, d.kv_extent, d.v_stride, box_rows)) {
      a.tma_kv = 1;
      a.box_rows = box_rows;
      return SGLD_KERNEL_MMA_SYNC_TMA;
    }
  }
  return SGLD_KERNEL_MMA_SYNC;
}

}  // namespace

extern "C" {

int sgld_decode_kernel_kind(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                            const sgld_plan_geometry* geometry) {
  const int rc = sgld::validate_decode(args, plan, geometry);
  if (rc) return -rc;
  sgld::DecodeLaunch a;
  return prepare_launch(*args, plan, geometry, a);
}

int sgld_decode_persistent(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                           const sgld_plan_geometry* geometry, void* stream) {
  int rc = sgld::validate_decode(args, plan, geometry);
  if (rc) return rc;
  const sgld_decode_args& d = *args;
  const bool kv_fp8 = d.kv_dtype == SGLD_DTYPE_E4M3;
  const int32_t q_rows = d.q_rows == 0 ? geometry->batch_capacity : d.q_rows;
  const bool kv_write = d.new_loc != nullptr;
  const int ps = d.page_size;
  sgld::DecodeLaunch a;
  const int kind = prepare_launch(d, plan, geometry, a);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (kv_write) {   // the step's KV-cache write, chained right before the decode
    sgld::KVWrite kw = {};
    kw.k_new = d.k_new;
    kw.v_new = d.v_new;
    kw.new_loc = d.new_loc;
    kw.k = const_cast<void*>(d.k);
    kw.v = const_cast<void*>(d.v);
    for (int i = 0; i < 4; ++i) kw.k_stride[i] = a.d.k_stride[i], kw.v_stride[i] = a.d.v_stride[i];
    for (int i = 0; i < 3; ++i) kw.kn_stride[i] = d.knew_stride[i], kw.vn_stride[i] = d.vnew_stride[i];
    kw.slots = d.kv_extent > 0 ? d.kv_extent * ps : 0;
    kw.rows = q_rows;
    kw.page_size = ps;
    kw.kv_heads = d.kv_heads;
    kw.head_dim = d.head_dim;
    kw.loc_int32 = d.new_loc_int32 != 0 ? 1 : 0;
    kw.dtype = d.dtype;
    kw.pool_fp8 = kv_fp8 ? 1 : 0;
    kw.k_scale = a.d.k_scale;
    kw.v_scale = a.d.v_scale;
    kw.status = d.status;
    e = sgld::launch_kv_write(kw, st, true);
    if (e != cudaSuccess) return cuda_fail(e, "sgld_decode_persistent KV-cache write launch");
  }
  if (kind == SGLD_KERNEL_TCGEN05 || kind == SGLD_KERNEL_TCGEN05_TMA) e = sgld::launch_decode_tc(a, st);
  else if (kind == SGLD_KERNEL_SMALL) e = sgld::launch_decode_small(a, st);
  else e = sgld::launch_decode(a, st);
  if (e != cudaSuccess) return cuda_fail(e, "sgld_decode_persistent launch");
  if (kind == SGLD_KERNEL_SMALL) return SGLD_OK;   // the small-batch kernel merges the splits itself
  e = sgld::launch_merge(d.partial, d.lse, plan->counts, plan->error, d.out, d.dtype, geometry->batch_capacity,
                         d.query_heads, d.head_dim, geometry->max_splits, st, true, d.counter);
  if (e != cudaSuccess) return cuda_fail(e, "sgld_decode_persistent merge launch");
  return SGLD_OK;
}

int sgld_merge_splits(const float* partial, const float* lse, const int32_t* counts,
                      const int32_t* error, void* out, int32_t dtype, int32_t batch_capacity,
                      int32_t query_heads, int32_t head_dim, int32_t max_splits, void* stream) {
  if (!partial || !lse || !counts || !error || !out)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "a merge pointer is NULL");
  if (dtype != SGLD_DTYPE_F16 && dtype != SGLD_DTYPE_BF16)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "dtype must be fp16 or bf16");
  if (batch_capacity <= 0 || query_heads <= 0 || max_splits <= 0 || batch_capacity > 65535 ||
      query_heads > 65535)
    return fail(SGLD_ERR_INVALID_ARGUMENT, "merge geometry out of range");
  if (head_dim <= 0 || head_dim % 4 != 0 || head_dim > 4096)
    return fail(SGLD_ERR_UNSUPPORTED, "head_dim must be a multiple of 4 up to 4096");
  if (!aligned16(partial)) return fail(SGLD_ERR_INVALID_ARGUMENT, "partial must be 16-byte aligned");
  cudaError_t e = sgld::launch_merge(partial, lse, counts, error, out, dtype, batch_capacity, query_heads,
                                     head_dim, max_splits, static_cast<cudaStream_t>(stream), false, nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "sgld_merge_splits launch");
  return SGLD_OK;
}

}  // extern "C"
