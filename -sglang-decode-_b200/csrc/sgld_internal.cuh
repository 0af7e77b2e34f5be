// Internal declarations shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sgld_b200.h"  // include/ is on the include path (-I)

namespace sgld {

constexpr int kBlockKV = 128;        // weight unit / tile of the reference (config.py:24)
constexpr int kSplitAlign = 32;      // split chunk alignment (config.py:25)
constexpr int kMaxRecords = 4096;    // record_capacity bound (config.py:37)
constexpr int kMaxPlanWorkers = 4096;
constexpr int kMaxBuckets = 32;

struct PlanLaunch {
  sgld_plan_buffers p;
  int32_t bcap, smax, maxctx, groups, workers, buckets;
  int32_t force;
  const int32_t* rules;
  int32_t n_rules;
  int32_t* counters;
  int32_t n_counters;
};

// Host-side launchers (return a cudaError_t of the launch).
cudaError_t launch_plan(const PlanLaunch& a, cudaStream_t stream);

// Kernel parameter block of one decode launch (passed as a __grid_constant__).
struct alignas(64) DecodeLaunch {
  CUtensorMap kmap;  // 4D tensor maps {D, Hkv, page_size, pages} of K and V (paged TMA path)
  CUtensorMap vmap;
  CUtensorMap qmap;  // 3D tensor map {D, Hq, q_rows} of Q (tcgen05 kernel)
  sgld_decode_args d;
  sgld_plan_buffers p;
  int32_t bcap, smax, workers, group_size;
  int32_t csr;
  int32_t fast_kv;   // K/V rows are 16-byte aligned, unit stride along D
  int32_t fast_q;    // Q rows are 16-byte aligned, unit stride along D
  int32_t kv_fp8;    // K/V are e4m3 (Q and the output are fp16/bf16)
  int32_t tma_kv;    // paged KV loaded by tensor-map TMA boxes of box_rows tokens
  int32_t box_rows;
  int32_t q_rows;    // rows of q (requests at or past it read a zero query, status bit 64)
};

// KV-cache write launched right before the decode of the same call (SGLang's
// set_kv_buffer): row (r, head) of k_new / v_new goes to token slot new_loc[r].
struct KVWrite {
  const void* k_new;
  const void* v_new;
  const void* new_loc;
  void* k;
  void* v;
  int64_t k_stride[4], v_stride[4];   // pool strides (page, token-in-page, head, dim)
  int64_t kn_stride[3], vn_stride[3]; // new-row strides (request, head, dim)
  int64_t slots;                      // token slots in the pool (0: unchecked)
  int32_t rows, page_size, kv_heads, head_dim, loc_int32;
  int32_t dtype;                      // of k_new / v_new (SGLD_DTYPE_F16 / BF16)
  int32_t pool_fp8;                   // pool holds e4m3: store e4m3(x / scale), saturating
  float k_scale, v_scale;
  int32_t* status;
};

// programmatic: launch as a programmatic dependent of the preceding kernel (PDL); the
// kernel still waits for that kernel (which may have produced k_new / v_new) to finish.
cudaError_t launch_kv_write(const KVWrite& kv, cudaStream_t stream, bool programmatic);

cudaError_t launch_decode(const DecodeLaunch& a, cudaStream_t stream);
// Small-batch kernel: one CTA per task of the capacity (head_dim 128, 16-bit K/V, group <= 8,
// 16-byte aligned K/V and Q rows).
cudaError_t launch_decode_small(const DecodeLaunch& a, cudaStream_t stream);
// tcgen05 kernel (head_dim 128, 16-bit K/V, 16-byte aligned rows, qmap encoded).
cudaError_t launch_decode_tc(const DecodeLaunch& a, cudaStream_t stream);

// Record `msg` as the calling host thread's sgld_last_error() message; returns `code`.
int set_last_error(int code, const char* msg);

// Every host-side check of sgld_decode_persistent (nothing is enqueued); SGLD_OK or the
// status that call would return, with sgld_last_error() set.
int validate_decode(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                    const sgld_plan_geometry* geometry);

// The calling thread's current CUDA context (a CUcontext), nullptr if unknown.
void* current_context();

// programmatic: launch as a programmatic dependent of the preceding kernel (PDL).
// claim: the preceding decode's two claim words, zeroed once that decode has completed
// (nullptr for a merge on its own).
cudaError_t launch_merge(const float* partial, const float* lse, const int32_t* counts,
                         const int32_t* error, void* out, int32_t dtype, int32_t bcap, int32_t hq,
                         int32_t d, int32_t smax, cudaStream_t stream, bool programmatic,
                         int32_t* claim);

}  // namespace sgld
