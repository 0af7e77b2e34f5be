// Split merge -- the reference's merge_splits (kernels/merge.py:7-30).
//
// One warp per (request, query head), four head dims per lane (float4).  Per row:
// merge_row4 (sgld_merge.cuh) over the first counts[request] split slots, in split order;
// rows without splits are zero and every output is NaN when the plan's error word is set.
// Slots >= counts[request] are never read (they may hold stale NaN).
//
// Launched right after the decode kernel with programmatic dependent launch: the
// CTAs may start while the decode grid drains and wait (griddepcontrol.wait) until
// its stores are visible.  Launched on its own (sgld_merge_splits) the wait is a no-op.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sgld_internal.cuh"
#include "sgld_merge.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr int kWarpsPerBlock = 4;

template <typename T>
__device__ __forceinline__ void store4(T* dst, float4 v) {
  dst[0] = from_float<T>(v.x);
  dst[1] = from_float<T>(v.y);
  dst[2] = from_float<T>(v.z);
  dst[3] = from_float<T>(v.w);
}

template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) merge_kernel(
    const float* __restrict__ partial, const float* __restrict__ lse, const int32_t* __restrict__ counts,
    const int32_t* __restrict__ error, T* __restrict__ out, int bcap, int hq, int d_dim, int smax,
    int32_t* __restrict__ claim) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The decode grid has completed: leave its two claim words at zero for the next decode
  // on this layer (the decode kernel itself ends without touching them again).
  if (claim != nullptr && blockIdx.x == 0 && threadIdx.x < 2) claim[threadIdx.x] = 0;
  const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);   // (request, head)
  const int lane = threadIdx.x & 31;
  if (row >= bcap * hq) return;
  const int request = row / hq;
  const int n = counts[request];
  const bool err = *error != 0;
  T* orow = out + static_cast<int64_t>(row) * d_dim;
  const int64_t base = static_cast<int64_t>(row) * smax;
  for (int d = lane * 4; d < d_dim; d += 128) {
    float4 r = merge_row4(partial + base * d_dim + d, lse + base, n, d_dim);
    if (err) {
      const float q = __int_as_float(0x7fc00000);
      r = make_float4(q, q, q, q);
    }
    store4(orow + d, r);
  }
}

}  // namespace

cudaError_t launch_merge(const float* partial, const float* lse, const int32_t* counts,
                         const int32_t* error, void* out, int32_t dtype, int32_t bcap, int32_t hq,
                         int32_t d, int32_t smax, cudaStream_t stream, bool programmatic, int32_t* claim) {
  cudaLaunchConfig_t cfg = {};
  const int64_t rows = static_cast<int64_t>(bcap) * hq;
  cfg.gridDim = dim3(static_cast<unsigned>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock));
  cfg.blockDim = dim3(kWarpsPerBlock * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = programmatic ? 1 : 0;
  if (dtype == SGLD_DTYPE_BF16) {
    return cudaLaunchKernelEx(&cfg, merge_kernel<__nv_bfloat16>, partial, lse, counts, error,
                              static_cast<__nv_bfloat16*>(out), static_cast<int>(bcap), static_cast<int>(hq),
                              static_cast<int>(d), static_cast<int>(smax), claim);
  }
  return cudaLaunchKernelEx(&cfg, merge_kernel<__half>, partial, lse, counts, error, static_cast<__half*>(out),
                            static_cast<int>(bcap), static_cast<int>(hq), static_cast<int>(d),
                            static_cast<int>(smax), claim);
}

}  // namespace sgld
