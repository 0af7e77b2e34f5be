// Split merge -- the reference's merge_splits (kernels/merge.py:7-30).
//
// One warp per (request, query head), four head dims per lane (float4).  Per row:
// the LSE-weighted merge of the first counts[request] split slots, in split order
// (the recurrence m' = max(m, l_s), acc = acc*e^(m-m') + p_s*e^(l_s-m'), same for
// the denominator), output = acc / max(den, 1e-30); rows without splits are zero and
// every output is NaN when the plan's error word is set.  Slots >= counts[request]
// are never read (they may hold stale NaN).  The split loads of a row are issued
// eight at a time so the merge costs a few memory round trips, not one per split.
//
// Launched right after the decode kernel with programmatic dependent launch: the
// CTAs may start while the decode grid drains and wait (griddepcontrol.wait) until
// its stores are visible.  Launched on its own (sgld_merge_splits) the wait is a no-op.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kWarpsPerBlock = 4;
constexpr int kUnroll = 8;

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
    const int32_t* __restrict__ error, T* __restrict__ out, int bcap, int hq, int d_dim, int smax) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);   // (request, head)
  const int lane = threadIdx.x & 31;
  if (row >= bcap * hq) return;
  const int request = row / hq;
  const int n = counts[request];
  const bool err = *error != 0;
  T* orow = out + static_cast<int64_t>(row) * d_dim;
  const int64_t base = static_cast<int64_t>(row) * smax;
  for (int d = lane * 4; d < d_dim; d += 128) {
    float mm = -INFINITY, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < n; s0 += kUnroll) {
      float l[kUnroll];
      float4 p[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (s0 + u < n) {
          l[u] = __ldcg(lse + base + s0 + u);
          p[u] = __ldcg(reinterpret_cast<const float4*>(partial + (base + s0 + u) * d_dim + d));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (s0 + u < n) {
          const float nm = fmaxf(mm, l[u]);
          const float ow = ex2((mm - nm) * kLog2e);
          const float w = ex2((l[u] - nm) * kLog2e);
          acc.x = acc.x * ow + p[u].x * w;
          acc.y = acc.y * ow + p[u].y * w;
          acc.z = acc.z * ow + p[u].z * w;
          acc.w = acc.w * ow + p[u].w * w;
          den = den * ow + w;
          mm = nm;
        }
      }
    }
    const float inv = 1.f / fmaxf(den, 1.0e-30f);
    float4 r = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (n == 0) r = make_float4(0.f, 0.f, 0.f, 0.f);
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
                         int32_t d, int32_t smax, cudaStream_t stream, bool programmatic) {
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
                              static_cast<int>(d), static_cast<int>(smax));
  }
  return cudaLaunchKernelEx(&cfg, merge_kernel<__half>, partial, lse, counts, error, static_cast<__half*>(out),
                            static_cast<int>(bcap), static_cast<int>(hq), static_cast<int>(d),
                            static_cast<int>(smax));
}

}  // namespace sgld
