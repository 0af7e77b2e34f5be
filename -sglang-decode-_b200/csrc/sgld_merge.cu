// Stand-alone split merge -- the reference's merge_splits (kernels/merge.py:7-30).
//
// Grid (Bcap, Hq), one thread per head-dim element.  Per (request, head): an
// LSE-weighted merge of the first counts[request] split slots, in split order,
// with the 1e-30 denominator floor; every output is NaN when the plan's error
// word is set.  Slots >= counts[request] are never read (they may hold stale NaN).
// The decode launch fuses this merge; this kernel serves callers that run the
// merge separately and the parity tests of the fused path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
__global__ void merge_kernel(const float* __restrict__ partial, const float* __restrict__ lse,
                             const int32_t* __restrict__ counts, const int32_t* __restrict__ error,
                             T* __restrict__ out, int hq, int d_dim, int smax) {
  const int request = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  if (d >= d_dim) return;
  const int n = counts[request];
  const int64_t base = (static_cast<int64_t>(request) * hq + head) * smax;
  float m = -INFINITY, den = 0.f, acc = 0.f;
  for (int s = 0; s < n; ++s) {
    const float l = lse[base + s];
    const float p = partial[(base + s) * d_dim + d];
    const float nm = fmaxf(m, l);
    const float ow = ex2((m - nm) * kLog2e);
    const float w = ex2((l - nm) * kLog2e);
    acc = acc * ow + p * w;
    den = den * ow + w;
    m = nm;
  }
  float result = acc / fmaxf(den, 1.0e-30f);
  if (*error != 0) result = __int_as_float(0x7fc00000);
  out[(static_cast<int64_t>(request) * hq + head) * d_dim + d] = from_float<T>(result);
}

}  // namespace

cudaError_t launch_merge(const float* partial, const float* lse, const int32_t* counts,
                         const int32_t* error, void* out, int32_t dtype, int32_t bcap, int32_t hq,
                         int32_t d, int32_t smax, cudaStream_t stream) {
  dim3 grid(bcap, hq);
  if (dtype == SGLD_DTYPE_BF16) {
    merge_kernel<__nv_bfloat16><<<grid, d, 0, stream>>>(partial, lse, counts, error,
                                                        static_cast<__nv_bfloat16*>(out), hq, d, smax);
  } else {
    merge_kernel<__half><<<grid, d, 0, stream>>>(partial, lse, counts, error, static_cast<__half*>(out),
                                                 hq, d, smax);
  }
  return cudaGetLastError();
}

}  // namespace sgld
