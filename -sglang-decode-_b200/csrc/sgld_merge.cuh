// The split merge of one output row chunk -- the reference's merge_splits
// (kernels/merge.py:7-30) -- shared by the stand-alone merge kernel and the small-batch
// decode kernel's fused merge, so both give the same bits.
//
// Four head dims of one (request, query head) row: the LSE-weighted merge of the first `n`
// split slots, in split order (m' = max(m, l_s), acc = acc*e^(m-m') + p_s*e^(l_s-m'), same
// for the denominator), result acc / max(den, 1e-30).  The multiply-adds are written as
// explicit __fmaf_rn / __fmul_rn so that the compiler cannot contract them differently at
// the two call sites.  Loads are issued kUnroll splits at a time (a few memory round trips per
// row, not one per split) and bypass L1 (.cg): the slots were written by other CTAs.
#pragma once

#include <cuda_runtime.h>

#include "sgld_ptx.cuh"

namespace sgld {

constexpr float kMergeLog2e = 1.4426950408889634f;

// `lse_row` = lse + row * smax, `partial_row` = partial + row * smax * d_dim + d.  kUnroll
// splits are loaded at a time; it changes the load batching only, not the arithmetic order.
template <int kUnroll = 8>
__device__ __forceinline__ float4 merge_row4(const float* __restrict__ partial_row, const float* __restrict__ lse_row,
                                             int n, int d_dim) {
  float mm = -INFINITY, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < n; s0 += kUnroll) {
    float l[kUnroll];
    float4 p[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (s0 + u < n) {
        l[u] = __ldcg(lse_row + s0 + u);
        p[u] = __ldcg(reinterpret_cast<const float4*>(partial_row + static_cast<int64_t>(s0 + u) * d_dim));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (s0 + u < n) {
        const float nm = fmaxf(mm, l[u]);
        const float ow = ex2((mm - nm) * kMergeLog2e);
        const float w = ex2((l[u] - nm) * kMergeLog2e);
        acc.x = __fmaf_rn(acc.x, ow, __fmul_rn(p[u].x, w));
        acc.y = __fmaf_rn(acc.y, ow, __fmul_rn(p[u].y, w));
        acc.z = __fmaf_rn(acc.z, ow, __fmul_rn(p[u].z, w));
        acc.w = __fmaf_rn(acc.w, ow, __fmul_rn(p[u].w, w));
        den = __fmaf_rn(den, ow, w);
        mm = nm;
      }
    }
  }
  if (n == 0) return make_float4(0.f, 0.f, 0.f, 0.f);
  const float inv = 1.f / fmaxf(den, 1.0e-30f);
  return make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
}

}  // namespace sgld
