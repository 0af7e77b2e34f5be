// KV-cache write of a decode step -- SGLang's set_kv_buffer, which the reference adapter
// calls before each layer's decode (integrations/sglang_backend.py:91-92).
//
// One warp per (request, KV head): row r of k_new / v_new goes to token slot new_loc[r]
// of the pool (paged: page new_loc / page_size, row new_loc % page_size).  Launched by
// sgld_decode_persistent right before the decode kernel, both with programmatic
// dependent launch: this kernel waits for its predecessor (the one that produced k_new /
// v_new) before reading, and the decode waits for this one before reading the pool, so
// the result is exactly "write, then decode" for any slots.  Slots outside the pool
// are skipped and set status bit 128.  An e4m3 pool stores e4m3(x / scale): the fp32
// quotient rounded once to nearest even, saturated to +-448 (torch's cast gives NaN past
// 464; SGLang divides in the 16-bit type first, a second rounding this write omits).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr int kWarpsPerBlock = 4;

__device__ __forceinline__ uint8_t to_e4m3(float x) {
  uint16_t pair;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.f), "f"(x));
  return static_cast<uint8_t>(pair & 0xffu);   // the second source lands in the low byte
}

template <typename T, typename P>
__device__ __forceinline__ void copy_row(P* dst, int64_t dst_stride, const T* src, int64_t src_stride, int d_dim,
                                         float scale) {
  const int lane = threadIdx.x & 31;
  for (int d = lane; d < d_dim; d += 32) {
    if constexpr (std::is_same<P, T>::value) {
      dst[d * dst_stride] = src[d * src_stride];
    } else {
      dst[d * dst_stride] = to_e4m3(to_float(src[d * src_stride]) / scale);   // one rounding, as fp32 x / s
    }
  }
}

template <typename T, typename P>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) kv_write_kernel(const __grid_constant__ KVWrite kv) {
  asm volatile("griddepcontrol.wait;" ::: "memory");   // k_new / v_new may come from the previous kernel
  const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= kv.rows * kv.kv_heads) return;
  const int r = row / kv.kv_heads, g = row - r * kv.kv_heads;
  const int64_t loc = kv.loc_int32 ? static_cast<int64_t>(static_cast<const int32_t*>(kv.new_loc)[r])
                                   : static_cast<const int64_t*>(kv.new_loc)[r];
  if (loc < 0 || (kv.slots > 0 && loc >= kv.slots)) {
    if ((threadIdx.x & 31) == 0) atomicOr(kv.status, 128);
    return;
  }
  const int64_t page = loc / kv.page_size, in = loc - page * kv.page_size;
  P* kd = static_cast<P*>(kv.k) + page * kv.k_stride[0] + in * kv.k_stride[1] + g * kv.k_stride[2];
  P* vd = static_cast<P*>(kv.v) + page * kv.v_stride[0] + in * kv.v_stride[1] + g * kv.v_stride[2];
  const T* ks = static_cast<const T*>(kv.k_new) + r * kv.kn_stride[0] + g * kv.kn_stride[1];
  const T* vs = static_cast<const T*>(kv.v_new) + r * kv.vn_stride[0] + g * kv.vn_stride[1];
  copy_row(kd, kv.k_stride[3], ks, kv.kn_stride[2], kv.head_dim, kv.k_scale);
  copy_row(vd, kv.v_stride[3], vs, kv.vn_stride[2], kv.head_dim, kv.v_scale);
}

template <typename T>
cudaError_t launch_typed(const KVWrite& kv, cudaLaunchConfig_t& cfg) {
  if (kv.pool_fp8) return cudaLaunchKernelEx(&cfg, kv_write_kernel<T, uint8_t>, kv);
  return cudaLaunchKernelEx(&cfg, kv_write_kernel<T, T>, kv);
}

}  // namespace

cudaError_t launch_kv_write(const KVWrite& kv, cudaStream_t stream, bool programmatic) {
  const int64_t rows = static_cast<int64_t>(kv.rows) * kv.kv_heads;
  if (rows <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock));
  cfg.blockDim = dim3(kWarpsPerBlock * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = programmatic ? 1 : 0;
  return kv.dtype == SGLD_DTYPE_BF16 ? launch_typed<__nv_bfloat16>(kv, cfg) : launch_typed<__half>(kv, cfg);
}

}  // namespace sgld
