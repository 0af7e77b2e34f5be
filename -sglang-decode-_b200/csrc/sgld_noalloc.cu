// sgld_decode_persistent_noalloc: the decode + merge of sgld_decode_persistent for
// callers that cannot allocate device memory.
//
// Some hosts hand the library only the input and output buffers of a call and cannot
// provide per-layer scratch: plugin interfaces whose signature carries no workspace, or
// servers that give all free device memory to their KV-cache pool at start-up and allow
// no allocation afterwards (cudaMalloc also synchronises the device, which a serving
// loop cannot afford).  For them the scratch of the decode -- the two claim words, and
// the fp32 partial outputs and LSEs of every split slot -- lives in one
// file-scope device array of kScratchBytes bytes, reserved on every GPU that loads the
// library until the process exits.  The status word stays with the caller (a word inside
// the array could not be read back, and a timed-out call would look like a good one).
//
// Host code only sees a stand-in for the array's name, never its device address: the
// address is obtained with cudaGetSymbolAddress (with the device current) on the first
// call made on a device, and again when the device's context changes (after a device
// reset), and passed to the kernels.  Make the first call on each device before any
// stream capture.  The entry point allocates and frees nothing.
//
// Every call shares the one array and leaves its last contents there.  Each call clears
// the words that must start at zero (the two claim words) on its stream before the
// decode, after every argument check has passed; calls whose GPU work overlaps
// (different streams, or several threads) race on the array and must be serialised by
// the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "sgld_internal.cuh"

namespace {

constexpr size_t kScratchBytes = size_t{16} << 20;   // 16 MiB per GPU
constexpr size_t kHeaderBytes = 256;                  // counter[2] + padding
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct ScratchAddress {
  void* context = nullptr;   // CUcontext the address was looked up in
  void* address = nullptr;
};

std::mutex g_setup_mutex;
ScratchAddress g_scratch[kMaxDevices];

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

extern "C" int sgld_decode_persistent_noalloc(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                                              const sgld_plan_geometry* geometry, void* stream) {
  if (args == nullptr || geometry == nullptr)
    return sgld::set_last_error(SGLD_ERR_INVALID_ARGUMENT, "decode args or geometry are NULL");
  if (args->status == nullptr)
    return sgld::set_last_error(SGLD_ERR_INVALID_ARGUMENT,
                                "status is NULL: the allocation-free entry point needs a caller-readable "
                                "status word (bounded-wait and slot errors are reported there)");
  if (geometry->batch_capacity <= 0 || geometry->max_splits <= 0 || args->query_heads <= 0 ||
      args->head_dim <= 0)
    return sgld::set_last_error(SGLD_ERR_INVALID_ARGUMENT, "geometry fields must be positive");
  // Layout of the array: [256-byte header: the two claim words][partial, rounded up to
  // 256 bytes][lse, rounded up to 256 bytes].
  const size_t slots = static_cast<size_t>(geometry->batch_capacity) * args->query_heads * geometry->max_splits;
  const size_t partial_bytes = round_up(slots * args->head_dim * sizeof(float), 256);
  const size_t lse_bytes = round_up(slots * sizeof(float), 256);
  const size_t needed = kHeaderBytes + partial_bytes + lse_bytes;
  if (needed > kScratchBytes) {
    static thread_local char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "this geometry needs %zu bytes of scratch; the allocation-free entry point holds at most "
                  "%zu bytes (16 MiB) -- use sgld_decode_persistent with caller-owned scratch",
                  needed, kScratchBytes);
    return sgld::set_last_error(SGLD_ERR_INVALID_ARGUMENT, msg);
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return sgld::set_last_error(SGLD_ERR_CUDA, "cudaGetDevice failed or device ordinal out of range");
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    ScratchAddress& slot = g_scratch[device];
    void* ctx = sgld::current_context();
    if (slot.address == nullptr || ctx == nullptr || slot.context != ctx) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
      if (e != cudaSuccess || addr == nullptr)
        return sgld::set_last_error(SGLD_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch failed");
      slot.address = addr;
      slot.context = ctx;
    }
    base = static_cast<unsigned char*>(slot.address);
  }
  sgld_decode_args a = *args;
  a.counter = reinterpret_cast<int32_t*>(base);
  a.partial = reinterpret_cast<float*>(base + kHeaderBytes);
  a.lse = reinterpret_cast<float*>(base + kHeaderBytes + partial_bytes);
  // Check everything before enqueueing anything, so a rejected call leaves no work behind.
  const int rc = sgld::validate_decode(&a, plan, geometry);
  if (rc != SGLD_OK) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The two claim words must start at zero; everything else is written
  // before it is read.
  if (cudaMemsetAsync(base, 0, 2 * sizeof(int32_t), st) != cudaSuccess)
    return sgld::set_last_error(SGLD_ERR_CUDA, "clearing the no-alloc scratch header failed");
  return sgld_decode_persistent(&a, plan, geometry, stream);
}
