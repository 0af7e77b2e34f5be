// GPU task-table builder: one CTA of 1024 threads does the whole step plan.
//
// Replaces the four Triton launches of the reference's build_plan
// (planning/builder.py:6-28) with one launch that reproduces every buffer they
// write, bit for bit:
//   1. count_scan          (kernels/plan.py:7-27)   validation, chunk, counts, offsets, error
//   2. emit_records        (kernels/plan.py:30-45)  SoA records
//   3. make_order_and_packs(kernels/plan.py:48-100) AUTO rules, uniform->R1, FORCE,
//                                                   stable ceil-log2 bucket order, packs
//   4. greedy_lists        (kernels/plan.py:103-135) exact LPT linked lists (mode STATIC)
// plus the per-layer claim-counter reset the reference issues as a memset per
// layer (runtime/engine.py:62).
//
// Stable ordering uses warp match/popc ranks (no comparison sort); the STATIC
// order is a bitonic sort on (weight desc, record asc) keys followed by a warp
// argmin per task with the reference's lowest-id tie rule.
#include <cuda_runtime.h>

#include "sgld_internal.cuh"

namespace sgld {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kIntMax = 0x7fffffff;

__device__ __forceinline__ int32_t wrap32(long long x) { return static_cast<int32_t>(static_cast<uint32_t>(x)); }

// floor division of an int32 by a positive int32 (Triton int32 cdiv on wrapped sums).
__device__ __forceinline__ int32_t floordiv(int32_t a, int32_t b) {
  return a >= 0 ? a / b : -static_cast<int32_t>((-static_cast<long long>(a) + b - 1) / b);
}

__device__ __forceinline__ int32_t cdiv32(int32_t a, int32_t b) { return floordiv(wrap32(static_cast<long long>(a) + b - 1), b); }

struct PlanShared {
  int32_t warp_scratch[kWarps];
  int32_t warp_scratch2[kWarps];
  int32_t scalars[8];
  int32_t bucket_count[kMaxBuckets];
  int32_t bucket_base[kMaxBuckets];
  int32_t bucket_running[kMaxBuckets];
  int32_t round_hist[kWarps][kMaxBuckets];
  int32_t round_prefix[kWarps][kMaxBuckets];
  int32_t pk_pack_base[kMaxBuckets];
  int32_t pk_record_base[kMaxBuckets];
  int32_t pk_width[kMaxBuckets];
  int32_t pk_ptasks[kMaxBuckets];
  int32_t pk_ppacks[kMaxBuckets];
  int32_t pk_count[kMaxBuckets];
  int32_t weight[kMaxRecords];
  unsigned long long keys[kMaxRecords];
  int32_t loads[kMaxPlanWorkers + 4];   // serial LPT loads, or the parallel LPT's run starts
  int32_t tails[kMaxPlanWorkers];
};

// Exclusive block scan of one int per thread; `total` receives the block sum.
__device__ int block_exclusive_scan(int v, PlanShared& s, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s.warp_scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s.warp_scratch[lane];
    int incl = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s.warp_scratch2[lane] = incl - w;
    if (lane == 31) s.scalars[7] = incl;
  }
  __syncthreads();
  total = s.scalars[7];
  int result = s.warp_scratch2[warp] + x - v;
  __syncthreads();
  return result;
}

__device__ int block_reduce_max(int v, PlanShared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_max_sync(0xffffffffu, v);
  if (lane == 0) s.warp_scratch[warp] = v;
  __syncthreads();
  int r = s.warp_scratch[0];
  for (int i = 1; i < kWarps; ++i) r = max(r, s.warp_scratch[i]);
  __syncthreads();
  return r;
}

__device__ int block_reduce_min(int v, PlanShared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_min_sync(0xffffffffu, v);
  if (lane == 0) s.warp_scratch[warp] = v;
  __syncthreads();
  int r = s.warp_scratch[0];
  for (int i = 1; i < kWarps; ++i) r = min(r, s.warp_scratch[i]);
  __syncthreads();
  return r;
}

// Saturating integer ceil-log2 exactly as kernels/plan.py:77-79 computes it.
__device__ __forceinline__ int bucket_of(int w, int buckets) {
  int b = 0;
  for (int k = 1; k < buckets; ++k) b += (w > (1 << (k - 1))) ? 1 : 0;
  return b;
}

// Exact LPT over the weight-sorted records (s.keys, heaviest first, lowest record id
// first among equal weights), one worker per thread (W <= 1024).
//
// The reference assigns tasks one at a time to the least-loaded worker, lowest worker id
// on ties (kernels/plan.py:120-135).  Within a run of k tasks of equal weight w this is
// the same as handing out the k smallest "slots" (L_i + m*w, i), m >= 0, in that order.
// With V0 = min L, L_i - V0 = q_i*w + rho_i (0 <= rho_i < w), slot (i, m) falls in round
// q_i + m at offset rho_i, so slots are ordered by (round, rho_i, i): each round takes its
// participants (q_i <= round) in (rho_i, i) order.  Rounds below max q_i need a block
// scan of the participant flags; from max q_i on every worker takes part and worker i
// gets task C + t*W + rank_i.  Every worker's tasks come in increasing order, so thread i
// links its own list (head, next) exactly as the reference's append sequence leaves it.
__device__ void static_lists_parallel(const PlanLaunch& a, PlanShared& s, int total, int G, int W) {
  const sgld_plan_buffers& p = a.p;
  const int tid = threadIdx.x;
  const bool worker = tid < W;
  int load = 0, tail = -1;
  int* run_start = s.loads;          // [runs + 1] (the serial path's arrays are free here)
  int* rank_of = s.tails;            // [W] position of worker i in (rho, i) order
  int* pos = s.tails + 1024;         // [W] position among this round's participants
  int* rho_s = s.tails + 2048;       // [W]
  int* q_s = s.tails + 3072;         // [W]
  // Run boundaries over the sorted positions (four contiguous positions per thread).
  int flags = 0;
  for (int k = 0; k < 4; ++k) {
    const int idx = tid * 4 + k;
    if (idx < total) {
      const unsigned wk = static_cast<unsigned>(s.keys[idx] >> 32);
      flags += (idx == 0 || wk != static_cast<unsigned>(s.keys[idx - 1] >> 32)) ? 1 : 0;
    }
  }
  int runs = 0;
  int rb = block_exclusive_scan(flags, s, runs);
  for (int k = 0; k < 4; ++k) {
    const int idx = tid * 4 + k;
    if (idx < total && (idx == 0 || static_cast<unsigned>(s.keys[idx] >> 32) !=
                                        static_cast<unsigned>(s.keys[idx - 1] >> 32)))
      run_start[rb++] = idx;
  }
  if (tid == 0) run_start[runs] = total;
  __syncthreads();
  for (int r = 0; r < runs; ++r) {
    const int rs = run_start[r], re = run_start[r + 1];
    const int w = kIntMax - static_cast<int>(s.keys[rs] >> 32);
    const int k = (re - rs) * G;                       // tasks in this run
    const int v0 = block_reduce_min(worker ? load : kIntMax, s);
    int q = 0, rho = 0;
    if (worker) {
      q = (load - v0) / w;
      rho = (load - v0) - q * w;
      q_s[tid] = q;
      rho_s[tid] = rho;
    }
    const int qmax = block_reduce_max(worker ? q : 0, s);   // also publishes q_s / rho_s
    int rank = 0;
    if (worker) {
      for (int j = 0; j < W; ++j) {
        const int rj = rho_s[j];
        rank += (rj < rho || (rj == rho && j < tid)) ? 1 : 0;
      }
      rank_of[rank] = tid;                             // rank -> worker
    }
    __syncthreads();
    int assigned = 0, c = 0;
    auto take = [&](int j) {                           // task j of the run goes to this worker
      const int rec = static_cast<int>(s.keys[rs + j / G] & 0xffffffffu);
      const int task = rec * G + j % G;
      if (tail < 0) p.static_head[tid] = task;
      else p.static_next[tail] = task;
      p.static_next[task] = -1;
      tail = task;
      ++assigned;
    };
    for (int round = 0; round < qmax && c < k; ++round) {
      // flag of the worker at sorted position tid, scanned in (rho, i) order
      const int at = tid < W ? rank_of[tid] : 0;
      const int flag = (tid < W && q_s[at] <= round) ? 1 : 0;
      int n = 0;
      const int before = block_exclusive_scan(flag, s, n);
      if (flag) pos[at] = before;
      __syncthreads();
      if (worker && q <= round && c + pos[tid] < k) take(c + pos[tid]);
      c += n;
      __syncthreads();
    }
    if (worker) {
      for (int j = c + rank; j < k; j += W) take(j);
      load += assigned * w;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads, 1) plan_kernel(PlanLaunch a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PlanShared& s = *reinterpret_cast<PlanShared*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const sgld_plan_buffers& p = a.p;
  const int bcap = a.bcap, G = a.groups, W = a.workers;
  // The decode launched after this plan may start its prologue now (programmatic
  // dependent launch); it waits for this grid's completion before reading the plan.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---------------------------------------------------------------- 1. count_scan
  const int active = *p.active;
  const int rows_per_thread = (bcap + kThreads - 1) / kThreads;   // <= 4 (Bcap <= 4096)
  int n_local[4] = {0, 0, 0, 0};
  bool invalid_any = false;
  for (int i = 0; i < rows_per_thread; ++i) {
    const int r = tid * rows_per_thread + i;
    if (r >= bcap) break;
    const bool live = r < active;
    const int len = live ? p.lengths[r] : 0;
    const int spl = live ? p.splits[r] : 1;
    const bool invalid = live && (len < 0 || len > a.maxctx || spl < 1 || spl > a.smax);
    invalid_any |= invalid;
    const int chunk = wrap32(static_cast<long long>(cdiv32(cdiv32(max(len, 0), max(spl, 1)), kSplitAlign)) * kSplitAlign);
    p.chunk[r] = chunk;
    n_local[i] = (live && !invalid) ? cdiv32(len, max(chunk, 1)) : 0;
  }
  const bool error = (active < 0) || (active > bcap) || __syncthreads_or(invalid_any);
  int local_sum = 0;
  for (int i = 0; i < rows_per_thread; ++i) {
    if (error) n_local[i] = 0;
    local_sum += n_local[i];
  }
  int total = 0;
  int base = block_exclusive_scan(local_sum, s, total);
  for (int i = 0; i < rows_per_thread; ++i) {
    const int r = tid * rows_per_thread + i;
    if (r >= bcap) break;
    p.counts[r] = n_local[i];
    p.offsets[r] = base;
    base += n_local[i];
  }
  if (tid == 0) {
    p.offsets[bcap] = total;
    *p.record_count = total;
    *p.error = error ? 1 : 0;
  }
  for (int i = tid; i < a.n_counters; i += kThreads) a.counters[i] = 0;

  if (a.force == 0) {   // builder.py:11-14 -- R0 plans stop after count/scan
    if (tid == 0) {
      *p.mode = 0;
      *p.num_packs = 0;
    }
    return;
  }
  __syncthreads();   // counts/offsets/chunk visible block-wide

  // ---------------------------------------------------------------- 2. emit_records
  for (int r = tid; r < bcap; r += kThreads) {
    const int n = min(p.counts[r], a.smax);
    const int off = p.offsets[r], chunk = p.chunk[r], len = p.lengths[r];
    for (int sp = 0; sp < n; ++sp) {
      const int i = off + sp;
      const int b = sp * chunk;
      const int e = min(b + chunk, len);
      const int w = cdiv32(e - b, kBlockKV);
      p.request[i] = r;
      p.split[i] = sp;
      p.begin[i] = b;
      p.end[i] = e;
      p.weight[i] = w;
      s.weight[i] = w;
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- 3. mode
  int vmax = 1, vmin = kIntMax;
  for (int i = tid; i < total; i += kThreads) {
    vmax = max(vmax, s.weight[i]);
    vmin = min(vmin, s.weight[i]);
  }
  const int max_w = block_reduce_max(vmax, s);
  const int min_w = block_reduce_min(vmin, s);
  if (tid == 0) {
    const int ratio = max_w * 100 / max(min_w, 1);
    const int tasks = total * G;
    int mode = 1;
    for (int row = 0; row < a.n_rules; ++row) {
      const int* r = a.rules + row * 5;
      if (tasks >= r[0] && tasks <= r[1] && ratio >= r[2] && ratio <= r[3]) mode = r[4];
    }
    if (max_w == min_w) mode = 1;
    if (a.force >= 0) mode = a.force;
    s.scalars[0] = mode;
    *p.mode = mode;
  }
  __syncthreads();
  const int mode = s.scalars[0];

  if (mode == 0 || mode == 1) {
    for (int i = tid; i < total; i += kThreads) p.order[i] = i;
    if (tid == 0) *p.num_packs = 0;
    return;
  }

  // ---------------------------------------------------------------- 3b. stable bucket order
  const int buckets = a.buckets;
  if (tid < kMaxBuckets) {
    s.bucket_count[tid] = 0;
    s.bucket_running[tid] = 0;
  }
  __syncthreads();
  for (int i = tid; i < total; i += kThreads) atomicAdd(&s.bucket_count[bucket_of(s.weight[i], buckets)], 1);
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int b = buckets - 1; b >= 0; --b) {   // heavy buckets first
      s.bucket_base[b] = acc;
      acc += s.bucket_count[b];
    }
  }
  for (int round = 0; round * kThreads < total; ++round) {
    const int i = round * kThreads + tid;
    const bool valid = i < total;
    const int b = valid ? bucket_of(s.weight[i], buckets) : kMaxBuckets;   // sentinel bucket
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    s.round_hist[tid >> 5][tid & 31] = 0;
    __syncthreads();
    if (valid && rank_in_warp == 0) s.round_hist[warp][b] = __popc(peers);
    __syncthreads();
    {   // thread (bucket bb, warp ww): exclusive prefix over warps
      const int bb = tid >> 5, ww = tid & 31;
      int acc = 0;
      for (int k = 0; k < ww; ++k) acc += s.round_hist[k][bb];
      s.round_prefix[ww][bb] = acc;
    }
    __syncthreads();
    if (valid) p.order[s.bucket_base[b] + s.bucket_running[b] + s.round_prefix[warp][b] + rank_in_warp] = i;
    __syncthreads();
    if (tid < kMaxBuckets) s.bucket_running[tid] += s.round_prefix[31][tid] + s.round_hist[31][tid];
    __syncthreads();
  }

  // ---------------------------------------------------------------- 3c. pack descriptors
  if (tid == 0) {
    int record_base = 0, pack_base = 0;
    for (int b = buckets - 1; b >= 0; --b) {
      const int size = s.bucket_count[b];
      const int tasks = size * G;
      const int width = (mode == 4) ? min(4, max(1, max_w >> b)) : 1;
      const int packed_tasks = max(0, tasks - W) / width * width;
      const int packed_packs = packed_tasks / width;
      const int pack_count = packed_packs + tasks - packed_tasks;
      s.pk_pack_base[b] = pack_base;
      s.pk_record_base[b] = record_base;
      s.pk_width[b] = width;
      s.pk_ptasks[b] = packed_tasks;
      s.pk_ppacks[b] = packed_packs;
      s.pk_count[b] = pack_count;
      record_base += size;
      pack_base += pack_count;
    }
    s.scalars[1] = pack_base;
    *p.num_packs = pack_base;
  }
  __syncthreads();
  const int num_packs = s.scalars[1];
  for (int pk = tid; pk < num_packs; pk += kThreads) {
    int b = buckets - 1;
    while (b > 0 && pk >= s.pk_pack_base[b] + s.pk_count[b]) --b;
    const int q = pk - s.pk_pack_base[b];
    const int ppacks = s.pk_ppacks[b], width = s.pk_width[b];
    p.pack_first[pk] = s.pk_record_base[b] * G + (q < ppacks ? q * width : s.pk_ptasks[b] + q - ppacks);
    p.pack_count[pk] = q < ppacks ? width : 1;
  }
  if (mode != 2) return;

  // ---------------------------------------------------------------- 4. STATIC LPT lists
  int n2 = 1;
  while (n2 < total) n2 <<= 1;
  for (int i = tid; i < n2; i += kThreads) {
    s.keys[i] = i < total ? (static_cast<unsigned long long>(kIntMax - s.weight[i]) << 32) | static_cast<unsigned>(i)
                          : ~0ull;
  }
  for (int i = tid; i < W; i += kThreads) {
    s.loads[i] = 0;
    s.tails[i] = -1;
    p.static_head[i] = -1;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = s.keys[i], y = s.keys[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            s.keys[i] = y;
            s.keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  if (W <= kThreads) {
    static_lists_parallel(a, s, total, G, W);
    return;
  }
  // More workers than threads: one warp runs the LPT task by task.
  if (warp != 0) return;
  for (int idx = 0; idx < total; ++idx) {
    const int rec = static_cast<int>(s.keys[idx] & 0xffffffffu);
    const int w = s.weight[rec];
    for (int g = 0; g < G; ++g) {
      const int task = rec * G + g;
      int best_load = kIntMax, best_id = kIntMax;
      for (int wk = lane; wk < W; wk += 32) {
        const int l = s.loads[wk];
        if (l < best_load) {
          best_load = l;
          best_id = wk;
        }
      }
      const unsigned min_load = __reduce_min_sync(0xffffffffu, static_cast<unsigned>(best_load));
      const unsigned owner = __reduce_min_sync(
          0xffffffffu, static_cast<unsigned>(best_load) == min_load ? static_cast<unsigned>(best_id) : 0xffffffffu);
      if (lane == static_cast<int>(owner & 31u)) {
        const int tail = s.tails[owner];
        if (tail < 0) p.static_head[owner] = task;
        else p.static_next[tail] = task;
        p.static_next[task] = -1;
        s.tails[owner] = task;
        s.loads[owner] += w;
      }
      __syncwarp();
    }
  }
}

}  // namespace

cudaError_t launch_plan(const PlanLaunch& a, cudaStream_t stream) {
  static bool configured = false;
  const int smem = static_cast<int>(sizeof(PlanShared));
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  plan_kernel<<<1, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace sgld
