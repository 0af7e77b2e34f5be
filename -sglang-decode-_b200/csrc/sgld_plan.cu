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
// The kernel is latency bound (kilobytes of metadata), so it is written to need few
// block barriers: reductions and scans take one barrier each (double-buffered warp
// partials), records are emitted one per thread with coalesced stores, the bucket
// order is one counting pass (each warp owns 128 consecutive records), and the STATIC
// lists are built run by run (runs of equal weight, heaviest first) without sorting.
#include <cuda_runtime.h>

#include <mutex>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kPerThread = kMaxRecords / kThreads;   // 4 consecutive records per thread
constexpr int kIntMax = 0x7fffffff;
constexpr int kMaxTableWeight = 4096;              // run table of STATIC up to this weight
static_assert(kMaxBuckets == kWarps, "one warp scans one bucket column");
static_assert(kMaxRecords == kWarps * 128, "each warp orders 128 consecutive records");

__device__ __forceinline__ int32_t wrap32(long long x) { return static_cast<int32_t>(static_cast<uint32_t>(x)); }

// floor division of an int32 by a positive int32 (Triton int32 cdiv on wrapped sums).
__device__ __forceinline__ int32_t floordiv(int32_t a, int32_t b) {
  return a >= 0 ? a / b : -static_cast<int32_t>((-static_cast<long long>(a) + b - 1) / b);
}

__device__ __forceinline__ int32_t cdiv32(int32_t a, int32_t b) { return floordiv(wrap32(static_cast<long long>(a) + b - 1), b); }

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

struct PlanShared {
  int32_t part_a[2][kWarps];          // warp partials of the one-barrier reductions / scans
  int32_t part_b[2][kWarps];
  int32_t part_c[2][kWarps];
  int32_t cnt[kWarps][kMaxBuckets];   // per-warp bucket counts, then (bucket, warp) prefixes
  int32_t bucket_count[kMaxBuckets];
  int32_t weight[kMaxRecords];
  int32_t hist[kMaxTableWeight + 1];  // records per weight (weights <= kMaxTableWeight)
  union {
    struct {                          // per-request inputs of emit_records
      int32_t off[kMaxRecords + 1];
      int32_t chunk[kMaxRecords];
      int32_t len[kMaxRecords];
    } req;
    struct {                          // STATIC with more workers than threads (serial LPT)
      unsigned long long keys[kMaxRecords];
      int32_t loads[kMaxPlanWorkers];
      int32_t tails[kMaxPlanWorkers];
    } serial;
    int32_t run_w[kMaxRecords];       // STATIC: run weights, heaviest first
  };
  // STATIC run state (W <= 1024), indexed by worker
  int32_t run_rec[kMaxRecords];       // records of the current run, ascending
  unsigned skey32[kThreads];          // holder warps' keys, each warp's 32 sorted ascending
  unsigned long long skey64[kThreads];
  int32_t q[kThreads];
  int32_t rank_of[kThreads];
  int32_t load[kThreads];
  int32_t tail[kThreads];
  int32_t head[kThreads];
};

// Block-wide collectives with one barrier each.  Successive calls alternate between two
// partial buffers; a buffer is rewritten only two calls later, after every thread has
// passed the barrier of the call in between, so no second barrier is needed.  Every
// thread of the block must make the same sequence of calls.
struct Block {
  PlanShared& s;
  int parity = 0;

  __device__ explicit Block(PlanShared& sh) : s(sh) {}

  // (max of a, min of b) over the block.
  __device__ void max_min(int a, int b, int& amax, int& bmin) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    a = __reduce_max_sync(0xffffffffu, a);
    b = __reduce_min_sync(0xffffffffu, b);
    if (lane == 0) {
      s.part_a[parity][warp] = a;
      s.part_b[parity][warp] = b;
    }
    __syncthreads();
    amax = __reduce_max_sync(0xffffffffu, s.part_a[parity][lane]);
    bmin = __reduce_min_sync(0xffffffffu, s.part_b[parity][lane]);
    parity ^= 1;
  }

  // Exclusive scan of v in thread order (returned), its total, the max of mx, the min of mn.
  __device__ int scan_max_min(int v, int mx, int mn, int& total, int& mxo, int& mno) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    mn = __reduce_min_sync(0xffffffffu, mn);
    if (lane == 31) s.part_a[parity][warp] = x;
    if (lane == 0) {
      s.part_b[parity][warp] = mx;
      s.part_c[parity][warp] = mn;
    }
    __syncthreads();
    const int part = s.part_a[parity][lane];
    total = __reduce_add_sync(0xffffffffu, part);
    const int before = __reduce_add_sync(0xffffffffu, lane < warp ? part : 0);
    mxo = __reduce_max_sync(0xffffffffu, s.part_b[parity][lane]);
    mno = __reduce_min_sync(0xffffffffu, s.part_c[parity][lane]);
    parity ^= 1;
    return before + x - v;
  }

  // Exclusive scan of v in thread order (returned), its total, and the max of m.
  __device__ int scan_max(int v, int m, int& total, int& mmax) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 31) s.part_a[parity][warp] = x;
    if (lane == 0) s.part_b[parity][warp] = m;
    __syncthreads();
    const int part = s.part_a[parity][lane];
    total = __reduce_add_sync(0xffffffffu, part);
    const int before = __reduce_add_sync(0xffffffffu, lane < warp ? part : 0);
    mmax = __reduce_max_sync(0xffffffffu, s.part_b[parity][lane]);
    parity ^= 1;
    return before + x - v;
  }
};

// Saturating integer ceil-log2 exactly as kernels/plan.py:77-79 computes it.
__device__ __forceinline__ int bucket_of(int w, int buckets) {
  int b = 0;
  for (int k = 1; k < buckets; ++k) b += (w > (1 << (k - 1))) ? 1 : 0;
  return b;
}

// Suffix-exclusive sum over the lanes of a warp: lane l gets the sum of x over lanes > l.
__device__ __forceinline__ int suffix_exclusive(int x, int& total) {
  const int lane = threadIdx.x & 31;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += y;
  }
  total = __shfl_sync(0xffffffffu, incl, 0);
  return incl - x;
}

// Bitonic sort of one key per lane, ascending in lane order.
template <typename Key>
__device__ __forceinline__ Key warp_sort(Key x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const Key y = __shfl_xor_sync(0xffffffffu, x, j);
      const bool keep_min = ((lane & j) == 0) == ((lane & k) == 0);
      x = keep_min ? (x < y ? x : y) : (x < y ? y : x);
    }
  }
  return x;
}

// Number of entries below x in 32 ascending keys.
template <typename Key>
__device__ __forceinline__ int lower_bound32(const Key* a, Key x) {
  int pos = 0;
#pragma unroll
  for (int step = 16; step > 0; step >>= 1) pos += a[pos + step - 1] < x ? step : 0;
  return pos + (a[pos] < x ? 1 : 0);
}

// Exact LPT lists (kernels/plan.py:103-135), W <= 1024 workers.
//
// The reference hands tasks out one at a time, heaviest record first (record id, then
// group, ascending among equal weights), each to the least-loaded worker, lowest worker
// id on ties.  Records of one weight w form a run of k = n*G consecutive tasks.  Handing
// out a run equals taking the k smallest "slots" (L_i + m*w, i), m >= 0, in that order.
// Writing L_i = q_i*w + rho_i (0 <= rho_i < w), slot (i, m) has value (q_i + m)*w + rho_i,
// so slots are ordered by (round, rho_i, i) with round = q_i + m: each round takes its
// participants (q_i <= round) in (rho_i, i) order.  Rounds from min q to max q - 1 scan
// the participant flags (one barrier each); from max q on every worker takes part and
// the worker of rank t gets tasks C + t + m*W, whose links are written task-parallel
// (next[task(j)] = task(j + W)).  Each next[] entry is written exactly once; a worker's
// last task gets -1 at the end.
//
// Run weights come from the weight histogram (heaviest first) when every weight is at
// most kMaxTableWeight, else from a max reduction per run.  The thread holding worker i
// during a run (the thread of its rank) publishes i's (q, rho) for the next run, so a run
// costs two barriers plus its pre-steady rounds.
template <typename Key>
__device__ void static_lists_runs(const PlanLaunch& a, PlanShared& s, Block& blk, Key* skey, int total, int G,
                                  int W, bool table) {
  const sgld_plan_buffers& p = a.p;
  const int tid = threadIdx.x;
  if (tid < W) {
    s.load[tid] = 0;
    s.tail[tid] = -1;
    s.head[tid] = -1;
  }
  const int lane = tid & 31, warp = tid >> 5;
  const int chunks = (W + 31) >> 5;                  // holder warps
  int nruns = 0;
  if (table) {                                       // distinct weights, heaviest first
    int f = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int v = kMaxTableWeight - (tid * 4 + k);
      f += (v >= 1 && s.hist[v] > 0) ? 1 : 0;
    }
    int unused_max = 0, unused_min = 0;
    int pos = blk.scan_max_min(f, 0, 0, nruns, unused_max, unused_min);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int v = kMaxTableWeight - (tid * 4 + k);
      if (v >= 1 && s.hist[v] > 0) s.run_w[pos++] = v;
    }
    __syncthreads();
  }
  int at = tid, my_load = 0;                         // worker held by this thread, its load
  int prev_w = kIntMax, consumed = 0;
  for (int r = 0; consumed < total; ++r) {
    int w = 0;
    if (table) {
      w = s.run_w[r];
    } else {
      int wl = 0, unused = 0;
#pragma unroll
      for (int k = 0; k < kPerThread; ++k) {
        const int i = tid * kPerThread + k;
        if (i < total && s.weight[i] < prev_w) wl = max(wl, s.weight[i]);
      }
      blk.max_min(wl, 0, w, unused);
    }
    // B. the run's records (ascending) and the held worker's (q, rho).
    int f = 0;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int i = tid * kPerThread + k;
      f += (i < total && s.weight[i] == w) ? 1 : 0;
    }
    int q = 0;
    Key key = static_cast<Key>(~static_cast<Key>(0));   // (rho, worker); padding sorts last
    if (tid < W) {
      q = my_load / w;
      const int rho = my_load - q * w;
      s.q[at] = q;
      if constexpr (sizeof(Key) == 4) key = static_cast<unsigned>(rho) * 1024u + static_cast<unsigned>(at);
      else key = (static_cast<unsigned long long>(rho) << 32) | static_cast<unsigned>(at);
    }
    if (warp < chunks) {                             // each holder warp sorts its own keys
      key = warp_sort(key);
      skey[tid] = key;
    }
    int nrun = 0, qmax = 0, qmin = 0;
    int at_run = blk.scan_max_min(f, tid < W ? q : 0, tid < W ? q : kIntMax, nrun, qmax, qmin);
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int i = tid * kPerThread + k;
      if (i < total && s.weight[i] == w) s.run_rec[at_run++] = i;
    }
    if (warp < chunks && key != static_cast<Key>(~static_cast<Key>(0))) {
      int rank = lane;                               // rank of the key this lane holds after the sort
      for (int c = 0; c < chunks; ++c)
        if (c != warp) rank += lower_bound32(skey + c * 32, key);
      s.rank_of[rank] = static_cast<int>(key & static_cast<Key>(sizeof(Key) == 4 ? 1023u : 0xffffffffu));
    }
    __syncthreads();
    // C. thread t holds the worker of rank t for the rest of the run.
    const int k = nrun * G;
    int qa = kIntMax, tail = -1, head = -1, assigned = 0;
    if (tid < W) {
      at = s.rank_of[tid];
      qa = s.q[at];
      tail = s.tail[at];
      head = s.head[at];
      my_load = s.load[at];
    }
    auto task_of = [&](int j) { return s.run_rec[j / G] * G + j % G; };
    auto take = [&](int j) {
      const int t = task_of(j);
      if (tail < 0) head = t;
      else p.static_next[tail] = t;
      tail = t;
      ++assigned;
    };
    int c = 0;
    for (int round = qmin; round < qmax && c < k; ++round) {
      const int flag = (tid < W && qa <= round) ? 1 : 0;
      int n = 0, unused_max = 0, unused_min = 0;
      const int pos = blk.scan_max_min(flag, 0, 0, n, unused_max, unused_min);
      if (flag && c + pos < k) take(c + pos);
      c += n;
    }
    // D. steady rounds: rank t takes c + t, c + t + W, ...
    if (tid < W && c + tid < k) {
      const int j0 = c + tid;
      const int m = (k - 1 - j0) / W;
      take(j0);
      tail = task_of(j0 + m * W);
      assigned += m;
    }
    if (c + tid + W < k) {                           // next[task(j)] = task(j + W), task-parallel
      int j = c + tid;
      int pos = j / G, g = j - pos * G;              // task(j) = run_rec[pos] * G + g
      int pos2 = (j + W) / G, g2 = j + W - pos2 * G;
      const int step_q = kThreads / G, step_r = kThreads - step_q * G;
      for (; j + W < k; j += kThreads) {
        p.static_next[s.run_rec[pos] * G + g] = s.run_rec[pos2] * G + g2;
        pos += step_q;
        g += step_r;
        if (g >= G) {
          g -= G;
          ++pos;
        }
        pos2 += step_q;
        g2 += step_r;
        if (g2 >= G) {
          g2 -= G;
          ++pos2;
        }
      }
    }
    // E. the held worker's state, read by its next holder after the next run's barriers.
    if (tid < W) {
      my_load += assigned * w;
      s.load[at] = my_load;
      s.tail[at] = tail;
      s.head[at] = head;
    }
    consumed += nrun;
    prev_w = w;
  }
  __syncthreads();
  if (tid < W) {
    p.static_head[tid] = s.head[tid];
    if (s.tail[tid] >= 0) p.static_next[s.tail[tid]] = -1;
  }
}

// STATIC with more workers than threads: bitonic sort of (weight desc, record asc) keys,
// then one warp runs the reference's LPT task by task (warp argmin, lowest id on ties).
__device__ void static_lists_serial(const PlanLaunch& a, PlanShared& s, int total, int G, int W) {
  const sgld_plan_buffers& p = a.p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int n2 = 1;
  while (n2 < total) n2 <<= 1;
  for (int i = tid; i < n2; i += kThreads) {
    s.serial.keys[i] = i < total ? (static_cast<unsigned long long>(kIntMax - s.weight[i]) << 32) | static_cast<unsigned>(i)
                                 : ~0ull;
  }
  for (int i = tid; i < W; i += kThreads) {
    s.serial.loads[i] = 0;
    s.serial.tails[i] = -1;
    p.static_head[i] = -1;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = s.serial.keys[i], y = s.serial.keys[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            s.serial.keys[i] = y;
            s.serial.keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  if (warp != 0) return;
  for (int idx = 0; idx < total; ++idx) {
    const int rec = static_cast<int>(s.serial.keys[idx] & 0xffffffffu);
    const int w = s.weight[rec];
    for (int g = 0; g < G; ++g) {
      const int task = rec * G + g;
      int best_load = kIntMax, best_id = kIntMax;
      for (int wk = lane; wk < W; wk += 32) {
        const int l = s.serial.loads[wk];
        if (l < best_load) {
          best_load = l;
          best_id = wk;
        }
      }
      const unsigned min_load = __reduce_min_sync(0xffffffffu, static_cast<unsigned>(best_load));
      const unsigned owner = __reduce_min_sync(
          0xffffffffu, static_cast<unsigned>(best_load) == min_load ? static_cast<unsigned>(best_id) : 0xffffffffu);
      if (lane == static_cast<int>(owner & 31u)) {
        const int tail = s.serial.tails[owner];
        if (tail < 0) p.static_head[owner] = task;
        else p.static_next[tail] = task;
        p.static_next[task] = -1;
        s.serial.tails[owner] = task;
        s.serial.loads[owner] += w;
      }
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) plan_kernel(PlanLaunch a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PlanShared& s = *reinterpret_cast<PlanShared*>(smem_raw);
  Block blk(s);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const sgld_plan_buffers& p = a.p;
  const int bcap = a.bcap, G = a.groups, W = a.workers;
  // The inputs read first (active count, lengths, split hints) are plan buffers of the
  // geometry's size, written before this launch.  Warming their sectors in L2 while the
  // preceding kernel drains takes an HBM round trip off those loads; a prefetch is only a
  // hint, and the loads after the wait below read the current values.
  {
    const int sectors = (bcap + 7) >> 3;             // 8 int32 per 32-byte sector
    for (int j = tid; j <= 2 * sectors; j += kThreads) {
      const int32_t* src = j == 2 * sectors ? p.active
                           : j < sectors    ? p.lengths + min(j * 8, bcap - 1)
                                            : p.splits + min((j - sectors) * 8, bcap - 1);
      prefetch_l2(src);
    }
  }
  // Launched as a programmatic dependent of the preceding kernel (the previous step's
  // merge, which still reads counts / error): the block is resident early, and waits here
  // for that kernel's completion before reading its inputs or writing any plan buffer.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The decode launched after this plan may start its prologue now (programmatic
  // dependent launch); it waits for this grid's completion before reading the plan.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---------------------------------------------------------------- 1. count_scan
  const int active = *p.active;
  const int rows_per_thread = (bcap + kThreads - 1) / kThreads;   // <= 4 (Bcap <= 4096)
  int n_local[4] = {0, 0, 0, 0};
  int local_sum = 0, invalid_any = 0;
  for (int i = 0; i < rows_per_thread; ++i) {
    const int r = tid * rows_per_thread + i;
    if (r >= bcap) break;
    // Loaded whatever `active` is (every row of the capacity is allocated), so these loads
    // and the load of `active` share one round trip.
    const int len_in = p.lengths[r], spl_in = p.splits[r];
    const bool live = r < active;
    const int len = live ? len_in : 0;
    const int spl = live ? spl_in : 1;
    const bool invalid = live && (len < 0 || len > a.maxctx || spl < 1 || spl > a.smax);
    invalid_any |= invalid ? 1 : 0;
    const int chunk = wrap32(static_cast<long long>(cdiv32(cdiv32(max(len, 0), max(spl, 1)), kSplitAlign)) * kSplitAlign);
    p.chunk[r] = chunk;
    s.req.chunk[r] = chunk;
    s.req.len[r] = len;
    n_local[i] = (live && !invalid) ? cdiv32(len, max(chunk, 1)) : 0;
    local_sum += n_local[i];
  }
  s.cnt[warp][lane] = 0;                             // bucket counters, used in step 3b
  for (int v = tid; v <= kMaxTableWeight; v += kThreads) s.hist[v] = 0;
  int total = 0, any_invalid = 0;
  int base = blk.scan_max(local_sum, invalid_any, total, any_invalid);
  const bool error = (active < 0) || (active > bcap) || any_invalid != 0;
  if (error) {                                       // no records at all (plan.py:16-20)
    total = 0;
    base = 0;
  }
  for (int i = 0; i < rows_per_thread; ++i) {
    const int r = tid * rows_per_thread + i;
    if (r >= bcap) break;
    const int n = error ? 0 : n_local[i];
    p.counts[r] = n;
    p.offsets[r] = base;
    s.req.off[r] = base;
    base += n;
  }
  if (tid == 0) {
    p.offsets[bcap] = total;
    s.req.off[bcap] = total;
    *p.record_count = total;
    *p.error = error ? 1 : 0;
  }
  for (int i = tid; i < a.n_counters; i += kThreads) a.counters[i] = 0;
  for (int i = tid; i < bcap * a.groups; i += kThreads) p.arrivals[i] = 0;   // fused-merge arrivals

  if (a.force == 0) {   // builder.py:11-14 -- R0 plans stop after count/scan
    if (tid == 0) {
      *p.mode = 0;
      *p.num_packs = 0;
    }
    return;
  }
  __syncthreads();   // per-request offsets / chunk / length visible block-wide

  // ---------------------------------------------------------------- 2. emit_records
  // One record per thread: its request is the last r with off[r] <= i.
  int vmax = 1, vmin = kIntMax;
  for (int i = tid; i < total; i += kThreads) {
    int lo = 0, hi = bcap;                           // off[lo] <= i < off[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s.req.off[mid] <= i) lo = mid;
      else hi = mid;
    }
    const int sp = i - s.req.off[lo];
    const int chunk = s.req.chunk[lo];
    const int b = sp * chunk;
    const int e = min(b + chunk, s.req.len[lo]);
    const int w = cdiv32(e - b, kBlockKV);
    p.request[i] = lo;
    p.split[i] = sp;
    p.begin[i] = b;
    p.end[i] = e;
    p.weight[i] = w;
    p.order[i] = i;                                  // R0/R1 order (the other modes rewrite it)
    s.weight[i] = w;
    vmax = max(vmax, w);
    vmin = min(vmin, w);
  }

  // ---------------------------------------------------------------- 3. mode
  int max_w = 1, min_w = kIntMax;
  blk.max_min(vmax, vmin, max_w, min_w);             // also publishes s.weight
  int mode = 1;
  {
    const int ratio = max_w * 100 / max(min_w, 1);
    const int tasks = total * G;
    for (int row = 0; row < a.n_rules; ++row) {
      const int* r = a.rules + row * 5;
      if (tasks >= r[0] && tasks <= r[1] && ratio >= r[2] && ratio <= r[3]) mode = r[4];
    }
    if (max_w == min_w) mode = 1;
    if (a.force >= 0) mode = a.force;
  }
  if (tid == 0) *p.mode = mode;

  if (mode == 0 || mode == 1) {                      // identity order, written during emission
    if (tid == 0) *p.num_packs = 0;
    return;
  }

  // ---------------------------------------------------------------- 3b. stable bucket order
  // Warp w owns records [128w, 128w + 128) in four passes of 32; within a warp equal
  // buckets are ranked by match_any/popc, across warps by a (bucket, warp) prefix.
  const int buckets = a.buckets;
  int local_off[4], bk[4];
#pragma unroll
  for (int sub = 0; sub < 4; ++sub) {
    const int i = warp * 128 + sub * 32 + lane;
    const bool valid = i < total;
    const int b = valid ? bucket_of(s.weight[i], buckets) : kMaxBuckets;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    const int r = __popc(peers & lanemask_lt());
    const int seen = valid ? s.cnt[warp][b] : 0;
    __syncwarp();
    if (valid && r == 0) s.cnt[warp][b] = seen + __popc(peers);
    __syncwarp();
    local_off[sub] = seen + r;
    bk[sub] = valid ? b : -1;
  }
  __syncthreads();
  if (warp < buckets) {                              // warp b: prefix of bucket b over warps
    const int v = s.cnt[lane][warp];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s.cnt[lane][warp] = incl - v;
    if (lane == 31) s.bucket_count[warp] = incl;
  }
  __syncthreads();
  // Lane l of every warp: bucket l's size, first record position (heavy buckets first),
  // and its pack parameters (plan.py:84-99).
  const int size = lane < buckets ? s.bucket_count[lane] : 0;
  int unused_total = 0;
  const int record_base = suffix_exclusive(size, unused_total);
#pragma unroll
  for (int sub = 0; sub < 4; ++sub) {
    const int b = bk[sub];
    const int rb = __shfl_sync(0xffffffffu, record_base, b < 0 ? 0 : b);
    if (b >= 0) p.order[rb + s.cnt[warp][b] + local_off[sub]] = warp * 128 + sub * 32 + lane;
  }

  // ---------------------------------------------------------------- 3c. pack descriptors
  const int tasks_b = size * G;
  const int width = (mode == 4) ? min(4, max(1, max_w >> lane)) : 1;
  const int ptasks = max(0, tasks_b - W) / width * width;
  const int ppacks = ptasks / width;
  const int count_b = lane < buckets ? ppacks + tasks_b - ptasks : 0;
  int num_packs = 0;
  const int pack_base = suffix_exclusive(count_b, num_packs);
  if (tid == 0) *p.num_packs = num_packs;
  for (int b = buckets - 1; b >= 0; --b) {
    const int pb = __shfl_sync(0xffffffffu, pack_base, b);
    const int cnt = __shfl_sync(0xffffffffu, count_b, b);
    const int pp = __shfl_sync(0xffffffffu, ppacks, b);
    const int wd = __shfl_sync(0xffffffffu, width, b);
    const int pt = __shfl_sync(0xffffffffu, ptasks, b);
    const int rb = __shfl_sync(0xffffffffu, record_base, b);
    for (int qk = tid; qk < cnt; qk += kThreads) {
      p.pack_first[pb + qk] = rb * G + (qk < pp ? qk * wd : pt + qk - pp);
      p.pack_count[pb + qk] = qk < pp ? wd : 1;
    }
  }
  if (mode != 2) return;

  // ---------------------------------------------------------------- 4. STATIC LPT lists
  if (W > kThreads) static_lists_serial(a, s, total, G, W);
  else if (max_w <= kMaxTableWeight) {
    // The weight histogram (run weights of the table path) is only needed here, so it is
    // counted here rather than during emission, which every mode runs.
    for (int i = tid; i < total; i += kThreads) atomicAdd(&s.hist[s.weight[i]], 1);
    __syncthreads();
    static_lists_runs(a, s, blk, s.skey32, total, G, W, true);
  }
  else static_lists_runs(a, s, blk, s.skey64, total, G, W, false);
}

}  // namespace

cudaError_t launch_plan(const PlanLaunch& a, cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  static void* configured[kMaxDevices] = {};   // context the smem attribute was set in
  static std::mutex mu;
  const int smem = static_cast<int>(sizeof(PlanShared));
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    void* ctx = current_context();
    if (ctx == nullptr || configured[device] != ctx) {
      e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      configured[device] = ctx;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, plan_kernel, a);
}

}  // namespace sgld
