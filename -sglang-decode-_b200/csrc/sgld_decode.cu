// Persistent paged GQA decode for sm_100a.
//
// Replaces the reference's persistent_decode + _attention_task
// (kernels/attention.py:12-130) and the per-layer counter memset
// (runtime/engine.py:62).  The split merge (merge.py) is the next launch
// (sgld_merge.cu), chained to this one by programmatic dependent launch.
//
// One CTA per worker (grid = workers).  Warps have fixed roles and are connected by
// shared-memory rings guarded by mbarriers:
//
//   scheduler (1 warp, lane 0)  claims tasks exactly as the reference's claim loop
//        (attention.py:99-130: R0/R1 stride-W round robin, STATIC list walk, D1/D4
//        relaxed atomic per pack), resolves each task to (request, split, kv_head,
//        token range) (attention.py:23-47) and pushes it into the task ring.
//   indexer (1 warp)  turns tasks into 64-token stage descriptors: it gathers the
//        page-table / CSR indices of four stages per round trip, with the next batch's
//        loads in flight while the current batch is written, and stores each token's
//        page, in-page row and K/V row offsets (any strides) in the descriptor ring.
//   producers (P warps)  fill the data ring.  Paged KV with a page_size that is a
//        multiple of 32 moves by tensor-map TMA boxes (64 dims x 32 tokens of one page
//        per instruction); CSR and other layouts move by 16-byte cp.async spread over
//        the P warps (the issue rate of one warp caps its bandwidth).
//        Producer 0 also loads each task's query group into a double-buffered Q slot.
//   consumers (4 or 8 warps)  each take 16 tokens of a stage, a task's stages two at a time
//        where the ring allows (one softmax update per 32 tokens); the fp8 kernel runs two
//        quads of 4 that take alternate iterations of a task.  QK and PV run on tensor
//        cores (mma.sync m16n8k16) in "swapped" form so the GQA group (padded to 8 or
//        16) is the N dimension: S^T = K Q^T and O^T += V^T P^T; movmatrix turns the
//        score accumulator into the P^T operand.  FP32 online softmax state is
//        warp-private; at the end of a task the warp states are combined and
//        the normalised partial and natural-log LSE of every query head of the group
//        are stored to slot (request*Hq + head)*Smax + split (attention.py:81-84).
//
// Shared-memory tiles use the 128-byte swizzle layout [D/64][rows][128 B] (16-byte
// chunk index XOR row%8) that TMA writes natively; ldmatrix reads are bank-conflict
// free.  Rows past a task's last token are masked in registers (scores -inf, V
// fragments zero), so stale shared memory never reaches the result.  Every mbarrier
// wait is bounded; on expiry a status bit is set and the warp unwinds.  The merge
// launched after this kernel leaves the claim counter at zero.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <type_traits>

#include "sgld_internal.cuh"
#include "sgld_merge.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s per wait
constexpr int kSmemBudget = 227 * 1024 - 1024;     // 1 KB slack to align the base to 1024
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum : int { kFlagFirst = 1, kFlagLast = 2, kFlagExit = 4 };
enum : int { kStatusWaitFull = 1, kStatusWaitEmpty = 2, kStatusWaitQ = 4, kStatusWaitTask = 8,
             kStatusStaticCycle = 16, kStatusWaitDesc = 32, kStatusQRows = 64 };

struct StageHdr {
  int request, split, group, ntok, flags, t0, pad[2];
};

struct TaskDesc {
  int request, split, group, begin, end, base, valid, pad;
};

template <int D, int NT, bool F8 = false>
struct Cfg {
  static constexpr bool kBig = D * NT >= 512;            // D=256 with a 16-row group
  // Consumer quads: four warps each take 16 rows of a stage.  A single quad is one
  // latency-bound warp per SM sub-partition.  The fp8 kernel (group <= 8), whose consumers
  // also widen every K/V byte, runs two quads that take alternate iterations of a task
  // (measured on B200: C3 946 -> 758 us).  The 16-bit kernels stay at one quad: with two,
  // they lose the paired stages (the ring has no stage to spare) and ran 5% slower.
  static constexpr int kQuads = (F8 && NT == 1) ? 2 : 1;
  static constexpr int kConsumerWarps = 4 * kQuads;
  // One warp's cp.async issue rate caps its bandwidth, so the copies are spread over
  // as many producer warps as the register file allows next to the consumers (16 warps
  // at 128 registers for D <= 128 and a group of at most 8).  With tensor-map copies
  // producer 0 works alone.
  // fp8 stages carry half the bytes: 6 producers keep the CTA at 16 warps (at most four per
  // SM sub-partition), hence 128 registers a thread for the widening consumers.
  static constexpr int kProducerWarps = kBig ? 2 : (NT == 2 ? 5 : (D >= 256 ? 6 : (F8 ? 6 : 10)));
  static constexpr int kProducerWarp0 = kConsumerWarps;
  static constexpr int kIndexerWarp = kProducerWarp0 + kProducerWarps;
  static constexpr int kSchedulerWarp = kIndexerWarp + 1;
  static constexpr int kWarps = kSchedulerWarp + 1;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kConsumerThreads = kConsumerWarps * 32;
  static constexpr int kTS = 64;                         // tokens per stage
  static constexpr int kKVBytes = F8 ? 1 : 2;            // bytes per K/V element (e4m3 or 16-bit)
  static constexpr int kRowBytes = D * kKVBytes;
  static constexpr int kChunks = kRowBytes / 16;         // 16-byte chunks per K/V row
  static constexpr int kEPC = 16 / kKVBytes;             // K/V elements per 16-byte chunk
  static constexpr int kQChunks = D / 8;                 // Q is 16-bit in shared memory
  static constexpr int kTPI = (32 / kChunks) > 0 ? 32 / kChunks : 1;  // tokens per warp copy
  static constexpr int kTileBytes = kTS * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kQRows = NT * 8;
  static constexpr int kQBytes = kQRows * D * 2;
  static constexpr int kRedStride = D + 4;               // floats; padding avoids bank conflicts
  static constexpr int kRedOne = kConsumerWarps * kQRows * kRedStride * 4;
  static constexpr int kTaskQ = 4;
  static constexpr int kSD = kBig ? 6 : 12;              // stage-descriptor ring depth
  static constexpr int kNB = 4;                          // stages indexed per round trip
  static constexpr int kSDEntry = kTS * 24;              // koff, voff (int64), page, row (int32)
  static constexpr int kSDBytes = kSD * kSDEntry;
  static constexpr int kMiscBytes = 4096;
  static constexpr int kFixed1 = 2 * kQBytes + kSDBytes + kMiscBytes;
  // Double-buffered reduction when it leaves enough stages (two quads hold two stages).
  static constexpr int kRedBufs = (kFixed1 + 2 * kRedOne + (kQuads == 2 ? 5 : 3) * kStageBytes <= kSmemBudget) ? 2 : 1;
  static constexpr int kFixed = kFixed1 + kRedBufs * kRedOne;
  static constexpr int kStagesRaw = (kSmemBudget - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  // Consumers hold two stages at a time (paired stages) when the ring is deep enough (each
  // quad holds two and as many stay in flight); the 16-row-group kernels have no registers
  // to spare for the second sub-tile.
  static constexpr bool kPair = kStages >= 4 * kQuads && NT == 1;
  static_assert(kStages >= 2, "shared memory budget too small");
  // Offsets from the 1024-byte aligned base (tiles first: they need the alignment).
  static constexpr int kOffQ = kStages * kStageBytes;
  static constexpr int kOffRed = kOffQ + 2 * kQBytes;
  static constexpr int kOffSD = kOffRed + kRedBufs * kRedOne;
  static constexpr int kOffMisc = kOffSD + kSDBytes;
  static constexpr int kSmemUsed = kOffMisc + kMiscBytes;
  static constexpr int kSmemBytes = kSmemUsed + 1024;    // launch size including alignment slack
  static_assert(kSmemUsed <= kSmemBudget, "shared memory budget exceeded");
  static_assert(kTileBytes % 1024 == 0 && kQBytes % 1024 == 0,
                "tiles must keep 1024-byte alignment");
};

// Barriers, ring headers and the per-warp softmax statistics of the epilogue.
struct Misc {
  uint64_t full[8], empty[8], qfull[2], qempty[2], tfull[4], tempty[4], sfull[12], sempty[12], join[2],
      drain;
  StageHdr hdr[8];
  StageHdr shdr[12];
  TaskDesc tq[4];
  float m[2][8][16], l[2][8][16];   // per consumer warp (up to two quads)
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile of ROWS rows laid out
// [D/64][ROWS][128 B] with the 128-byte swizzle (chunk bits 0-2 XOR row bits 0-2).
template <int ROWS>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return static_cast<uint32_t>(((chunk >> 3) * ROWS + row) * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Bounded wait that also reconverges the warp (the callers run warp-collective code next).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_wait(bar, parity, global_timer_ns() + kWaitLimitNs);
  __syncwarp();
  if (!ok && (threadIdx.x & 31) == 0) atomicOr(status, code);
  return ok;
}

// Bounded join of the four consumer warps on an mbarrier (count 4, one arrival per
// warp); unlike a named barrier it cannot hang if a warp has unwound after a timeout.
__device__ __forceinline__ bool consumer_join(uint64_t* bar, uint32_t parity, int* status) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  return warp_wait(bar, parity, status, kStatusWaitFull);
}

template <typename T, int D, int NT, bool F8 = false>
struct Kernel {
  using C = Cfg<D, NT, F8>;
  // With fp8 K/V the MMAs run in f16 (every e4m3 value is exact in f16; a bf16 Q is converted
  // on load); otherwise in the Q dtype.
  using MT = typename std::conditional<F8, __half, T>::type;
  using KVT = typename std::conditional<F8, uint8_t, T>::type;
  static_assert(sizeof(Misc) <= C::kMiscBytes, "misc area too small");

  // ------------------------------------------------------------------ scheduler (lane 0)
  __device__ static bool push_task(Misc& ms, int& ti, uint32_t& tph, const TaskDesc& t, int* status) {
    if (!mbar_wait(&ms.tempty[ti], tph ^ 1u, global_timer_ns() + kWaitLimitNs)) {
      atomicOr(status, kStatusWaitTask);
      return false;
    }
    ms.tq[ti] = t;
    mbar_arrive(&ms.tfull[ti]);
    if (++ti == C::kTaskQ) {
      ti = 0;
      tph ^= 1u;
    }
    return true;
  }

  __device__ static void prefetch_q(const DecodeLaunch& a, const TaskDesc& t) {
    const int gs = a.group_size;
    const T* row0 = static_cast<const T*>(a.d.q) + static_cast<int64_t>(t.request) * a.d.q_stride[0] +
                    static_cast<int64_t>(t.group * gs) * a.d.q_stride[1];
    if (a.d.q_stride[1] == D) {
      bulk_prefetch_l2(row0, static_cast<uint32_t>(gs * D * sizeof(T)));
    } else {
      for (int r = 0; r < gs; ++r) bulk_prefetch_l2(row0 + static_cast<int64_t>(r) * a.d.q_stride[1], D * sizeof(T));
    }
  }

  // R0 / R1 (static stride W): the tasks a CTA will claim are known in advance (worker,
  // worker + W, ...), so lanes 0..kLook-1 of the scheduler warp resolve the next kLook tasks
  // in parallel (each a chain of dependent global loads: record fields, request counts /
  // indptr) and lane 0 pushes them in claim order.  The serial claim loop costs those round
  // trips once per task, which dominates small batches.
  //
  // R1's last rounds are claimed from the layer's claim counter instead of by stride: SMs
  // stream at measurably different rates (on B200 the CTAs of a C3 step finished up to
  // 110 us apart with equal task counts), so a fully static split leaves the fastest SMs
  // idle for the tail.  The task set is R1's and each task runs once, so the outputs are
  // bit-identical; R0, the prefix-search ablation, stays a pure stride.
  static constexpr int kLook = 4;

  // One task of an R0 / R1 plan (attention.py:23-47).  The caller checks the task against the
  // task count: a task past it reads an in-bounds record and must be dropped.
  __device__ static TaskDesc resolve_strided(const DecodeLaunch& a, int mode, int task) {
    const sgld_plan_buffers& p = a.p;
    const int G = a.d.kv_heads;
    TaskDesc t{};
    t.valid = 0;
    t.group = task % G;
    const int record = min(task / G, a.bcap * a.smax - 1);   // in bounds while the count is in flight
    if (mode == 0) {   // attention.py:25-39 -- upper-bound search over offsets
      int lo = 0, hi = *p.active;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (record >= p.offsets[mid + 1]) lo = mid + 1;
        else hi = mid;
      }
      t.request = lo;
      t.split = record - p.offsets[lo];
      const int chunk = p.chunk[lo];
      t.begin = t.split * chunk;
      t.end = min(t.begin + chunk, p.lengths[lo]);
    } else {           // attention.py:41-47; an R1 plan's order is the identity (kernels/plan.py:72-74)
      t.request = p.request[record];
      t.split = p.split[record];
      t.begin = p.begin[record];
      t.end = p.end[record];
    }
    return finish_task(a, t);
  }

  // Validity check, CSR base and Q prefetch of a resolved task.
  __device__ static TaskDesc finish_task(const DecodeLaunch& a, TaskDesc t) {
    // never produced by a valid plan; skipping keeps every access in bounds
    if (!(t.request < 0 || t.request >= a.bcap || t.end <= t.begin || t.split < 0 || t.split >= a.smax)) {
      t.base = a.csr ? a.d.indptr[t.request] : t.request;
      t.valid = 1;
      if (a.fast_q && t.request < a.q_rows) prefetch_q(a, t);
    }
    return t;
  }

  // The R1 record fields of this lane's first task (lanes 0..kLook-1), loaded before the
  // mode is known: the addresses do not depend on it and every record slot is in bounds,
  // so the loads share the mode's round trip.  Unused unless the mode is R1.
  struct FirstRound {
    int request, split, begin, end, records;
  };
  __device__ static FirstRound load_first_round(const DecodeLaunch& a) {
    const int lane = threadIdx.x & 31;
    const int task = blockIdx.x + lane * gridDim.x;
    const int record = min(task / a.d.kv_heads, a.bcap * a.smax - 1);
    FirstRound f{0, 0, 0, 0, 0};
    if (lane < kLook) {
      f.request = a.p.request[record];
      f.split = a.p.split[record];
      f.begin = a.p.begin[record];
      f.end = a.p.end[record];
    }
    f.records = *a.p.record_count;
    return f;
  }

  __device__ static void scheduler_strided(const DecodeLaunch& a, Misc& ms, int mode, const FirstRound& first) {
    const int lane = threadIdx.x & 31;
    const int W = gridDim.x;
    const int total = first.records * a.d.kv_heads;
    int ti = 0;
    uint32_t tph = 0;
    bool ok = true;
    int static_end = -1;
    for (int base = blockIdx.x; ok; base += kLook * W) {
      const int task = base + lane * W;
      TaskDesc t{};
      t.valid = 0;
      if (lane < kLook) {
        if (mode == 1 && base == static_cast<int>(blockIdx.x)) {
          TaskDesc r{};
          r.valid = 0;
          r.group = task % a.d.kv_heads;
          r.request = first.request;
          r.split = first.split;
          r.begin = first.begin;
          r.end = first.end;
          t = finish_task(a, r);
        } else {
          t = resolve_strided(a, mode, task);
        }
      }
      if (static_end < 0) {
        // Static rounds (every round for R0); R1 leaves about an eighth of them, at least
        // two, to the claimed tail.
        static_end = total;
        if (mode == 1) {
          const int rounds = total / W;
          static_end = (rounds - min(rounds, max(2, rounds / 8))) * W;
        }
      }
      if (task >= static_end) t.valid = 0;
      for (int l = 0; l < kLook; ++l) {
        TaskDesc u;
        u.request = __shfl_sync(0xffffffffu, t.request, l);
        u.split = __shfl_sync(0xffffffffu, t.split, l);
        u.group = __shfl_sync(0xffffffffu, t.group, l);
        u.begin = __shfl_sync(0xffffffffu, t.begin, l);
        u.end = __shfl_sync(0xffffffffu, t.end, l);
        u.base = __shfl_sync(0xffffffffu, t.base, l);
        u.valid = __shfl_sync(0xffffffffu, t.valid, l);
        if (u.valid && lane == 0) ok = push_task(ms, ti, tph, u, a.d.status);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      if (base + kLook * W >= static_end) break;
    }
    // R1 tail: tasks [static_end, total) one claim at a time, each claimed only once the
    // indexer has taken the task pushed before it, so a CTA holds few claimed tasks and the
    // CTAs finish close together.
    if (lane == 0) {
      int last_slot = -1;
      uint32_t last_phase = 0;
      while (ok && static_end < total) {
        if (last_slot >= 0 && !mbar_wait(&ms.tempty[last_slot], last_phase, global_timer_ns() + kWaitLimitNs)) {
          atomicOr(a.d.status, kStatusWaitTask);
          ok = false;
          break;
        }
        const int task = static_end + atomicAdd(a.d.counter, 1);
        if (task >= total) break;
        const TaskDesc t = resolve_strided(a, mode, task);
        if (!t.valid) continue;
        last_slot = ti;
        last_phase = tph;
        ok = push_task(ms, ti, tph, t, a.d.status);
      }
      TaskDesc end_marker{};
      end_marker.valid = 0;
      push_task(ms, ti, tph, end_marker, a.d.status);
    }
    __syncwarp();
  }

  __device__ static void scheduler(const DecodeLaunch& a, Misc& ms) {
    const sgld_plan_buffers& p = a.p;
    const int G = a.d.kv_heads;
    const int W = gridDim.x, worker = blockIdx.x;
    const int mode = *p.mode;
    const int total = *p.record_count * G;
    const bool dynamic = mode >= 3;
    // D1 packs are single tasks in pack order: with width 1 the plan writes pack_first[c] = c
    // and pack_count[c] = 1 (kernels/plan.py:84-99), so a D1 claim is the task itself.
    const bool d1 = mode == 3;
    int ti = 0;
    uint32_t tph = 0;
    int cursor, limit;
    if (dynamic) {
      cursor = atomicAdd(a.d.counter, 1);
      limit = *p.num_packs;
    } else if (mode == 2) {
      cursor = p.static_head[worker];
      limit = total;
    } else {
      cursor = worker;
      limit = total;
    }
    int guard = 0;
    bool ok = true;
    while (ok && cursor >= 0 && cursor < limit) {
      int first = cursor, count = 1;
      if (dynamic && !d1) {
        first = p.pack_first[cursor];
        count = p.pack_count[cursor];
      }
      for (int item = 0; item < count && ok; ++item) {
        const int task = first + item;
        TaskDesc t;
        t.group = task % G;
        int record = task / G;
        if (mode == 0) {   // attention.py:25-39 -- upper-bound search over offsets
          int lo = 0, hi = *p.active;
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (record >= p.offsets[mid + 1]) lo = mid + 1;
            else hi = mid;
          }
          t.request = lo;
          t.split = record - p.offsets[lo];
          const int chunk = p.chunk[lo];
          t.begin = t.split * chunk;
          t.end = min(t.begin + chunk, p.lengths[lo]);
        } else {           // attention.py:41-47; an R1 plan's order is the identity (kernels/plan.py:72-74)
          if (mode >= 3) record = p.order[record];
          t.request = p.request[record];
          t.split = p.split[record];
          t.begin = p.begin[record];
          t.end = p.end[record];
        }
        if (t.request < 0 || t.request >= a.bcap || t.end <= t.begin || t.split < 0 ||
            t.split >= a.smax)
          continue;   // never produced by a valid plan; skipping keeps every access in bounds
        t.base = a.csr ? a.d.indptr[t.request] : t.request;
        t.valid = 1;
        // The task's query rows are read by producer 0 a few stages before the consumers
        // need them; fetching them into L2 now, a few tasks ahead, keeps that read off HBM
        // (measured at B=256: an uncached Q cost about 10% of the decode).
        if (a.fast_q && t.request < a.q_rows) prefetch_q(a, t);
        ok = push_task(ms, ti, tph, t, a.d.status);
      }
      if (dynamic) {
        cursor = atomicAdd(a.d.counter, 1);
      } else if (mode == 2) {
        cursor = p.static_next[cursor];
        if (++guard > limit) {
          atomicOr(a.d.status, kStatusStaticCycle);
          break;
        }
      } else {
        cursor += W;
      }
    }
    TaskDesc end_marker{};
    end_marker.valid = 0;
    push_task(ms, ti, tph, end_marker, a.d.status);
  }

  // ------------------------------------------------------------------ indexer (warp)
  // Ring entry layout: koff[kTS], voff[kTS] (int64 element offsets of the rows, without
  // the dim term), then page[kTS], row[kTS] (int32, paged TMA coordinates).
  struct Batch {
    TaskDesc t;
    int tb;       // first token of the batch
    int phys[C::kNB][2], inner[C::kNB][2];
  };

  // Issue the index loads of up to kNB stages starting at token tb (tokens past the
  // task's end are clamped to its last token so every index read stays in bounds).
  __device__ static void gather(const DecodeLaunch& a, Batch& b) {
    const int lane = threadIdx.x & 31;
    const int ps = a.d.page_size;
#pragma unroll
    for (int i = 0; i < C::kNB; ++i) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int tok = min(b.tb + i * C::kTS + h * 32 + lane, b.t.end - 1);
        if (a.csr) {
          b.phys[i][h] = __ldg(a.d.pages + b.t.base + tok);
          b.inner[i][h] = 0;
        } else {
          const int page = tok / ps;
          b.phys[i][h] = __ldg(a.d.pages + static_cast<int64_t>(b.t.base) * a.d.pt_stride[0] +
                               static_cast<int64_t>(page) * a.d.pt_stride[1]);
          b.inner[i][h] = tok - page * ps;
        }
      }
    }
  }

  // Next batch after `cur`: the rest of the same task, or the first batch of the next
  // task from the task ring.  Returns false at the end of the work (or on a timeout).
  __device__ static bool next_batch(Misc& ms, const Batch& cur, bool have_cur, Batch& nxt, int& ti,
                                    uint32_t& tph, int* status) {
    const int lane = threadIdx.x & 31;
    if (have_cur && cur.tb + C::kNB * C::kTS < cur.t.end) {
      nxt.t = cur.t;
      nxt.tb = cur.tb + C::kNB * C::kTS;
      return true;
    }
    if (!warp_wait(&ms.tfull[ti], tph, status, kStatusWaitTask)) return false;
    nxt.t = ms.tq[ti];
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.tempty[ti]);
    if (++ti == C::kTaskQ) {
      ti = 0;
      tph ^= 1u;
    }
    nxt.tb = nxt.t.begin;
    return nxt.t.valid != 0;
  }

  __device__ static void indexer(const DecodeLaunch& a, unsigned char* smem, Misc& ms) {
    const int lane = threadIdx.x & 31;
    int* status = a.d.status;
    const int64_t* ks = a.d.k_stride;
    const int64_t* vs = a.d.v_stride;
    int ti = 0, sd = 0;
    uint32_t tph = 0, sph = 0;
    Batch b, n;
    bool have = next_batch(ms, b, false, b, ti, tph, status);
    if (have) gather(a, b);
    bool ok = true;
    while (have && ok) {
      // Put the next batch's loads in flight before writing this one (they land while
      // this batch waits for free descriptor slots).
      const bool have_next = next_batch(ms, b, true, n, ti, tph, status);
      if (have_next) gather(a, n);
#pragma unroll
      for (int i = 0; i < C::kNB; ++i) {
        const int t0 = b.tb + i * C::kTS;
        if (t0 >= b.t.end) break;
        ok = warp_wait(&ms.sempty[sd], sph ^ 1u, status, kStatusWaitDesc);
        if (!ok) break;
        unsigned char* entry = smem + C::kOffSD + sd * C::kSDEntry;
        int64_t* koff = reinterpret_cast<int64_t*>(entry);
        int64_t* voff = koff + C::kTS;
        int* page = reinterpret_cast<int*>(voff + C::kTS);
        int* row = page + C::kTS;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t pr = b.phys[i][h], in = b.inner[i][h];
          const int j = h * 32 + lane;
          koff[j] = pr * ks[0] + in * ks[1] + static_cast<int64_t>(b.t.group) * ks[2];
          voff[j] = pr * vs[0] + in * vs[1] + static_cast<int64_t>(b.t.group) * vs[2];
          page[j] = b.phys[i][h];
          row[j] = b.inner[i][h];
        }
        if (lane == 0) {
          StageHdr h;
          h.request = b.t.request;
          h.split = b.t.split;
          h.group = b.t.group;
          h.ntok = min(C::kTS, b.t.end - t0);
          h.flags = (t0 == b.t.begin ? kFlagFirst : 0) | (t0 + C::kTS >= b.t.end ? kFlagLast : 0);
          h.t0 = t0;
          h.pad[0] = h.pad[1] = 0;
          ms.shdr[sd] = h;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms.sfull[sd]);
        if (++sd == C::kSD) {
          sd = 0;
          sph ^= 1u;
        }
      }
      have = have_next;
      b = n;
    }
    if (!ok) return;
    if (!warp_wait(&ms.sempty[sd], sph ^ 1u, status, kStatusWaitDesc)) return;
    if (lane == 0) {
      StageHdr h{};
      h.flags = kFlagExit;
      ms.shdr[sd] = h;
      mbar_arrive(&ms.sfull[sd]);
    }
    __syncwarp();
  }

  // ------------------------------------------------------------------ producers (P warps)
  __device__ static void load_q(const DecodeLaunch& a, const StageHdr& h, unsigned char* qdst, uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    const T* q = static_cast<const T*>(a.d.q);
    const int gs = a.group_size;
    // A request past q's rows (the plan's active count exceeds q_rows) reads a zero query.
    const bool in_q = h.request < a.q_rows;
    if (!in_q && lane == 0) atomicOr(a.d.status, kStatusQRows);
    const T* qrow0 = q + static_cast<int64_t>(in_q ? h.request : 0) * a.d.q_stride[0] +
                     static_cast<int64_t>(h.group * gs) * a.d.q_stride[1];
    if (a.fast_q && std::is_same<MT, T>::value) {
      const uint32_t dst0 = smem_addr(qdst);
      for (int idx = lane; idx < C::kQRows * C::kQChunks; idx += 32) {
        const int r = idx / C::kQChunks, c = idx % C::kQChunks;
        const bool live = in_q && r < gs;   // rows past the group read as zeros
        const T* src = qrow0 + static_cast<int64_t>(live ? r : 0) * a.d.q_stride[1] + c * 8;
        cp_async_16_fill(dst0 + tile_off<C::kQRows>(r, c), src, live ? 16u : 0u);
      }
      cp_async_arrive_noinc(bar);
    } else {
      for (int idx = lane; idx < C::kQRows * D; idx += 32) {
        const int r = idx / D, d = idx % D;
        MT v = from_float<MT>(0.f);
        if (in_q && r < gs)
          v = from_float<MT>(to_float(qrow0[static_cast<int64_t>(r) * a.d.q_stride[1] +
                                            static_cast<int64_t>(d) * a.d.q_stride[2]]));
        *reinterpret_cast<MT*>(qdst + tile_off<C::kQRows>(r, d >> 3) + (d & 7) * 2) = v;
      }
      mbar_arrive(bar);
    }
  }

  __device__ static void producer(const DecodeLaunch& a, unsigned char* smem, Misc& ms) {
    const int lane = threadIdx.x & 31;
    const int pw = (threadIdx.x >> 5) - C::kProducerWarp0;   // 0 .. P-1
    // Tensor-map copies are issued by one thread: the other producer warps would only add
    // barrier traffic (the barrier counts at set-up leave them out).
    if (a.tma_kv && pw != 0) return;
    int* status = a.d.status;
    const KVT* kbase = static_cast<const KVT*>(a.d.k);
    const KVT* vbase = static_cast<const KVT*>(a.d.v);
    int sd = 0, s = 0, qcount = 0;
    uint32_t sph = 0, ph = 0;
    bool ok = true;
    while (true) {
      ok = warp_wait(&ms.sfull[sd], sph, status, kStatusWaitDesc);
      if (!ok) break;
      const StageHdr h = ms.shdr[sd];
      if (h.flags & kFlagExit) break;
      if ((h.flags & kFlagFirst) && pw == 0) {
        const int qs = qcount & 1;
        ok = warp_wait(&ms.qempty[qs], ((qcount >> 1) & 1) ^ 1u, status, kStatusWaitQ);
        if (!ok) break;
        load_q(a, h, smem + C::kOffQ + qs * C::kQBytes, &ms.qfull[qs]);
      }
      if (h.flags & kFlagFirst) ++qcount;
      ok = warp_wait(&ms.empty[s], ph ^ 1u, status, kStatusWaitEmpty);
      if (!ok) break;
      const unsigned char* entry = smem + C::kOffSD + sd * C::kSDEntry;
      const int64_t* koff = reinterpret_cast<const int64_t*>(entry);
      const int64_t* voff = koff + C::kTS;
      const int* page = reinterpret_cast<const int*>(voff + C::kTS);
      const int* prow = page + C::kTS;
      unsigned char* stage = smem + s * C::kStageBytes;
      const uint32_t kdst = smem_addr(stage);
      const uint32_t vdst = kdst + C::kTileBytes;
      if (!F8 && a.tma_kv) {
        // Tensor-map boxes: {64 dims, 1 head, R rows of one page}; only producer 0 issues.
        if (pw == 0 && lane == 0) {
          const int R = a.box_rows;
          const int nchunks = (h.ntok + R - 1) / R;
          ms.hdr[s] = h;
          mbar_arrive_expect_tx(&ms.full[s], static_cast<uint32_t>(nchunks * R * C::kRowBytes * 2));
          for (int c = 0; c < nchunks; ++c) {
            const int j = c * R;   // the box never crosses a page (R divides the page size)
#pragma unroll
            for (int part = 0; part < D / 64; ++part) {
              const uint32_t off = static_cast<uint32_t>((part * C::kTS + j) * 128);
              tma_load_4d(kdst + off, &a.kmap, part * 64, h.group, prow[j], page[j], &ms.full[s]);
              tma_load_4d(vdst + off, &a.vmap, part * 64, h.group, prow[j], page[j], &ms.full[s]);
            }
          }
        }
        __syncwarp();
        mbar_arrive(&ms.full[s]);   // 32P plain arrivals + the expect_tx arrival above
      } else if (a.fast_kv) {
        // 16-byte cp.async, token pairs spread over the producer warps; tokens past the
        // task's end are not copied (the consumers mask them).
        const int c = lane % C::kChunks;
#pragma unroll 4
        for (int i = pw; i < C::kTS / C::kTPI; i += C::kProducerWarps) {
          const int jt = i * C::kTPI + lane / C::kChunks;
          if (jt < h.ntok) {
            const uint32_t off = tile_off<C::kTS>(jt, c);
            cp_async_16(kdst + off, kbase + koff[jt] + c * C::kEPC);
            cp_async_16(vdst + off, vbase + voff[jt] + c * C::kEPC);
          }
        }
        cp_async_arrive_noinc(&ms.full[s]);
        if (pw == 0 && lane == 0) {
          ms.hdr[s] = h;
          mbar_arrive(&ms.full[s]);
        }
      } else {
        // Generic strides: element loads into the same swizzled layout.
        const int64_t kd = a.d.k_stride[3], vd = a.d.v_stride[3];
        for (int jt = pw; jt < h.ntok; jt += C::kProducerWarps) {
          const int64_t kr = koff[jt], vr = voff[jt];
          for (int d = lane; d < D; d += 32) {
            const uint32_t o = tile_off<C::kTS>(jt, d / C::kEPC) + (d % C::kEPC) * C::kKVBytes;
            *reinterpret_cast<KVT*>(stage + o) = kbase[kr + d * kd];
            *reinterpret_cast<KVT*>(stage + C::kTileBytes + o) = vbase[vr + d * vd];
          }
        }
        mbar_arrive(&ms.full[s]);
        if (pw == 0 && lane == 0) {
          ms.hdr[s] = h;
          mbar_arrive(&ms.full[s]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.sempty[sd]);   // this warp is done with the descriptor
      if (++sd == C::kSD) {
        sd = 0;
        sph ^= 1u;
      }
      if (++s == C::kStages) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (!ok) return;
    // Exit marker for the consumers (every producer lane arrives, producer 0 writes it).
    if (!warp_wait(&ms.empty[s], ph ^ 1u, status, kStatusWaitEmpty)) return;
    if (pw == 0 && lane == 0) {
      StageHdr h{};
      h.flags = kFlagExit;
      ms.hdr[s] = h;
      mbar_arrive(&ms.full[s]);
    }
    mbar_arrive(&ms.full[s]);
    __syncwarp();
  }

  // ------------------------------------------------------------------ consumers (4 warps)
  __device__ static void consumer(const DecodeLaunch& a, unsigned char* smem, Misc& ms) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g8 = lane >> 2, t4 = lane & 3;
    const int quad = warp >> 2;   // with two quads, quad q takes iterations q, q+2, ... of each task
    // Scores go to the log2 domain.  With a soft cap (logit_cap > 0) the scaled score s
    // becomes cap * tanh(s / cap) first; tanh comes from 1 - 2 / (2^(2x log2 e) + 1), exact at
    // both saturations (2^big = inf gives 1, 2^-big = 0 gives -1).
    const float cap = a.d.logit_cap;
    const bool capped = cap > 0.f;
    const float sc = (capped ? a.d.scale : a.d.scale * kLog2e) * a.d.k_scale;
    const float cap_log2e = cap * kLog2e, two_log2e_over_cap = capped ? 2.f * kLog2e / cap : 0.f;
    int* status = a.d.status;

    constexpr int KS = D / 16;   // k-steps of QK == m-tiles of O^T
    uint32_t qf[NT][KS][2];
    float o[KS][NT][4];
    float m[NT][2], lsum[NT][2];

    int s = 0, task_idx = 0, titer = 0;
    uint32_t ph = 0;
    while (true) {
      if (!warp_wait(&ms.full[s], ph, status, kStatusWaitFull)) return;
      const StageHdr h = ms.hdr[s];
      if (h.flags & kFlagExit) break;
      unsigned char* stage = smem + s * C::kStageBytes;
      if (h.flags & kFlagFirst) {
        titer = 0;
        const int qs = task_idx & 1;
        if (!warp_wait(&ms.qfull[qs], (task_idx >> 1) & 1, status, kStatusWaitQ)) return;
        const uint32_t qbase = smem_addr(smem + C::kOffQ + qs * C::kQBytes);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int ks = 0; ks < KS; ks += 2) {
            if constexpr (F8) {
              // Contraction order of the fp8 K fragments (below): k-step ks, B rows 2*t4 + {0,1}
              // and 8 + 2*t4 + {0,1} are dims 32*t4 + 4*ks + {0,1} and {2,3}.  Lane (g8, t4)
              // reads query row g8's dims [32*t4 + 4*ks, +8), i.e. chunk 4*t4 + ks/2.
              uint32_t w[4];
              lds_v4(qbase + tile_off<C::kQRows>(nt * 8 + g8, 4 * t4 + ks / 2), w);
              qf[nt][ks][0] = w[0];
              qf[nt][ks][1] = w[1];
              qf[nt][ks + 1][0] = w[2];
              qf[nt][ks + 1][1] = w[3];
            } else {
              const int row = nt * 8 + (lane & 7);
              const int chunk = 2 * ks + (lane >> 3);
              ldsm_x4(qbase + tile_off<C::kQRows>(row, chunk), qf[nt][ks][0], qf[nt][ks][1],
                      qf[nt][ks + 1][0], qf[nt][ks + 1][1]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms.qempty[qs]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          m[nt][0] = m[nt][1] = -INFINITY;
          lsum[nt][0] = lsum[nt][1] = 0.f;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
        }
      }

      // Paired stages: a stage that is not its task's last is followed in the ring by the
      // task's next stage; the warp takes its 16 rows of both, so one softmax update, one O
      // rescale and one set of shuffles cover 32 tokens and the two sub-tiles' MMAs overlap.
      // Pairs restart at every task, so the arithmetic does not depend on the dispatch mode.
      // Every warp reads every stage header (the task boundaries); the owning quad computes.
      // Ownership counts iterations (a stage or a pair) from the task's first stage, so it
      // does not depend on the dispatch mode.
      const bool own = C::kQuads == 1 || titer % C::kQuads == quad;
      const int row0 = (warp & 3) * 16;
      const bool pair = C::kPair && !(h.flags & kFlagLast);
      int s2 = s + 1;
      uint32_t ph2 = ph;
      if (s2 == C::kStages) {
        s2 = 0;
        ph2 ^= 1u;
      }
      int flags2 = 0, ntok2 = 0;
      if (pair) {
        if (!warp_wait(&ms.full[s2], ph2, status, kStatusWaitFull)) return;
        flags2 = ms.hdr[s2].flags;
        ntok2 = ms.hdr[s2].ntok;
      }
      const int valid_a = h.ntok - row0;            // live tokens of this warp's rows in each
      const int valid_b = pair ? ntok2 - row0 : 0;  // stage (a non-last stage is full)
      if (own && valid_a > 0) {
        const uint32_t ka = smem_addr(stage), kb2 = smem_addr(smem + s2 * C::kStageBytes);
        const bool has_b = valid_b > 0;
        float sv[2][NT][4];
        qk_tile(ka, row0, qf, sv[0]);
        if (has_b) qk_tile(kb2, row0, qf, sv[1]);
        // ---- online softmax (log2 domain) over both sub-tiles; masked tokens score -inf
        uint32_t pb[2][NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int tok = g8 + (i >= 2 ? 8 : 0);
              float x = sv[u][nt][i] * sc;
              if (capped) x = cap_log2e * (1.f - 2.f / (ex2(x * two_log2e_over_cap) + 1.f));
              sv[u][nt][i] = tok < (u == 0 ? valid_a : valid_b) ? x : -INFINITY;
            }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            float mx = fmaxf(fmaxf(sv[0][nt][jj], sv[0][nt][jj + 2]), fmaxf(sv[1][nt][jj], sv[1][nt][jj + 2]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(m[nt][jj], mx);
            const float alpha = ex2(m[nt][jj] - mnew);   // ex2(-inf) == 0 on the first tile
            float psum = 0.f;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float p0 = ex2(sv[u][nt][jj] - mnew), p1 = ex2(sv[u][nt][jj + 2] - mnew);
              sv[u][nt][jj] = p0;
              sv[u][nt][jj + 2] = p1;
              psum += p0 + p1;
            }
            lsum[nt][jj] = lsum[nt][jj] * alpha + psum;
            m[nt][jj] = mnew;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              o[mt][nt][jj] *= alpha;
              o[mt][nt][jj + 2] *= alpha;
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            pb[u][nt][0] = movmatrix_t(Mma<MT>::pack(sv[u][nt][0], sv[u][nt][1]));
            pb[u][nt][1] = movmatrix_t(Mma<MT>::pack(sv[u][nt][2], sv[u][nt][3]));
          }
        }
        // ---- O^T += V^T P^T per sub-tile
        pv_tile(smem_addr(stage) + C::kTileBytes, row0, valid_a, pb[0], o);
        if (has_b) pv_tile(smem_addr(smem + s2 * C::kStageBytes) + C::kTileBytes, row0, valid_b, pb[1], o);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ms.empty[s]);
        if (pair) mbar_arrive(&ms.empty[s2]);
      }

      if ((pair ? flags2 : h.flags) & kFlagLast) {
        if (!epilogue(a, smem, ms, h, task_idx, o, m, lsum)) return;
        ++task_idx;
      }
      ++titer;
      if (pair) {
        s = s2;
        ph = ph2;
      }
      if (++s == C::kStages) {
        s = 0;
        ph ^= 1u;
      }
    }
  }

  // S^T = K Q^T for rows [row0, row0 + 16) of the K tile at `kb` (summed over kChains
  // independent accumulators: a dependent chain of MMAs is latency bound).
  __device__ static void qk_tile(uint32_t kb, int row0, const uint32_t (&qf)[NT][D / 16][2],
                                 float (&out)[NT][4]) {
    constexpr int KS = D / 16;
    const int lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
    constexpr int kChains = C::kPair ? (NT == 1 ? 4 : 2) : (NT == 1 ? (KS < 8 ? KS : 8) : 2);
    float sacc[kChains][NT][4];
#pragma unroll
    for (int c = 0; c < kChains; ++c)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sacc[c][nt][i] = 0.f;
    // fp8 K straight into A fragments: lane (g8, t4) reads bytes [32*t4, +32) of rows g8 and
    // g8 + 8 (two 16-byte chunks each, conflict-free under the swizzle) and widens dims
    // 32*t4 + 4*ks + {0,1} / {2,3} to the k-pairs 2*t4 / 8 + 2*t4 of k-step ks.  The
    // contraction over D is order-free; Q's fragments follow the same order.
    uint32_t kw[F8 ? 2 : 1][F8 ? 8 : 1];
    if constexpr (F8) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        uint32_t w0[4], w1[4];
        lds_v4(kb + tile_off<C::kTS>(row0 + g8 + 8 * r, 2 * t4), w0);
        lds_v4(kb + tile_off<C::kTS>(row0 + g8 + 8 * r, 2 * t4 + 1), w1);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          kw[r][i] = w0[i];
          kw[r][4 + i] = w1[i];
        }
      }
    }
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a0, a1, a2, a3;
      if constexpr (F8) {
        a0 = e4m3x2_to_f16x2(kw[0][ks] & 0xffffu);
        a2 = e4m3x2_to_f16x2(kw[0][ks] >> 16);
        a1 = e4m3x2_to_f16x2(kw[1][ks] & 0xffffu);
        a3 = e4m3x2_to_f16x2(kw[1][ks] >> 16);
      } else {
        ldsm_x4(kb + tile_off<C::kTS>(row0 + (lane & 15), 2 * ks + (lane >> 4)), a0, a1, a2, a3);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        Mma<MT>::run(sacc[ks % kChains][nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
    }
#pragma unroll
    for (int w = kChains / 2; w >= 1; w /= 2)
#pragma unroll
      for (int c = 0; c < w; ++c)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) sacc[c][nt][i] += sacc[c + w][nt][i];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) out[nt][i] = sacc[0][nt][i];
  }

  // O^T += V^T P^T for rows [row0, row0 + 16) of the V tile at `vb`; rows past `valid` are
  // zeroed in the fragments (their P is already zero, stale shared memory may not be).
  __device__ static void pv_tile(uint32_t vb, int row0, int valid, const uint32_t (&pb)[NT][2],
                                 float (&o)[D / 16][NT][4]) {
    constexpr int KS = D / 16;
    const int lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
    const bool partial = valid < 16;
    const uint32_t mlo = (2 * t4 < valid ? 0x0000ffffu : 0u) | (2 * t4 + 1 < valid ? 0xffff0000u : 0u);
    const uint32_t mhi = (2 * t4 + 8 < valid ? 0x0000ffffu : 0u) | (2 * t4 + 9 < valid ? 0xffff0000u : 0u);
    // fp8 V: lane (g8, t4) holds dims [16*g8, +16) of token rows 2*t4, 2*t4 + 1, 2*t4 + 8,
    // 2*t4 + 9 (one conflict-free 16-byte chunk each); m-tile mt's rows g8 and g8 + 8 are
    // dims 16*g8 + 2*mt and +1 (the epilogue writes O in that order), and a byte permute
    // pairs the two tokens of each k-pair before widening.
    uint32_t vw[F8 ? 4 : 1][4];
    if constexpr (F8) {
#pragma unroll
      for (int r = 0; r < 4; ++r) lds_v4(vb + tile_off<C::kTS>(row0 + 2 * t4 + (r & 1) + (r >> 1) * 8, g8), vw[r]);
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      uint32_t a0, a1, a2, a3;
      if constexpr (F8) {
        const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
        const uint32_t x = __byte_perm(vw[0][mt >> 1], vw[1][mt >> 1], sel);
        const uint32_t y = __byte_perm(vw[2][mt >> 1], vw[3][mt >> 1], sel);
        a0 = e4m3x2_to_f16x2(x & 0xffffu);
        a1 = e4m3x2_to_f16x2(x >> 16);
        a2 = e4m3x2_to_f16x2(y & 0xffffu);
        a3 = e4m3x2_to_f16x2(y >> 16);
      } else {
        const int row = row0 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = 2 * mt + ((lane >> 3) & 1);
        ldsm_x4_t(vb + tile_off<C::kTS>(row, chunk), a0, a1, a2, a3);
      }
      if (partial) {
        a0 &= mlo;
        a1 &= mlo;
        a2 &= mhi;
        a3 &= mhi;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) Mma<MT>::run(o[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
    }
  }

  // Combine the consumer warps' (m, l, O) of one task and store the normalised partial and
  // natural-log LSE of every query head of the group.
  __device__ static bool epilogue(const DecodeLaunch& a, unsigned char* smem, Misc& ms, const StageHdr& h,
                                  int task_idx, float (&o)[D / 16][NT][4], float (&m)[NT][2],
                                  float (&lsum)[NT][2]) {
    constexpr int KS = D / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ctid = threadIdx.x;
    const int g8 = lane >> 2, t4 = lane & 3;
    const int hq = a.d.query_heads, gs = a.group_size, smax = a.smax;
    const int buf = C::kRedBufs == 2 ? (task_idx & 1) : 0;
    float* red = reinterpret_cast<float*>(smem + C::kOffRed + buf * C::kRedOne);
    // 1. per-warp statistics and unscaled O^T to shared memory
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        float l = lsum[nt][jj];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (g8 == 0) {
          ms.m[buf][warp][nt * 8 + 2 * t4 + jj] = m[nt][jj];
          ms.l[buf][warp][nt * 8 + 2 * t4 + jj] = l;
        }
      }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = F8 ? 16 * g8 + 2 * mt + (i >= 2 ? 1 : 0) : mt * 16 + g8 + (i >= 2 ? 8 : 0);
          const int head = nt * 8 + 2 * t4 + (i & 1);
          red[(warp * C::kQRows + head) * C::kRedStride + d] = o[mt][nt][i];
        }
    if (!consumer_join(&ms.join[buf], (task_idx >> (C::kRedBufs == 2 ? 1 : 0)) & 1, a.d.status)) return false;
    // 2. rescale every warp's state to the group max, sum the warps, normalise, store.  One
    //    item is four consecutive dims of one head: the head's scale factors are computed
    //    once per item and every warp's row is read as a float4 (rows are 16-byte aligned:
    //    kRedStride is a multiple of 4).  Sums run over the warps in order, as one element
    //    at a time would.
    const int64_t slot0 = (static_cast<int64_t>(h.request) * hq + h.group * gs) * smax + h.split;
    constexpr int D4 = D / 4;
    for (int idx = ctid; idx < gs * D4; idx += C::kConsumerThreads) {
      const int head = idx / D4, d = (idx - head * D4) * 4;
      float sw[C::kConsumerWarps];
      float gm = -INFINITY;
#pragma unroll
      for (int w = 0; w < C::kConsumerWarps; ++w) {
        sw[w] = ms.m[buf][w][head];
        gm = fmaxf(gm, sw[w]);
      }
      float gl = 0.f;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < C::kConsumerWarps; ++w) {
        sw[w] = sw[w] == -INFINITY ? 0.f : ex2(sw[w] - gm);
        gl += ms.l[buf][w][head] * sw[w];
        const float4 r = *reinterpret_cast<const float4*>(red + (w * C::kQRows + head) * C::kRedStride + d);
        v.x += r.x * sw[w];
        v.y += r.y * sw[w];
        v.z += r.z * sw[w];
        v.w += r.w * sw[w];
      }
      const float vs = a.d.v_scale;
      const float f = vs / gl;   // one division per item, not one per dim (IEEE division is a long sequence)
      const float4 res = make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
      const int64_t slot = slot0 + static_cast<int64_t>(head) * smax;
      *reinterpret_cast<float4*>(a.d.partial + slot * D + d) = res;   // 16-byte aligned (checked at entry)
      if (d == 0) a.d.lse[slot] = (gm + lg2(gl)) * kLn2;
    }
    if (C::kRedBufs == 1) {   // single reduction buffer: drain before the next task reuses it
      if (!consumer_join(&ms.drain, task_idx & 1, a.d.status)) return false;
    }
    return true;
  }

  // ------------------------------------------------------------------ entry
  __device__ static void run(const DecodeLaunch& a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned base (the launch reserves 1 KB of slack): TMA's 128-byte swizzle
    // and the tile layout assume it.
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    Misc& ms = *reinterpret_cast<Misc*>(smem + C::kOffMisc);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
      const int producers = a.tma_kv ? 1 : C::kProducerWarps;   // warps that run the data ring
      for (int i = 0; i < C::kStages; ++i) {
        mbar_init(&ms.full[i], 32 * producers + 1);
        mbar_init(&ms.empty[i], C::kConsumerWarps);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&ms.qfull[i], 32);
        mbar_init(&ms.qempty[i], C::kConsumerWarps);
      }
      for (int i = 0; i < C::kTaskQ; ++i) {
        mbar_init(&ms.tfull[i], 1);
        mbar_init(&ms.tempty[i], 1);
      }
      for (int i = 0; i < C::kSD; ++i) {
        mbar_init(&ms.sfull[i], 1);
        mbar_init(&ms.sempty[i], producers);
      }
      mbar_init(&ms.join[0], C::kConsumerWarps);
      mbar_init(&ms.join[1], C::kConsumerWarps);
      mbar_init(&ms.drain, C::kConsumerWarps);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Programmatic dependent launch: everything above overlapped the previous kernel;
    // from here on its results (the plan, the previous layer) must be visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (warp < C::kConsumerWarps) {
      consumer(a, smem, ms);
    } else if (warp < C::kIndexerWarp) {
      producer(a, smem, ms);
    } else if (warp == C::kIndexerWarp) {
      indexer(a, smem, ms);
    } else {
      const FirstRound first = load_first_round(a);
      const int mode = *a.p.mode;
      if (mode <= 1) {
        scheduler_strided(a, ms, mode, first);
      } else {
        if (lane == 0) scheduler(a, ms);
        __syncwarp();
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // Let the dependent merge launch start filling SMs as this CTA leaves.  The merge
    // zeroes the claim words once this grid has completed, so the last CTA leaves without
    // a fence-and-atomic exit chain on the step's critical path.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }
};

template <typename T, int D, int NT, bool F8>
__global__ void __launch_bounds__(Cfg<D, NT, F8>::kThreads, 1) decode_kernel(const __grid_constant__ DecodeLaunch a) {
  Kernel<T, D, NT, F8>::run(a);
}

template <typename T, int D, int NT, bool F8>
cudaError_t launch_typed(const DecodeLaunch& a, cudaStream_t stream) {
  using C = Cfg<D, NT, F8>;
  constexpr int kMaxDevices = 64;
  // The shared-memory attribute belongs to the device's context: remember the context it
  // was set in (a device reset creates a new one).  Host threads may race here; setting
  // the attribute twice is harmless.
  static std::atomic<void*> configured[kMaxDevices] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  void* ctx = current_context();
  if (ctx == nullptr || configured[device].load(std::memory_order_acquire) != ctx) {
    e = cudaFuncSetAttribute(decode_kernel<T, D, NT, F8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[device].store(ctx, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.workers);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_kernel<T, D, NT, F8>, a);
}

// ------------------------------------------------------------------ small-batch kernel
// One CTA of four warps per task, for geometries whose whole task capacity
// (Bcap * Smax * Hkv) fits in a few waves (a handful of short requests, e.g. 8 requests of
// up to 1K tokens).  There is no persistent pipeline: each CTA resolves its task from the plan
// (attention.py:23-47, R0 prefix search or the record arrays; the dispatch order of a mode
// does not change a task's arithmetic), gathers the task's indices and K/V rows with cp.async
// in 64-token stages, and runs the persistent kernel's fragment code on them
// (qk_tile / pv_tile, the same online softmax and the same four-warp combine), so a task of
// one stage gives the same bits on both kernels.  Tasks past the plan's count exit at once.
// The split merge is fused: the last split CTA of a (request, KV head) to finish merges that
// group's rows (merge_row4, the merge kernel's arithmetic), counting arrivals in the plan's
// `arrivals` words, so a step is two launches (plan, decode) instead of three.
template <typename T>
struct Small {
  using K = Kernel<T, 128, 1, false>;
  using C = Cfg<128, 1, false>;
  static constexpr int D = 128;
  static constexpr int kThreads = 128;                  // four warps, 16 rows of a stage each
  static constexpr int kTS = C::kTS;                    // 64 tokens per stage
  // One stage buffer (K and V, 32 KB): with about 36 KB a CTA, registers (122 a thread) rather
  // than shared memory bound the CTAs per SM (four), so a small batch's tasks run in one wave.
  static constexpr int kOffQ = C::kStageBytes;
  static constexpr int kOffIdx = kOffQ + C::kQBytes;    // koff / voff of the stage
  static constexpr int kOffMl = kOffIdx + 2 * kTS * 8;
  static constexpr int kSmemUsed = kOffMl + 2 * 4 * 8 * 4;
  static constexpr int kSmemBytes = kSmemUsed + 1024;
  static_assert(4 * C::kQRows * C::kRedStride * 4 <= C::kStageBytes, "the combine reuses stage 0");

  // Index loads and cp.async of the stage starting at token t0.
  __device__ static void load_stage(const DecodeLaunch& a, unsigned char* smem, const TaskDesc& t, int t0) {
    const int tid = threadIdx.x;
    int64_t* koff = reinterpret_cast<int64_t*>(smem + kOffIdx);
    int64_t* voff = koff + kTS;
    if (tid < kTS) {
      const int tok = min(t0 + tid, t.end - 1);
      int64_t phys, inner = 0;
      if (a.csr) {
        phys = __ldg(a.d.pages + t.base + tok);
      } else {
        const int page = tok / a.d.page_size;
        phys = __ldg(a.d.pages + static_cast<int64_t>(t.base) * a.d.pt_stride[0] +
                     static_cast<int64_t>(page) * a.d.pt_stride[1]);
        inner = tok - page * a.d.page_size;
      }
      koff[tid] = phys * a.d.k_stride[0] + inner * a.d.k_stride[1] + static_cast<int64_t>(t.group) * a.d.k_stride[2];
      voff[tid] = phys * a.d.v_stride[0] + inner * a.d.v_stride[1] + static_cast<int64_t>(t.group) * a.d.v_stride[2];
    }
    __syncthreads();
    const int ntok = min(kTS, t.end - t0);
    const T* kb = static_cast<const T*>(a.d.k);
    const T* vb = static_cast<const T*>(a.d.v);
    const uint32_t kdst = smem_addr(smem);
    const uint32_t vdst = kdst + C::kTileBytes;
    const int c = tid & 15;
#pragma unroll
    for (int j = tid >> 4; j < kTS; j += kThreads / 16) {
      const bool live = j < ntok;
      const uint32_t off = tile_off<kTS>(j, c);
      cp_async_16_fill(kdst + off, live ? kb + koff[j] + c * 8 : kb, live ? 16u : 0u);
      cp_async_16_fill(vdst + off, live ? vb + voff[j] + c * 8 : vb, live ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  __device__ static void run(const DecodeLaunch& a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const sgld_plan_buffers& p = a.p;
    const int G = a.d.kv_heads;
    const int task = blockIdx.x;
    const int mode = *p.mode;
    const bool plan_error = *p.error != 0;
    // ---- rows the fused merge never reaches, by merge_kernel's rules: a request without
    // splits is zero, and every row is NaN when the plan's error word is set (the plan then
    // has no records).  CTA r*G+g covers request r's query heads of KV head g.
    if (task < a.bcap * G) {
      const int r = task / G, g = task - r * G;
      if (plan_error || p.counts[r] == 0) {
        const T fill = from_float<T>(plan_error ? __int_as_float(0x7fc00000) : 0.f);
        T* orow = static_cast<T*>(a.d.out) + (static_cast<int64_t>(r) * a.d.query_heads + g * a.group_size) * D;
        for (int i = threadIdx.x; i < a.group_size * D; i += kThreads) orow[i] = fill;
      }
    }
    if (plan_error || task >= *p.record_count * G) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g8 = lane >> 2, t4 = lane & 3;
    TaskDesc t;
    t.group = task % G;
    const int record = task / G;
    if (mode == 0) {   // attention.py:25-39 -- upper-bound search over offsets
      int lo = 0, hi = *p.active;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (record >= p.offsets[mid + 1]) lo = mid + 1;
        else hi = mid;
      }
      t.request = lo;
      t.split = record - p.offsets[lo];
      const int chunk = p.chunk[lo];
      t.begin = t.split * chunk;
      t.end = min(t.begin + chunk, p.lengths[lo]);
    } else {           // every record once; the mode's order does not change a task's result
      t.request = p.request[record];
      t.split = p.split[record];
      t.begin = p.begin[record];
      t.end = p.end[record];
    }
    if (t.request < 0 || t.request >= a.bcap || t.end <= t.begin || t.split < 0 || t.split >= a.smax) return;
    t.base = a.csr ? a.d.indptr[t.request] : t.request;
    // ---- query group (rows past the group, or a request past q's rows, read as zeros)
    const int gs = a.group_size;
    const bool in_q = t.request < a.q_rows;
    if (!in_q && tid == 0) atomicOr(a.d.status, kStatusQRows);
    {
      const int r = tid >> 4, c = tid & 15;   // 8 rows x 16 chunks: one copy per thread
      const bool live = in_q && r < gs;
      const T* src = static_cast<const T*>(a.d.q) + static_cast<int64_t>(in_q ? t.request : 0) * a.d.q_stride[0] +
                     static_cast<int64_t>(t.group * gs + (live ? r : 0)) * a.d.q_stride[1] + c * 8;
      cp_async_16_fill(smem_addr(smem + kOffQ) + tile_off<C::kQRows>(r, c), src, live ? 16u : 0u);
    }
    load_stage(a, smem, t, t.begin);   // commits the query copies with the first stage
    const float cap = a.d.logit_cap;
    const bool capped = cap > 0.f;
    const float sc = (capped ? a.d.scale : a.d.scale * kLog2e) * a.d.k_scale;
    const float cap_log2e = cap * kLog2e, two_log2e_over_cap = capped ? 2.f * kLog2e / cap : 0.f;
    constexpr int KS = D / 16;
    uint32_t qf[1][KS][2];
    float o[KS][1][4];
    float m[1][2], lsum[1][2];
    m[0][0] = m[0][1] = -INFINITY;
    lsum[0][0] = lsum[0][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) o[mt][0][0] = o[mt][0][1] = o[mt][0][2] = o[mt][0][3] = 0.f;
    const int row0 = warp * 16;
    for (int t0 = t.begin; t0 < t.end; t0 += kTS) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncthreads();
      if (t0 == t.begin) {
        const uint32_t qbase = smem_addr(smem + kOffQ);
#pragma unroll
        for (int ks = 0; ks < KS; ks += 2) {
          const int row = lane & 7;
          const int chunk = 2 * ks + (lane >> 3);
          ldsm_x4(qbase + tile_off<C::kQRows>(row, chunk), qf[0][ks][0], qf[0][ks][1], qf[0][ks + 1][0], qf[0][ks + 1][1]);
        }
      }
      const int valid = min(kTS, t.end - t0) - row0;
      if (valid > 0) {
        const uint32_t kb = smem_addr(smem);
        float sv[1][4];
        K::qk_tile(kb, row0, qf, sv);
        uint32_t pb[1][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = g8 + (i >= 2 ? 8 : 0);
          float x = sv[0][i] * sc;
          if (capped) x = cap_log2e * (1.f - 2.f / (ex2(x * two_log2e_over_cap) + 1.f));
          sv[0][i] = tok < valid ? x : -INFINITY;
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          float mx = fmaxf(sv[0][jj], sv[0][jj + 2]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mnew = fmaxf(m[0][jj], mx);
          const float alpha = ex2(m[0][jj] - mnew);
          const float p0 = ex2(sv[0][jj] - mnew), p1 = ex2(sv[0][jj + 2] - mnew);
          sv[0][jj] = p0;
          sv[0][jj + 2] = p1;
          lsum[0][jj] = lsum[0][jj] * alpha + (p0 + p1);
          m[0][jj] = mnew;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            o[mt][0][jj] *= alpha;
            o[mt][0][jj + 2] *= alpha;
          }
        }
        pb[0][0] = movmatrix_t(Mma<T>::pack(sv[0][0], sv[0][1]));
        pb[0][1] = movmatrix_t(Mma<T>::pack(sv[0][2], sv[0][3]));
        K::pv_tile(kb + C::kTileBytes, row0, valid, pb, o);
      }
      __syncthreads();   // every warp is done with the stage before it is refilled
      if (t0 + kTS < t.end) load_stage(a, smem, t, t0 + kTS);
    }
    // ---- combine the four warps (the persistent kernel's epilogue order) and store
    float* red = reinterpret_cast<float*>(smem);   // the stage buffer is free now
    float* ms_m = reinterpret_cast<float*>(smem + kOffMl);
    float* ms_l = ms_m + 4 * 8;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      float l = lsum[0][jj];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      if (g8 == 0) {
        ms_m[warp * 8 + 2 * t4 + jj] = m[0][jj];
        ms_l[warp * 8 + 2 * t4 + jj] = l;
      }
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = mt * 16 + g8 + (i >= 2 ? 8 : 0);
        const int head = 2 * t4 + (i & 1);
        red[(warp * C::kQRows + head) * C::kRedStride + d] = o[mt][0][i];
      }
    __syncthreads();
    const int64_t slot0 = (static_cast<int64_t>(t.request) * a.d.query_heads + t.group * gs) * a.smax + t.split;
    constexpr int D4 = D / 4;
    for (int idx = tid; idx < gs * D4; idx += kThreads) {
      const int head = idx / D4, d = (idx - head * D4) * 4;
      float sw[4];
      float gm = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        sw[w] = ms_m[w * 8 + head];
        gm = fmaxf(gm, sw[w]);
      }
      float gl = 0.f;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        sw[w] = sw[w] == -INFINITY ? 0.f : ex2(sw[w] - gm);
        gl += ms_l[w * 8 + head] * sw[w];
        const float4 r = *reinterpret_cast<const float4*>(red + (w * C::kQRows + head) * C::kRedStride + d);
        v.x += r.x * sw[w];
        v.y += r.y * sw[w];
        v.z += r.z * sw[w];
        v.w += r.w * sw[w];
      }
      const float vs = a.d.v_scale;
      const float f = vs / gl;   // one division per item, not one per dim (IEEE division is a long sequence)
      const float4 res = make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
      const int64_t slot = slot0 + static_cast<int64_t>(head) * a.smax;
      *reinterpret_cast<float4*>(a.d.partial + slot * D + d) = res;
      if (d == 0) a.d.lse[slot] = (gm + lg2(gl)) * kLn2;
    }
    // ---- fused merge: the last of the request's split CTAs of this KV head to arrive merges
    // the group's rows with merge_row4 (the stand-alone merge kernel's arithmetic, so the
    // output has the same bits) and leaves the arrival counter at zero for the next decode.
    // Release: every thread fences its partial/LSE stores before the arrival; acquire: the
    // last CTA fences after it and reads the slots through L2.
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    int* arrival = p.arrivals + static_cast<int64_t>(t.request) * G + t.group;
    const int n_splits = p.counts[t.request];
    if (tid == 0) s_last = atomicAdd(arrival, 1) == n_splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = tid; idx < gs * D4; idx += kThreads) {
      const int head = idx / D4, d = (idx - head * D4) * 4;
      const int64_t row = static_cast<int64_t>(t.request) * a.d.query_heads + t.group * gs + head;
      const float4 r = merge_row4(a.d.partial + row * a.smax * D + d, a.d.lse + row * a.smax, n_splits, D);
      T* o = static_cast<T*>(a.d.out) + row * D + d;
      o[0] = from_float<T>(r.x);
      o[1] = from_float<T>(r.y);
      o[2] = from_float<T>(r.z);
      o[3] = from_float<T>(r.w);
    }
    if (tid == 0) *arrival = 0;
  }
};

template <typename T>
__global__ void __launch_bounds__(Small<T>::kThreads, 4) decode_small_kernel(const __grid_constant__ DecodeLaunch a) {
  Small<T>::run(a);
}

template <typename T>
cudaError_t launch_small(const DecodeLaunch& a, cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  static std::atomic<void*> configured[kMaxDevices] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  void* ctx = current_context();
  if (ctx == nullptr || configured[device].load(std::memory_order_acquire) != ctx) {
    e = cudaFuncSetAttribute(decode_small_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, Small<T>::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[device].store(ctx, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.bcap * a.smax * a.d.kv_heads));   // the task capacity
  cfg.blockDim = dim3(Small<T>::kThreads);
  cfg.dynamicSmemBytes = Small<T>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_small_kernel<T>, a);
}

template <typename T>
cudaError_t launch_dtype(const DecodeLaunch& a, cudaStream_t stream) {
  const bool wide = a.group_size > 8;
  if (a.kv_fp8) {   // e4m3 K/V: head_dim 128 only (checked by the caller)
    if (a.d.head_dim != 128) return cudaErrorInvalidValue;
    return wide ? launch_typed<T, 128, 2, true>(a, stream) : launch_typed<T, 128, 1, true>(a, stream);
  }
  switch (a.d.head_dim) {
    case 64: return wide ? launch_typed<T, 64, 2, false>(a, stream) : launch_typed<T, 64, 1, false>(a, stream);
    case 128: return wide ? launch_typed<T, 128, 2, false>(a, stream) : launch_typed<T, 128, 1, false>(a, stream);
    case 256: return wide ? launch_typed<T, 256, 2, false>(a, stream) : launch_typed<T, 256, 1, false>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_decode(const DecodeLaunch& a, cudaStream_t stream) {
  return a.d.dtype == SGLD_DTYPE_BF16 ? launch_dtype<__nv_bfloat16>(a, stream) : launch_dtype<__half>(a, stream);
}

cudaError_t launch_decode_small(const DecodeLaunch& a, cudaStream_t stream) {
  return a.d.dtype == SGLD_DTYPE_BF16 ? launch_small<__nv_bfloat16>(a, stream) : launch_small<__half>(a, stream);
}

}  // namespace sgld
