// Persistent paged GQA decode for sm_100a with the split merge fused in.
//
// Replaces the reference's persistent_decode + _attention_task
// (kernels/attention.py:12-130) and merge_splits (kernels/merge.py:7-30), and the
// per-layer counter memset (runtime/engine.py:62).
//
// One CTA per worker (grid = workers), six warps with fixed roles:
//
//   warp 5  scheduler  claims tasks exactly as the reference's claim loop
//                      (attention.py:99-130: R0/R1 stride-W round robin, STATIC list
//                      walk, D1/D4 relaxed atomic per pack), resolves each task to
//                      (request, split, kv_head, token range) (attention.py:23-47)
//                      and pushes it into a 4-deep shared-memory task queue.
//   warp 4  producer   streams each task's K/V rows, 64 tokens per stage, into a
//                      multi-stage shared-memory ring with 16-byte cp.async
//                      (page-table or CSR gather, arbitrary 16B-aligned strides),
//                      completion tracked by mbarriers; loads the task's query
//                      group into a double-buffered Q slot.  Indices for the next
//                      stage are prefetched while the current one is issued.
//   warps 0-3 consumers each take 16 tokens of a stage.  QK and PV run on tensor
//                      cores (mma.sync m16n8k16) in "swapped" form so the GQA group
//                      (padded to 8 or 16) is the N dimension: S^T = K Q^T and
//                      O^T += V^T P^T; movmatrix turns the score accumulator into
//                      the P^T operand.  FP32 online softmax state is warp-private;
//                      at the end of a task the four warp states are combined.
//
// Every task writes its normalised partial and natural-log LSE to slot
// (request*Hq + head)*Smax + split (attention.py:81-84).  The CTA whose split is the
// last to arrive for (request, kv_head) merges all splits in split order
// (merge.py:17-27) and writes the output; single-split requests write the output
// directly (the merge of one split is the identity).  Rows without records are
// written as zeros, or NaN when the plan's error word is set (merge.py:28-30).
//
// Every mbarrier wait is bounded; on expiry a status bit is set and the CTA
// unwinds.  The claim counter and the arrival counters are left at zero.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s per wait
constexpr int kSmemBudget = 227 * 1024;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum : int { kFlagFirst = 1, kFlagLast = 2, kFlagExit = 4 };
enum : int { kStatusWaitFull = 1, kStatusWaitEmpty = 2, kStatusWaitQ = 4, kStatusWaitTask = 8,
             kStatusStaticCycle = 16 };

struct StageHdr {
  int request, split, group, ntok, flags, count_r, qslot, pad;
};

struct TaskDesc {
  int request, split, group, begin, end, count_r, base, valid;
};

template <int D, int NT>
struct Cfg {
  static constexpr int kConsumerWarps = 4;
  static constexpr int kProducerWarp = 4;   // warp 5 is the scheduler
  static constexpr int kThreads = 6 * 32;
  static constexpr int kConsumerThreads = kConsumerWarps * 32;
  static constexpr int kTS = 64;                         // tokens per stage
  static constexpr int kRowBytes = D * 2;
  static constexpr int kChunks = kRowBytes / 16;         // 16-byte chunks per row
  static constexpr int kTPI = (32 / kChunks) > 0 ? 32 / kChunks : 1;  // tokens per warp copy
  static constexpr int kTileBytes = kTS * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kQRows = NT * 8;
  static constexpr int kQBytes = kQRows * kRowBytes;
  static constexpr int kRedStride = D + 4;               // floats; padding avoids bank conflicts
  static constexpr int kRedBytes = kConsumerWarps * kQRows * kRedStride * 4;
  static constexpr int kTaskQ = 4;
  static constexpr int kMiscBytes = 4096;
  static constexpr int kFixed = 2 * kQBytes + kRedBytes + kMiscBytes;
  static constexpr int kStagesRaw = (kSmemBudget - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static_assert(kStages >= 2, "shared memory budget too small");
  // Offsets.
  static constexpr int kOffQ = kStages * kStageBytes;
  static constexpr int kOffRed = kOffQ + 2 * kQBytes;
  static constexpr int kOffMisc = kOffRed + kRedBytes;
  static constexpr int kSmemBytes = kOffMisc + kMiscBytes;
};

// Small shared-memory area: barriers, stage headers, task queue, reduction scalars.
template <int D, int NT>
struct Misc {
  uint64_t full[8], empty[8], qfull[2], qempty[2], tfull[4], tempty[4];
  StageHdr hdr[8];
  TaskDesc tq[4];
  float m[4][16], l[4][16], gm[16], gl[16];
  int flag;
};

// Byte offset of 16-byte chunk `chunk` inside row `row` of a tile: the low three chunk
// bits are XORed with the row so eight consecutive rows at one logical chunk hit eight
// distinct bank groups (conflict-free ldmatrix).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <typename T, int D, int NT>
struct Kernel {
  using C = Cfg<D, NT>;
  using M = Misc<D, NT>;

  // ------------------------------------------------------------------ scheduler
  __device__ static bool push_task(M& ms, int& ti, uint32_t& tph, const TaskDesc& t, int* status) {
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

  __device__ static void scheduler(const DecodeLaunch& a, M& ms) {
    const sgld_plan_buffers& p = a.p;
    const int G = a.d.kv_heads;
    const int W = gridDim.x, worker = blockIdx.x;
    const int mode = *p.mode;
    const int total = *p.record_count * G;
    const bool dynamic = mode >= 3;
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
      if (dynamic) {
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
        } else {           // attention.py:41-47
          if (mode != 2) record = p.order[record];
          t.request = p.request[record];
          t.split = p.split[record];
          t.begin = p.begin[record];
          t.end = p.end[record];
        }
        if (t.request < 0 || t.request >= a.bcap || t.end <= t.begin || t.split < 0 ||
            t.split >= a.smax)
          continue;   // never produced by a valid plan; skipping keeps every access in bounds
        t.count_r = p.counts[t.request];
        t.base = a.csr ? a.d.indptr[t.request] : t.request;
        t.valid = 1;
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

  // ------------------------------------------------------------------ producer
  struct Job {
    TaskDesc t;
    int t0;
    int first;
  };

  __device__ static bool pop_task(M& ms, int& ti, uint32_t& tph, TaskDesc& t, int* status) {
    const int lane = threadIdx.x & 31;
    const bool ok = mbar_wait(&ms.tfull[ti], tph, global_timer_ns() + kWaitLimitNs);
    __syncwarp();
    if (!ok) {
      if (lane == 0) atomicOr(status, kStatusWaitTask);
      return false;
    }
    t = ms.tq[ti];
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.tempty[ti]);
    if (++ti == C::kTaskQ) {
      ti = 0;
      tph ^= 1u;
    }
    return true;
  }

  // Row index of token `tok` of the job's request: CSR -> kv_indices row,
  // paged -> physical page.  Issued one stage ahead of its use.
  __device__ static void prefetch(const DecodeLaunch& a, const Job& j, int (&phys)[2]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tok = min(j.t0 + h * 32 + lane, j.t.end - 1);
      if (a.csr) {
        phys[h] = __ldg(a.d.pages + j.t.base + tok);
      } else {
        const int ps = a.d.page_size;
        phys[h] = __ldg(a.d.pages + static_cast<int64_t>(j.t.base) * a.d.pt_stride[0] +
                        static_cast<int64_t>(tok / ps) * a.d.pt_stride[1]);
      }
    }
  }

  __device__ static void load_q(const DecodeLaunch& a, const TaskDesc& t, unsigned char* qdst,
                                uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    const T* q = static_cast<const T*>(a.d.q);
    const int group_size = a.group_size;
    const uint32_t dst0 = smem_addr(qdst);
    if (a.fast_q) {
      for (int idx = lane; idx < C::kQRows * C::kChunks; idx += 32) {
        const int h = idx / C::kChunks, c = idx % C::kChunks;
        const bool live = h < group_size;
        const T* src = q + static_cast<int64_t>(t.request) * a.d.q_stride[0] +
                       static_cast<int64_t>(t.group * group_size + (live ? h : 0)) * a.d.q_stride[1] + c * 8;
        cp_async_16_fill(dst0 + h * C::kRowBytes + swz(h, c), src, live ? 16u : 0u);
      }
      cp_async_arrive_noinc(bar);
    } else {
      for (int idx = lane; idx < C::kQRows * D; idx += 32) {
        const int h = idx / D, d = idx % D;
        T v = from_float<T>(0.f);
        if (h < group_size) {
          v = q[static_cast<int64_t>(t.request) * a.d.q_stride[0] +
                static_cast<int64_t>(t.group * group_size + h) * a.d.q_stride[1] +
                static_cast<int64_t>(d) * a.d.q_stride[2]];
        }
        *reinterpret_cast<T*>(qdst + h * C::kRowBytes + swz(h, d >> 3) + (d & 7) * 2) = v;
      }
      mbar_arrive(bar);
    }
  }

  __device__ static void issue_stage(const DecodeLaunch& a, const Job& j, const int (&phys)[2],
                                     unsigned char* stage, uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    const T* kbase = static_cast<const T*>(a.d.k);
    const T* vbase = static_cast<const T*>(a.d.v);
    const int64_t* ks = a.d.k_stride;
    const int64_t* vs = a.d.v_stride;
    const int ps = a.d.page_size;
    const int group = j.t.group;
    const uint32_t kdst = smem_addr(stage);
    const uint32_t vdst = kdst + C::kTileBytes;
    if (a.fast_kv) {
#pragma unroll
      for (int i = 0; i < C::kTS / C::kTPI; ++i) {
        const int jt = i * C::kTPI + lane / C::kChunks;   // token within the stage
        const int c = lane % C::kChunks;
        const int ph = __shfl_sync(0xffffffffu, phys[(i * C::kTPI) >> 5], jt & 31);
        const int tok = min(j.t0 + jt, j.t.end - 1);
        const int inner = a.csr ? 0 : tok % ps;
        const int64_t koff = static_cast<int64_t>(ph) * ks[0] + static_cast<int64_t>(inner) * ks[1] +
                             static_cast<int64_t>(group) * ks[2] + c * 8;
        const int64_t voff = static_cast<int64_t>(ph) * vs[0] + static_cast<int64_t>(inner) * vs[1] +
                             static_cast<int64_t>(group) * vs[2] + c * 8;
        const uint32_t off = jt * C::kRowBytes + swz(jt, c);
        cp_async_16(kdst + off, kbase + koff);
        cp_async_16(vdst + off, vbase + voff);
      }
      cp_async_arrive_noinc(bar);
    } else {
      // Generic strides: element loads into the same swizzled layout.
      for (int jt = 0; jt < C::kTS; ++jt) {
        const int ph = __shfl_sync(0xffffffffu, phys[jt >> 5], jt & 31);
        const int tok = min(j.t0 + jt, j.t.end - 1);
        const int inner = a.csr ? 0 : tok % ps;
        const int64_t krow = static_cast<int64_t>(ph) * ks[0] + static_cast<int64_t>(inner) * ks[1] +
                             static_cast<int64_t>(group) * ks[2];
        const int64_t vrow = static_cast<int64_t>(ph) * vs[0] + static_cast<int64_t>(inner) * vs[1] +
                             static_cast<int64_t>(group) * vs[2];
        unsigned char* krow_s = stage + jt * C::kRowBytes;
        unsigned char* vrow_s = krow_s + C::kTileBytes;
        for (int d = lane; d < D; d += 32) {
          const uint32_t o = swz(jt, d >> 3) + (d & 7) * 2;
          *reinterpret_cast<T*>(krow_s + o) = kbase[krow + static_cast<int64_t>(d) * ks[3]];
          *reinterpret_cast<T*>(vrow_s + o) = vbase[vrow + static_cast<int64_t>(d) * vs[3]];
        }
      }
      mbar_arrive(bar);
    }
  }

  __device__ static void producer(const DecodeLaunch& a, unsigned char* smem, M& ms) {
    const int lane = threadIdx.x & 31;
    int ti = 0;
    uint32_t tph = 0;
    int s = 0;
    uint32_t ph = 0;
    int qcount = 0;
    int* status = a.d.status;
    Job cur{}, nxt{};
    int cidx[2] = {0, 0}, nidx[2] = {0, 0};
    bool have = pop_task(ms, ti, tph, cur.t, status) && cur.t.valid;
    cur.t0 = have ? cur.t.begin : 0;
    cur.first = 1;
    if (have) prefetch(a, cur, cidx);
    bool aborted = false;
    while (have) {
      // Advance: next stage of this task, or the first stage of the next task.
      bool nhave;
      if (cur.t0 + C::kTS < cur.t.end) {
        nxt = cur;
        nxt.t0 = cur.t0 + C::kTS;
        nxt.first = 0;
        nhave = true;
      } else {
        // A failed pop (bounded wait expired, status already set) ends the stream.
        nhave = pop_task(ms, ti, tph, nxt.t, status) && nxt.t.valid;
        nxt.t0 = nhave ? nxt.t.begin : 0;
        nxt.first = 1;
      }
      if (nhave) prefetch(a, nxt, nidx);
      if (cur.first) {
        const int qs = qcount & 1;
        const bool qok = mbar_wait(&ms.qempty[qs], ((qcount >> 1) & 1) ^ 1u, global_timer_ns() + kWaitLimitNs);
        __syncwarp();
        if (!qok) {
          if (lane == 0) atomicOr(status, kStatusWaitQ);
          aborted = true;
          break;
        }
        load_q(a, cur.t, smem + C::kOffQ + qs * C::kQBytes, &ms.qfull[qs]);
        ++qcount;
      }
      const bool eok = mbar_wait(&ms.empty[s], ph ^ 1u, global_timer_ns() + kWaitLimitNs);
      __syncwarp();
      if (!eok) {
        if (lane == 0) atomicOr(status, kStatusWaitEmpty);
        aborted = true;
        break;
      }
      issue_stage(a, cur, cidx, smem + s * C::kStageBytes, &ms.full[s]);
      if (lane == 0) {
        StageHdr h;
        h.request = cur.t.request;
        h.split = cur.t.split;
        h.group = cur.t.group;
        h.ntok = min(C::kTS, cur.t.end - cur.t0);
        h.flags = (cur.first ? kFlagFirst : 0) | (cur.t0 + C::kTS >= cur.t.end ? kFlagLast : 0);
        h.count_r = cur.t.count_r;
        h.qslot = (qcount - 1) & 1;
        h.pad = 0;
        ms.hdr[s] = h;
        mbar_arrive(&ms.full[s]);
      }
      __syncwarp();
      if (++s == C::kStages) {
        s = 0;
        ph ^= 1u;
      }
      cur = nxt;
      cidx[0] = nidx[0];
      cidx[1] = nidx[1];
      have = nhave;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (aborted) return;
    // Exit marker for the consumers.
    const bool eok = mbar_wait(&ms.empty[s], ph ^ 1u, global_timer_ns() + kWaitLimitNs);
    __syncwarp();
    if (!eok) {
      if (lane == 0) atomicOr(status, kStatusWaitEmpty);
      return;
    }
    if (lane == 0) {
      StageHdr h{};
      h.flags = kFlagExit;
      ms.hdr[s] = h;
      mbar_arrive(&ms.full[s]);
    }
    __syncwarp();
    mbar_arrive(&ms.full[s]);
  }

  // ------------------------------------------------------------------ consumers
  __device__ static void write_empty_rows(const DecodeLaunch& a) {
    const int ctid = threadIdx.x;   // 0..127
    const int G = a.d.kv_heads, gs = a.group_size, hq = a.d.query_heads;
    const bool err = *a.p.error != 0;
    const T fill = from_float<T>(err ? __int_as_float(0x7fc00000) : 0.f);
    T* out = static_cast<T*>(a.d.out);
    for (int pair = blockIdx.x; pair < a.bcap * G; pair += gridDim.x) {
      const int r = pair / G, g = pair % G;
      if (__ldg(a.p.counts + r) != 0) continue;
      T* row = out + (static_cast<int64_t>(r) * hq + g * gs) * D;
      for (int idx = ctid; idx < gs * D; idx += C::kConsumerThreads) row[idx] = fill;
    }
  }

  __device__ static void consumer(const DecodeLaunch& a, unsigned char* smem, M& ms) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g8 = lane >> 2;
    const float sc = a.d.scale * kLog2e;
    int* status = a.d.status;

    write_empty_rows(a);

    constexpr int KS = D / 16;   // k-steps of QK == m-tiles of O^T
    uint32_t qf[NT][KS][2];
    float o[KS][NT][4];
    float m[NT][2], lsum[NT][2];

    int s = 0;
    uint32_t ph = 0;
    int task_idx = 0;
    while (true) {
      const bool got = mbar_wait(&ms.full[s], ph, global_timer_ns() + kWaitLimitNs);
      __syncwarp();
      if (!got) {
        if (lane == 0) atomicOr(status, kStatusWaitFull);
        return;
      }
      const StageHdr h = ms.hdr[s];
      if (h.flags & kFlagExit) return;
      unsigned char* stage = smem + s * C::kStageBytes;
      if (h.flags & kFlagFirst) {
        const int qs = task_idx & 1;
        const bool qok = mbar_wait(&ms.qfull[qs], (task_idx >> 1) & 1, global_timer_ns() + kWaitLimitNs);
        __syncwarp();
        if (!qok) {
          if (lane == 0) atomicOr(status, kStatusWaitQ);
          return;
        }
        const uint32_t qbase = smem_addr(smem + C::kOffQ + qs * C::kQBytes);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int ks = 0; ks < KS; ks += 2) {
            const int row = nt * 8 + (lane & 7);
            const int chunk = 2 * ks + (lane >> 3);
            ldsm_x4(qbase + row * C::kRowBytes + swz(row, chunk), qf[nt][ks][0], qf[nt][ks][1],
                    qf[nt][ks + 1][0], qf[nt][ks + 1][1]);
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

      const int row0 = warp * 16;
      if (row0 < h.ntok) {
        const int valid = h.ntok - row0;   // tokens of this warp's 16 that are live
        const uint32_t kb = smem_addr(stage);
        const uint32_t vb = kb + C::kTileBytes;
        // ---- S^T = K Q^T  (two independent accumulator chains)
        float sa[NT][4], sb[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) sa[nt][i] = sb[nt][i] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int row = row0 + (lane & 15);
          const int chunk = 2 * ks + (lane >> 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kb + row * C::kRowBytes + swz(row, chunk), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (ks & 1) Mma<T>::run(sb[nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
            else Mma<T>::run(sa[nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
          }
        }
        // ---- online softmax (log2 domain)
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float sv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tok = g8 + (i >= 2 ? 8 : 0);
            sv[i] = tok < valid ? (sa[nt][i] + sb[nt][i]) * sc : -INFINITY;
          }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            float mx = fmaxf(sv[jj], sv[jj + 2]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(m[nt][jj], mx);
            const float alpha = ex2(m[nt][jj] - mnew);   // ex2(-inf) == 0 on the first tile
            const float p0 = ex2(sv[jj] - mnew), p1 = ex2(sv[jj + 2] - mnew);
            sv[jj] = p0;
            sv[jj + 2] = p1;
            lsum[nt][jj] = lsum[nt][jj] * alpha + p0 + p1;
            m[nt][jj] = mnew;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              o[mt][nt][jj] *= alpha;
              o[mt][nt][jj + 2] *= alpha;
            }
          }
          pb[nt][0] = movmatrix_t(Mma<T>::pack(sv[0], sv[1]));
          pb[nt][1] = movmatrix_t(Mma<T>::pack(sv[2], sv[3]));
        }
        // ---- O^T += V^T P^T
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          const int row = row0 + (lane & 7) + ((lane >> 4) << 3);
          const int chunk = 2 * mt + ((lane >> 3) & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vb + row * C::kRowBytes + swz(row, chunk), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma<T>::run(o[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.empty[s]);

      if (h.flags & kFlagLast) {
        __syncwarp();
        epilogue(a, smem, ms, h, o, m, lsum);
        ++task_idx;
      }
      if (++s == C::kStages) {
        s = 0;
        ph ^= 1u;
      }
    }
  }

  __device__ static void epilogue(const DecodeLaunch& a, unsigned char* smem, M& ms, const StageHdr& h,
                                  float (&o)[D / 16][NT][4], float (&m)[NT][2], float (&lsum)[NT][2]) {
    constexpr int KS = D / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ctid = threadIdx.x;
    const int g8 = lane >> 2, t4 = lane & 3;
    const int hq = a.d.query_heads, gs = a.group_size, smax = a.smax, G = a.d.kv_heads;
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    // 1. warp-level row sums, publish per-warp (m, l)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        float l = lsum[nt][jj];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (g8 == 0) {
          ms.m[warp][nt * 8 + 2 * t4 + jj] = m[nt][jj];
          ms.l[warp][nt * 8 + 2 * t4 + jj] = l;
        }
      }
    consumer_sync();
    // 2. combine (m, l) across warps; scale this warp's O^T into the reduction buffer
    float scale[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int head = nt * 8 + 2 * t4 + jj;
        float gm = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::kConsumerWarps; ++w) gm = fmaxf(gm, ms.m[w][head]);
        float gl = 0.f;
#pragma unroll
        for (int w = 0; w < C::kConsumerWarps; ++w) {
          const float mw = ms.m[w][head];
          gl += mw == -INFINITY ? 0.f : ms.l[w][head] * ex2(mw - gm);
        }
        scale[nt][jj] = m[nt][jj] == -INFINITY ? 0.f : ex2(m[nt][jj] - gm);
        if (warp == 0 && g8 == 0) {
          ms.gm[head] = gm;
          ms.gl[head] = gl;
        }
      }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = mt * 16 + g8 + (i >= 2 ? 8 : 0);
          const int head = nt * 8 + 2 * t4 + (i & 1);
          red[(warp * C::kQRows + head) * C::kRedStride + d] = o[mt][nt][i] * scale[nt][i & 1];
        }
    consumer_sync();
    // 3. sum the four warp partials, normalise, store partial / LSE (and the output
    //    directly when the request has a single split)
    const int64_t slot0 = (static_cast<int64_t>(h.request) * hq + h.group * gs) * smax + h.split;
    T* out = static_cast<T*>(a.d.out);
    const int64_t orow0 = (static_cast<int64_t>(h.request) * hq + h.group * gs) * D;
    for (int idx = ctid; idx < gs * D; idx += C::kConsumerThreads) {
      const int head = idx / D, d = idx % D;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < C::kConsumerWarps; ++w) v += red[(w * C::kQRows + head) * C::kRedStride + d];
      const float gl = ms.gl[head];
      const float res = v / gl;
      const int64_t slot = slot0 + static_cast<int64_t>(head) * smax;
      a.d.partial[slot * D + d] = res;
      if (d == 0) a.d.lse[slot] = (ms.gm[head] + lg2(gl)) * kLn2;
      if (h.count_r == 1) out[orow0 + idx] = from_float<T>(res);
    }
    if (h.count_r <= 1) {
      consumer_sync();   // reduction buffers are reused by the next task
      return;
    }
    // 4. fused merge: the CTA completing the last split of (request, kv_head) merges
    __threadfence();
    consumer_sync();
    if (ctid == 0) {
      int* counter = a.d.arrive + h.request * G + h.group;
      const int old = atomicAdd(counter, 1);
      const int last = old == h.count_r - 1;
      if (last) atomicExch(counter, 0);
      ms.flag = last;
    }
    consumer_sync();
    if (ms.flag) {
      __threadfence();
      const int64_t base = (static_cast<int64_t>(h.request) * hq + h.group * gs) * smax;
      for (int idx = ctid; idx < gs * D; idx += C::kConsumerThreads) {
        const int head = idx / D, d = idx % D;
        const int64_t hs = base + static_cast<int64_t>(head) * smax;
        float mm = -INFINITY, den = 0.f, acc = 0.f;
        for (int sp = 0; sp < h.count_r; ++sp) {
          const float l = ld_cg(a.d.lse + hs + sp);
          const float pv = ld_cg(a.d.partial + (hs + sp) * D + d);
          const float nm = fmaxf(mm, l);
          const float ow = ex2((mm - nm) * kLog2e);
          const float w = ex2((l - nm) * kLog2e);
          acc = acc * ow + pv * w;
          den = den * ow + w;
          mm = nm;
        }
        out[orow0 + idx] = from_float<T>(acc / fmaxf(den, 1.0e-30f));
      }
    }
    consumer_sync();
  }

  // ------------------------------------------------------------------ entry
  __device__ static void run(const DecodeLaunch& a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    M& ms = *reinterpret_cast<M*>(smem + C::kOffMisc);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
      for (int i = 0; i < C::kStages; ++i) {
        mbar_init(&ms.full[i], 33);
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
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp < C::kConsumerWarps) {
      consumer(a, smem, ms);
    } else if (warp == C::kProducerWarp) {
      producer(a, smem, ms);
    } else {
      if (lane == 0) scheduler(a, ms);
      __syncwarp();
    }
    __syncthreads();
    // Exit ticket: the last CTA to finish leaves the claim counter at zero.
    if (threadIdx.x == 0) {
      __threadfence();
      const int ticket = atomicAdd(a.d.counter + 1, 1);
      if (ticket == static_cast<int>(gridDim.x) - 1) {
        atomicExch(a.d.counter, 0);
        atomicExch(a.d.counter + 1, 0);
      }
    }
  }
};

template <typename T, int D, int NT>
__global__ void __launch_bounds__(192, 1) decode_kernel(DecodeLaunch a) {
  Kernel<T, D, NT>::run(a);
}

template <typename T, int D, int NT>
cudaError_t launch_typed(const DecodeLaunch& a, cudaStream_t stream) {
  using C = Cfg<D, NT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, D, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  decode_kernel<T, D, NT><<<a.workers, C::kThreads, C::kSmemBytes, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dtype(const DecodeLaunch& a, cudaStream_t stream) {
  const bool wide = a.group_size > 8;
  switch (a.d.head_dim) {
    case 64: return wide ? launch_typed<T, 64, 2>(a, stream) : launch_typed<T, 64, 1>(a, stream);
    case 128: return wide ? launch_typed<T, 128, 2>(a, stream) : launch_typed<T, 128, 1>(a, stream);
    case 256: return wide ? launch_typed<T, 256, 2>(a, stream) : launch_typed<T, 256, 1>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_decode(const DecodeLaunch& a, cudaStream_t stream) {
  return a.d.dtype == SGLD_DTYPE_BF16 ? launch_dtype<__nv_bfloat16>(a, stream) : launch_dtype<__half>(a, stream);
}

}  // namespace sgld
