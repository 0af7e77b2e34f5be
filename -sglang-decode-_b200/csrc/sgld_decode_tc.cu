// Persistent paged GQA decode on the 5th-generation tensor cores (sm_100a): QK and PV run as
// tcgen05.mma with their accumulators in tensor memory (TMEM), for head_dim 128 and 16-bit
// K/V (the shape of every benchmark configuration).  Other geometries (head_dim 64 / 256,
// fp8 K/V, K/V rows that are not 16-byte aligned) keep the mma.sync kernel of
// sgld_decode.cu.
//
// Replaces the reference's persistent_decode + _attention_task (kernels/attention.py:12-130)
// with the same task dispatch (R0 prefix search, R1 stride, STATIC lists, D1/D4 atomic pack
// claims) and the same slot contract: every task writes the normalised partial and the
// natural-log LSE of its query heads to slot (request*Hq + head)*Smax + split
// (attention.py:81-84); the split merge (sgld_merge.cu) follows as a programmatic dependent
// launch.
//
// One CTA per worker; warps with fixed roles connected by mbarrier rings:
//
//   scheduler (1 warp, lane 0)  the reference's claim loop; pushes tasks into the task ring.
//   indexer (1 warp)            turns tasks into 128-token stage descriptors (page-table / CSR
//                               index gathers, two stages per round trip, K/V row offsets).
//   producers (8 warps)         fill a 3-stage ring of 128-token K and V tiles (separate
//                               barriers for K and V) with 16-byte cp.async, rows past the
//                               task's end zero-filled; paged KV whose page size is a multiple
//                               of 32 may use tensor-map TMA boxes from producer 0 instead.
//                               Producer 0 also loads each task's query group by a TMA box.
//   MMA issuer (1 warp, lane 0) per tile: S^T = K Q^T (M = 128 tokens, N = 16 query heads,
//                               K = 128 dims: eight tcgen05.mma) into one of two TMEM score
//                               buffers, then, one tile behind, O^T += V^T P^T (M = 128 dims,
//                               N = 16 heads, K = 128 tokens) into the task's TMEM output
//                               buffer.  Completion is signalled by tcgen05.commit.
//   softmax (4 warps)           warp w owns TMEM lanes 32w..32w+31 = tokens (scores) and dims
//                               (output).  Per tile: load the scores, mask, take the tile max
//                               per head (warp butterfly, then the four warps through shared
//                               memory), compute P = 2^(s - m) in FP32, store it as the 16-bit
//                               B operand of the PV MMA, keep the per-thread row sums.  The
//                               reference maximum m of a head changes only when a tile's max
//                               exceeds it by more than 2^8 (P stays <= 256): the output in
//                               TMEM is then rescaled in place.  At a task's end the warps
//                               read O^T, divide by the row sums and store partial and LSE.
//
// Shared-memory tiles use the 128-byte swizzle ([2 halves of 64 dims][rows][128 B]), which
// is both what TMA writes and the canonical K-major (K tile, Q) and MN-major (V tile)
// layouts of the MMA descriptors.  Every mbarrier wait is bounded (4 s); on expiry a status
// bit is set and the warp unwinds; tensor memory is released on every path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <type_traits>

#include "sgld_internal.cuh"
#include "sgld_ptx.cuh"

namespace sgld {
namespace {

constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s per wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.f;                // lazy rescale threshold (log2 units)

// Stage flags and the status bits of sgld_decode_args.status (same values as the mma.sync
// kernel: 1-32 a bounded wait expired, 64 a request past q_rows).
enum : int { kFlagFirst = 1, kFlagLast = 2, kFlagExit = 4 };
enum : int { kStatusWaitFull = 1, kStatusWaitEmpty = 2, kStatusWaitQ = 4, kStatusWaitTask = 8,
             kStatusStaticCycle = 16, kStatusWaitDesc = 32, kStatusQRows = 64 };

struct Hdr {
  int request, split, group, ntok, flags, count_r, t0, pad;
};

struct Task {
  int request, split, group, begin, end, count_r, base, valid;
};

constexpr int kD = 128;                        // head dim of this kernel
constexpr int kTS = 128;                       // tokens per stage (the MMA M of QK)
constexpr int kStages = 3;
constexpr int kTile = kTS * kD * 2;            // one K or V tile: 32 KB
constexpr int kStage = 2 * kTile;              // K tile then V tile
constexpr int kHalf = kTS * 128;               // bytes of one 64-dim half of a tile
constexpr int kQRows = 16;                     // MMA N: query heads of a group, padded
constexpr int kQBytes = kQRows * kD * 2;       // 4 KB
constexpr int kPBytes = kTS * kQRows * 2;      // 4 KB
constexpr int kPBufs = 4;                      // P buffers: the softmax runs up to 3 tiles ahead of PV
constexpr int kSD = 4;                         // stage-descriptor ring depth
constexpr int kNB = 2;                         // stages indexed per round trip
constexpr int kSDEntry = kTS * 8;              // page (or CSR slot) and row in page, int32 each
constexpr int kTaskQ = 4;
constexpr int kHdrQ = 4;                       // softmax header ring
constexpr int kSoftmaxWarps = 8;               // two groups of four: each group owns half the head columns
constexpr int kMmaWarp = kSoftmaxWarps;
constexpr int kProducerWarp0 = kMmaWarp + 1;
constexpr int kProducerWarps = 8;              // copy_tile covers 16 rows per step with 8 warps
constexpr int kIndexerWarp = kProducerWarp0 + kProducerWarps;
constexpr int kSchedulerWarp = kIndexerWarp + 1;
constexpr int kWarps = kSchedulerWarp + 1;
constexpr int kThreads = kWarps * 32;
constexpr int kSBufs = 4;                      // TMEM score buffers (QK runs up to 3 tiles ahead)
constexpr int kTmemCols = 128;                 // S[4] (16 columns each), O[2] (16 each) at column 64
constexpr int kOffQ = kStages * kStage;
constexpr int kOffP = kOffQ + 2 * kQBytes;
constexpr int kOffSD = kOffP + kPBufs * kPBytes;
constexpr int kOffMisc = kOffSD + kSD * kSDEntry;
constexpr int kMiscBytes = 3072;
constexpr int kSmemUsed = kOffMisc + kMiscBytes;
constexpr int kSmemBytes = kSmemUsed + 1024;   // launch size including 1 KB alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");

struct Misc {
  uint64_t full_k[kStages], full_v[kStages], empty_k[kStages], empty_v[kStages];
  uint64_t s_full[kSBufs], s_free[kSBufs], p_full[kPBufs], p_free[kPBufs];
  uint64_t q_full[2], q_empty[2], o_full[2], o_free[2];
  uint64_t tfull[kTaskQ], tempty[kTaskQ], sdfull[kSD], sdempty[kSD], hfull[kHdrQ], hempty[kHdrQ];
  uint64_t join[2][2], join_l[2][2], drain;   // [column group][parity]
  Hdr hdr[kStages];       // data ring headers (MMA issuer)
  int4 pend[kSBufs];      // MMA issuer: (stage, phase, task, flags) of tiles awaiting PV
  Hdr shdr[kSD];          // descriptor ring headers (producers)
  Hdr xhdr[kHdrQ];        // softmax header ring
  Task tq[kTaskQ];
  alignas(16) float red[2][4][16];     // [tile parity][TMEM quadrant][head]: per-warp tile maxima
  alignas(16) float red_l[2][4][16];   // [task parity][quadrant][head]: per-warp row sums at a task's end
  uint32_t tmem_base;
};
static_assert(sizeof(Misc) <= kMiscBytes, "misc area too small");
static_assert(offsetof(Misc, red) % 16 == 0 && offsetof(Misc, red_l) % 16 == 0, "float4 rows need 16-byte alignment");
static_assert(kOffMisc % 1024 == 0 && kOffP % 16 == 0 && kOffSD % 8 == 0, "shared-memory region alignment");

template <int ROWS>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return static_cast<uint32_t>(((chunk >> 3) * ROWS + row) * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// Bounded waits.  The common case (phase already complete, or completing within try_wait's
// own suspend window) stays inline; the deadline loop is out of line to keep every call site
// small (instruction-cache misses are a measured stall of this kernel).
//
// Waiting warps issue instructions while they poll, and most of this kernel's warps wait most
// of the time, so roles off the critical path (scheduler, indexer, producers) sleep between
// polls (kBackoffNs); the softmax warps and the MMA issuer poll promptly.
constexpr uint32_t kBackoffNs = 128;

__device__ __noinline__ bool wait_slow(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity, global_timer_ns() + kWaitLimitNs);
}

__device__ __noinline__ bool wait_slow_backoff(uint64_t* bar, uint32_t parity) {
  const uint64_t deadline = global_timer_ns() + kWaitLimitNs;
  while (!mbar_try_wait(bar, parity)) {
    __nanosleep(kBackoffNs);
    if (global_timer_ns() > deadline) return false;
  }
  return true;
}

template <bool kBackoff = false>
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_try_wait(bar, parity) || (kBackoff ? wait_slow_backoff(bar, parity) : wait_slow(bar, parity));
  if (!ok) atomicOr(status, code);
  return ok;
}

// Bounded wait that also reconverges the warp.
template <bool kBackoff = false>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_try_wait(bar, parity) || (kBackoff ? wait_slow_backoff(bar, parity) : wait_slow(bar, parity));
  __syncwarp();
  if (!ok && (threadIdx.x & 31) == 0) atomicOr(status, code);
  return ok;
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld<2>(uint32_t taddr, float (&v)[2]) {
  uint32_t r0, r1;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  v[0] = __uint_as_float(r0), v[1] = __uint_as_float(r1);
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float (&v)[8]) {
  tmem_ld8(taddr, v);
}

template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_st<2>(uint32_t taddr, const float (&v)[2]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1,%2};" ::"r"(taddr), "r"(__float_as_uint(v[0])),
               "r"(__float_as_uint(v[1])) : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
template <>
__device__ __forceinline__ void tmem_st<4>(uint32_t taddr, const float (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(__float_as_uint(v[0])),
               "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])) : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
template <>
__device__ __forceinline__ void tmem_st<8>(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])) : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// NHW: head columns per softmax warp (two groups cover 2*NHW heads: 4, 8 or 16 for groups of up
// to 4, 8 or 16).  The MMAs always use N = 16; P columns past 2*NHW stay zero.
template <typename T, int NHW>
struct TcKernel {
  // ------------------------------------------------------------------ scheduler (lane 0)
  __device__ static bool push_task(Misc& ms, int& ti, uint32_t& tph, const Task& t, int* status) {
    if (!wait_bar<true>(&ms.tempty[ti], tph ^ 1u, status, kStatusWaitTask)) return false;
    ms.tq[ti] = t;
    mbar_arrive(&ms.tfull[ti]);
    if (++ti == kTaskQ) {
      ti = 0;
      tph ^= 1u;
    }
    return true;
  }

  __device__ static void scheduler(const DecodeLaunch& a, Misc& ms) {
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
        Task t;
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
        if (t.request < 0 || t.request >= a.bcap || t.end <= t.begin || t.split < 0 || t.split >= a.smax)
          continue;   // never produced by a valid plan; skipping keeps every access in bounds
        t.count_r = p.counts[t.request];
        t.base = a.csr ? a.d.indptr[t.request] : t.request;
        t.valid = 1;
        // The query rows are loaded by producer 0 a little later; bring them into L2 now.
        if (a.fast_q && t.request < a.q_rows) {
          const T* row0 = static_cast<const T*>(a.d.q) + static_cast<int64_t>(t.request) * a.d.q_stride[0] +
                          static_cast<int64_t>(t.group * a.group_size) * a.d.q_stride[1];
          if (a.d.q_stride[1] == kD) {
            bulk_prefetch_l2(row0, static_cast<uint32_t>(a.group_size * kD * sizeof(T)));
          } else {
            for (int r = 0; r < a.group_size; ++r)
              bulk_prefetch_l2(row0 + static_cast<int64_t>(r) * a.d.q_stride[1], kD * sizeof(T));
          }
        }
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
    Task end_marker{};
    end_marker.valid = 0;
    push_task(ms, ti, tph, end_marker, a.d.status);
  }

  // ------------------------------------------------------------------ indexer (warp)
  struct Batch {
    Task t;
    int tb;                          // first token of the batch
    int phys[kNB][4], inner[kNB][4];
  };

  // Index loads of up to kNB stages from token tb (clamped to the task's last token so every
  // read stays in bounds).  Lane l handles tokens l, l+32, l+64, l+96 of each stage.
  __device__ static void gather(const DecodeLaunch& a, Batch& b) {
    const int lane = threadIdx.x & 31;
    const int ps = a.d.page_size;
#pragma unroll
    for (int i = 0; i < kNB; ++i) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tok = min(b.tb + i * kTS + u * 32 + lane, b.t.end - 1);
        if (a.csr) {
          b.phys[i][u] = __ldg(a.d.pages + b.t.base + tok);
          b.inner[i][u] = 0;
        } else {
          const int page = tok / ps;
          b.phys[i][u] = __ldg(a.d.pages + static_cast<int64_t>(b.t.base) * a.d.pt_stride[0] +
                               static_cast<int64_t>(page) * a.d.pt_stride[1]);
          b.inner[i][u] = tok - page * ps;
        }
      }
    }
  }

  __device__ static bool next_batch(Misc& ms, const Batch& cur, bool have_cur, Batch& nxt, int& ti, uint32_t& tph,
                                    int* status) {
    const int lane = threadIdx.x & 31;
    if (have_cur && cur.tb + kNB * kTS < cur.t.end) {
      nxt.t = cur.t;
      nxt.tb = cur.tb + kNB * kTS;
      return true;
    }
    if (!warp_wait<true>(&ms.tfull[ti], tph, status, kStatusWaitTask)) return false;
    nxt.t = ms.tq[ti];
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.tempty[ti]);
    if (++ti == kTaskQ) {
      ti = 0;
      tph ^= 1u;
    }
    nxt.tb = nxt.t.begin;
    return nxt.t.valid != 0;
  }

  __device__ static void indexer(const DecodeLaunch& a, unsigned char* smem, Misc& ms) {
    const int lane = threadIdx.x & 31;
    int* status = a.d.status;
    int ti = 0, sd = 0;
    uint32_t tph = 0, sph = 0;
    Batch b, n;
    bool have = next_batch(ms, b, false, b, ti, tph, status);
    if (have) gather(a, b);
    bool ok = true;
    while (have && ok) {
      const bool have_next = next_batch(ms, b, true, n, ti, tph, status);
      if (have_next) gather(a, n);
#pragma unroll
      for (int i = 0; i < kNB; ++i) {
        const int t0 = b.tb + i * kTS;
        if (t0 >= b.t.end) break;
        ok = warp_wait<true>(&ms.sdempty[sd], sph ^ 1u, status, kStatusWaitDesc);
        if (!ok) break;
        int* page = reinterpret_cast<int*>(smem + kOffSD + sd * kSDEntry);
        int* row = page + kTS;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = u * 32 + lane;
          page[j] = b.phys[i][u];
          row[j] = b.inner[i][u];
        }
        if (lane == 0) {
          Hdr h;
          h.request = b.t.request;
          h.split = b.t.split;
          h.group = b.t.group;
          h.ntok = min(kTS, b.t.end - t0);
          h.flags = (t0 == b.t.begin ? kFlagFirst : 0) | (t0 + kTS >= b.t.end ? kFlagLast : 0);
          h.count_r = b.t.count_r;
          h.t0 = t0;
          h.pad = 0;
          ms.shdr[sd] = h;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms.sdfull[sd]);
        if (++sd == kSD) {
          sd = 0;
          sph ^= 1u;
        }
      }
      have = have_next;
      b = n;
    }
    if (!ok) return;
    if (!warp_wait(&ms.sdempty[sd], sph ^ 1u, status, kStatusWaitDesc)) return;
    if (lane == 0) {
      Hdr h{};
      h.flags = kFlagExit;
      ms.shdr[sd] = h;
      mbar_arrive(&ms.sdfull[sd]);
    }
    __syncwarp();
  }

  // ------------------------------------------------------------------ producers
  // 16-byte cp.async of one 128-token tile; rows at or past ntok are zero-filled (the PV
  // MMA multiplies them by P = 0, so they must hold finite values).
  // Thread (pw, lane) copies chunk c = lane % 16 of rows jt0 + 16k (jt0 = 2 pw + lane / 16):
  // rows 16 apart share the swizzle phase, so their offsets step by 16 rows of 128 bytes.
  // Row jt lives at page[jt] * st[0] + row[jt] * st[1] + group * st[2] elements (CSR: st[1] = 0).
  __device__ static void copy_tile(uint32_t dst, const T* base, const int* page, const int* row, const int64_t* st,
                                   int group, int ntok, int pw, int lane) {
    static_assert(kProducerWarps * 2 == 16, "eight producer warps cover 16 rows per step");
    const int c = lane & 15, jt0 = pw * 2 + (lane >> 4);
    const uint32_t d0 = dst + tile_off<kTS>(jt0, c);
    const T* base_c = base + static_cast<int64_t>(group) * st[2] + c * 8;
    const int64_t s0 = st[0], s1 = st[1];
#pragma unroll
    for (int k = 0; k < kTS / 16; ++k) {
      const int jt = jt0 + 16 * k;
      const bool live = jt < ntok;
      const T* src = live ? base_c + page[jt] * s0 + row[jt] * s1 : base;
      cp_async_16_fill(d0 + k * 16 * 128, src, live ? 16u : 0u);
    }
  }

  __device__ static void producer(const DecodeLaunch& a, unsigned char* smem, Misc& ms) {
    const int lane = threadIdx.x & 31;
    const int pw = (threadIdx.x >> 5) - kProducerWarp0;
    if (a.tma_kv && pw != 0) return;   // tensor-map copies are issued by producer 0 alone
    int* status = a.d.status;
    const T* kbase = static_cast<const T*>(a.d.k);
    const T* vbase = static_cast<const T*>(a.d.v);
    const bool lead = pw == 0 && lane == 0;
    int sd = 0, s = 0, qcount = 0, hs = 0;
    uint32_t sph = 0, ph = 0, hph = 0;
    bool ok = true;
    while (true) {
      ok = warp_wait<true>(&ms.sdfull[sd], sph, status, kStatusWaitDesc);
      if (!ok) break;
      const Hdr h = ms.shdr[sd];
      if (h.flags & kFlagExit) break;
      const int* page = reinterpret_cast<const int*>(smem + kOffSD + sd * kSDEntry);
      const int* prow = page + kTS;
      if ((h.flags & kFlagFirst) && pw == 0) {
        const int qb = qcount & 1;
        ok = warp_wait<true>(&ms.q_empty[qb], ((qcount >> 1) & 1) ^ 1u, status, kStatusWaitQ);
        if (!ok) break;
        if (lane == 0) {
          // A request past q's rows reads zeros: the box is out of bounds of the tensor map.
          if (h.request >= a.q_rows) atomicOr(status, kStatusQRows);
          const uint32_t qdst = smem_addr(smem + kOffQ + qb * kQBytes);
          mbar_arrive_expect_tx(&ms.q_full[qb], kQBytes);
          tma_load_3d(qdst, &a.qmap, 0, h.group * a.group_size, h.request, &ms.q_full[qb]);
          tma_load_3d(qdst + kQRows * 128, &a.qmap, 64, h.group * a.group_size, h.request, &ms.q_full[qb]);
        }
        __syncwarp();
      }
      if (h.flags & kFlagFirst) ++qcount;
      const uint32_t kdst = smem_addr(smem + s * kStage);
      const uint32_t vdst = kdst + kTile;
      const int nchunks = (h.ntok + 31) >> 5;   // TMA boxes of 32 tokens
      // ---- K tile
      ok = warp_wait<true>(&ms.empty_k[s], ph ^ 1u, status, kStatusWaitEmpty);
      if (!ok) break;
      if (a.tma_kv) {
        if (lane == 0) {
          ms.hdr[s] = h;
          mbar_arrive_expect_tx(&ms.full_k[s], static_cast<uint32_t>(nchunks * 32 * 256));
          for (int c = 0; c < nchunks; ++c) {
            const int j = c * 32;   // a box never crosses a page (32 divides the page size)
            tma_load_4d(kdst + j * 128, &a.kmap, 0, h.group, prow[j], page[j], &ms.full_k[s]);
            tma_load_4d(kdst + kHalf + j * 128, &a.kmap, 64, h.group, prow[j], page[j], &ms.full_k[s]);
          }
        }
        __syncwarp();
        mbar_arrive(&ms.full_k[s]);
      } else {
        copy_tile(kdst, kbase, page, prow, a.d.k_stride, h.group, h.ntok, pw, lane);
        cp_async_arrive_noinc(&ms.full_k[s]);
        if (lead) {
          ms.hdr[s] = h;
          mbar_arrive(&ms.full_k[s]);
        }
      }
      // ---- V tile
      ok = warp_wait<true>(&ms.empty_v[s], ph ^ 1u, status, kStatusWaitEmpty);
      if (!ok) break;
      if (a.tma_kv) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&ms.full_v[s], static_cast<uint32_t>(nchunks * 32 * 256));
          for (int c = 0; c < nchunks; ++c) {
            const int j = c * 32;
            tma_load_4d(vdst + j * 128, &a.vmap, 0, h.group, prow[j], page[j], &ms.full_v[s]);
            tma_load_4d(vdst + kHalf + j * 128, &a.vmap, 64, h.group, prow[j], page[j], &ms.full_v[s]);
          }
        }
        __syncwarp();
        mbar_arrive(&ms.full_v[s]);
      } else {
        copy_tile(vdst, vbase, page, prow, a.d.v_stride, h.group, h.ntok, pw, lane);
        cp_async_arrive_noinc(&ms.full_v[s]);
        if (lead) mbar_arrive(&ms.full_v[s]);
      }
      // ---- the softmax warps' copy of the header
      if (pw == 0) {
        ok = warp_wait<true>(&ms.hempty[hs], hph ^ 1u, status, kStatusWaitEmpty);
        if (!ok) break;
        if (lane == 0) {
          ms.xhdr[hs] = h;
          mbar_arrive(&ms.hfull[hs]);
        }
        if (++hs == kHdrQ) {
          hs = 0;
          hph ^= 1u;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.sdempty[sd]);
      if (++sd == kSD) {
        sd = 0;
        sph ^= 1u;
      }
      if (++s == kStages) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (!ok) return;
    // Exit markers: the MMA issuer's (data ring) and the softmax warps' (header ring).
    if (!warp_wait(&ms.empty_k[s], ph ^ 1u, status, kStatusWaitEmpty)) return;
    if (lead) {
      Hdr h{};
      h.flags = kFlagExit;
      ms.hdr[s] = h;
      mbar_arrive(&ms.full_k[s]);
    }
    mbar_arrive(&ms.full_k[s]);
    __syncwarp();
    if (pw == 0) {
      if (!warp_wait(&ms.hempty[hs], hph ^ 1u, status, kStatusWaitEmpty)) return;
      if (lane == 0) {
        Hdr h{};
        h.flags = kFlagExit;
        ms.xhdr[hs] = h;
        mbar_arrive(&ms.hfull[hs]);
      }
      __syncwarp();
    }
  }

  // ------------------------------------------------------------------ MMA issuer (lane 0)
  // An event loop over two in-order streams of work: QK of the next tile (its K tile has
  // landed, a score buffer is free; up to kSBufs tiles ahead of the softmax) and PV of the
  // oldest tile whose P is ready.  Neither waits for the other, so the tensor cores' latency
  // overlaps the softmax instead of adding to it.
  __device__ static void mma_issuer(const DecodeLaunch& a, unsigned char* smem, Misc& ms, uint32_t tmem) {
    int* status = a.d.status;
    constexpr uint32_t bf = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t idesc_qk = mma_idesc(bf, 0u, 0u, 16u, 128u);
    constexpr uint32_t idesc_pv = mma_idesc(bf, 1u, 1u, 16u, 128u);
    int sq = 0, tq = 0, tp = 0, qtask = 0;
    uint32_t phq = 0;
    bool exit_seen = false;
    uint64_t deadline = global_timer_ns() + kWaitLimitNs;
    int idle = 0;
    while (!(exit_seen && tp == tq)) {
      bool progressed = false;
      // ---- QK of tile tq
      if (!exit_seen && tq - tp < kSBufs && mbar_test_wait(&ms.full_k[sq], phq)) {
        const Hdr h = ms.hdr[sq];
        if (h.flags & kFlagExit) {
          exit_seen = true;
          progressed = true;
        } else {
          const bool first = (h.flags & kFlagFirst) != 0;
          const int task = first ? qtask : qtask - 1, qb = task & 1;
          if ((!first || mbar_test_wait(&ms.q_full[qb], (task >> 1) & 1)) &&
              mbar_test_wait(&ms.s_free[tq & (kSBufs - 1)], ((tq / kSBufs) & 1) ^ 1u)) {
            if (first) ++qtask;
            if (!a.tma_kv) fence_proxy_async_smem();   // cp.async rows arrived through the generic proxy
            tc_fence_after();
            const uint32_t kb = smem_addr(smem + sq * kStage);
            const uint32_t qbase = smem_addr(smem + kOffQ + qb * kQBytes);
            const uint32_t d = tmem + (tq & (kSBufs - 1)) * 16;
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks)
              mma_f16(d, smem_desc(kb + (ks >> 2) * kHalf + (ks & 3) * 32, 16, 1024, 2),
                      smem_desc(qbase + (ks >> 2) * (kQRows * 128) + (ks & 3) * 32, 16, 1024, 2), idesc_qk,
                      ks > 0 ? 1u : 0u);
            mma_commit(&ms.s_full[tq & (kSBufs - 1)]);
            mma_commit(&ms.empty_k[sq]);
            if (h.flags & kFlagLast) mma_commit(&ms.q_empty[qb]);
            ms.pend[tq & (kSBufs - 1)] = make_int4(sq, static_cast<int>(phq), task, h.flags);
            ++tq;
            if (++sq == kStages) {
              sq = 0;
              phq ^= 1u;
            }
            progressed = true;
          }
        }
      }
      // ---- PV of tile tp
      if (tp < tq) {
        const int4 u = ms.pend[tp & (kSBufs - 1)];   // stage, phase, task, flags
        const bool first = (u.w & kFlagFirst) != 0;
        const int ob = u.z & 1;
        if (mbar_test_wait(&ms.p_full[tp % kPBufs], (tp / kPBufs) & 1) && mbar_test_wait(&ms.full_v[u.x], u.y) &&
            (!first || mbar_test_wait(&ms.o_free[ob], ((u.z >> 1) & 1) ^ 1u))) {
          if (!a.tma_kv) fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t vb = smem_addr(smem + u.x * kStage + kTile);
          const uint32_t pb = smem_addr(smem + kOffP + (tp % kPBufs) * kPBytes);
          const uint32_t d = tmem + 64 + ob * 16;
#pragma unroll
          for (int ks = 0; ks < kTS / 16; ++ks)
            mma_f16(d, smem_desc(vb + ks * 2048, kHalf, 1024, 2), smem_desc(pb + ks * 512, 256, 128, 0), idesc_pv,
                    (first && ks == 0) ? 0u : 1u);
          mma_commit(&ms.empty_v[u.x]);
          mma_commit(&ms.p_free[tp % kPBufs]);
          if (u.w & kFlagLast) mma_commit(&ms.o_full[ob]);
          ++tp;
          progressed = true;
        }
      }
      if (progressed) {
        idle = 0;
      } else {
        __nanosleep(32);   // leave the issue slots to the softmax warp on this sub-partition
        if ((++idle & 63) == 0) {
          if (idle == 64) deadline = global_timer_ns() + kWaitLimitNs;
          else if (global_timer_ns() > deadline) {
            atomicOr(status, kStatusWaitFull);
            break;
          }
        }
      }
    }
    // Wait until every MMA this thread issued has completed (tensor memory is released after).
    mma_commit(&ms.drain);
    wait_bar(&ms.drain, 0, status, kStatusWaitFull);
  }

  // ------------------------------------------------------------------ softmax (8 warps)
  // Warp w covers TMEM quadrant q = w % 4 (lanes 32q..32q+31: tokens of the scores, dims of
  // the output) and head columns [g*NHW, g*NHW + NHW) with g = w / 4.  The two column groups
  // share the tile stream and nothing else: each keeps its own joins, reference maxima, row
  // sums, rescaling and epilogue.

  // Reduction over the warp of x[i] per column i (max or sum); afterwards lane l holds column
  // reduced_col(l) (transposed butterfly: each exchange halves the columns a lane keeps).
  template <bool kSum>
  __device__ static float warp_reduce_cols(const float (&x)[NHW]) {
    const int lane = threadIdx.x & 31;
    float v[NHW];
#pragma unroll
    for (int i = 0; i < NHW; ++i) v[i] = x[i];
    auto op = [](float p, float q) { return kSum ? p + q : fmaxf(p, q); };
#pragma unroll
    for (int width = NHW / 2, bit = 16; width >= 1; width >>= 1, bit >>= 1) {
      const bool upper = (lane & bit) != 0;
#pragma unroll
      for (int i = 0; i < width; ++i) {
        const float send = upper ? v[i] : v[i + width];
        const float keep = upper ? v[i + width] : v[i];
        v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, bit));
      }
    }
    // log2(NHW) exchanges used lane bits 16 .. 32/NHW; finish over the lower bits.
    float r = v[0];
#pragma unroll
    for (int bit = 16 / NHW; bit >= 1; bit >>= 1) r = op(r, __shfl_xor_sync(0xffffffffu, r, bit));
    return r;
  }

  __device__ static int reduced_col(int lane) { return lane / (32 / NHW); }
  __device__ static bool col_writer(int lane) { return (lane % (32 / NHW)) == 0; }

  // Task end: normalise this warp's columns of O^T and store partial rows and LSE.  Out of
  // line: it runs once per task, and the kernel's instruction footprint is a measured stall.
  __device__ __noinline__ static bool epilogue(const DecodeLaunch& a, Misc& ms, uint32_t tmem, const Hdr& h, int task,
                                  const float (&m)[NHW], const float (&lsum)[NHW]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3, g = warp >> 2;
    int* status = a.d.status;
    const int ob = task & 1;
    if (!warp_wait(&ms.o_full[ob], (task >> 1) & 1, status, kStatusWaitFull)) return false;
    tc_fence_after();
    float o[NHW];
    tmem_ld<NHW>(tmem + (static_cast<uint32_t>(q * 32) << 16) + 64 + ob * 16 + g * NHW, o);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.o_free[ob]);
    const float wl = warp_reduce_cols<true>(lsum);
    if (col_writer(lane)) ms.red_l[ob][q][g * NHW + reduced_col(lane)] = wl;
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.join_l[g][ob]);
    if (!warp_wait(&ms.join_l[g][ob], (task >> 1) & 1, status, kStatusWaitFull)) return false;
    const int gs = a.group_size, smax = a.smax;
    const int64_t slot0 = (static_cast<int64_t>(h.request) * a.d.query_heads + h.group * gs) * smax + h.split;
#pragma unroll
    for (int i = 0; i < NHW; ++i) {
      const int head = g * NHW + i;
      if (head < gs) {
        const float l = ms.red_l[ob][0][head] + ms.red_l[ob][1][head] + ms.red_l[ob][2][head] + ms.red_l[ob][3][head];
        const int64_t slot = slot0 + static_cast<int64_t>(head) * smax;
        a.d.partial[slot * kD + q * 32 + lane] = o[i] * __fdividef(a.d.v_scale, l);
        if (q == 0 && lane == i) a.d.lse[slot] = (m[i] + lg2(l)) * kLn2;
      }
    }
    return true;
  }

  // The running maximum of some head grew by more than 2^kRescaleLog2: once the previous
  // tile's PV has completed, scale this warp's lanes of the group's O columns (and the row
  // sums) to the new maxima.  Rare; out of line.
  __device__ __noinline__ static bool rescale(const DecodeLaunch& a, Misc& ms, uint32_t taddr, int tile,
                                              const float (&tmax)[NHW], float (&m_ref)[NHW], float (&lsum)[NHW]) {
    if (!warp_wait(&ms.p_free[(tile - 1) % kPBufs], ((tile - 1) / kPBufs) & 1, a.d.status, kStatusWaitFull))
      return false;
    tc_fence_after();
    float o[NHW];
    tmem_ld<NHW>(taddr, o);
#pragma unroll
    for (int i = 0; i < NHW; ++i) {
      const float mn = fmaxf(m_ref[i], tmax[i]);
      const float alpha = ex2(m_ref[i] - mn);
      o[i] *= alpha;
      lsum[i] *= alpha;
      m_ref[i] = mn;
    }
    tmem_st<NHW>(taddr, o);
    return true;
  }

  __device__ static void softmax(const DecodeLaunch& a, unsigned char* smem, Misc& ms, uint32_t tmem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3, g = warp >> 2;
    int* status = a.d.status;
    const float cap = a.d.logit_cap;
    const bool capped = cap > 0.f;
    const float sc = (capped ? a.d.scale : a.d.scale * kLog2e) * a.d.k_scale;
    const float cap_log2e = cap * kLog2e, two_log2e_over_cap = capped ? 2.f * kLog2e / cap : 0.f;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const int tok = q * 32 + lane, col0 = g * NHW;
    float m_ref[NHW], lsum[NHW];
#pragma unroll
    for (int i = 0; i < NHW; ++i) m_ref[i] = 0.f, lsum[i] = 0.f;
    // The previous task's epilogue runs after the next tile's P is published, so the wait
    // for its last PV overlaps that tile.
    bool pending = false;
    Hdr ph{};
    int ptask = 0;
    float pm[NHW], pl[NHW];
    int tile = 0, task = 0, hs = 0, s = 0;
    uint32_t hph = 0, ph_v = 0;
    while (true) {
      if (!warp_wait(&ms.hfull[hs], hph, status, kStatusWaitFull)) return;
      const Hdr h = ms.xhdr[hs];
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.hempty[hs]);
      if (++hs == kHdrQ) {
        hs = 0;
        hph ^= 1u;
      }
      if (h.flags & kFlagExit) break;
      const bool first = (h.flags & kFlagFirst) != 0;
      // ---- scores of this warp's 32 tokens and NHW heads
      const int sb = tile & (kSBufs - 1);
      if (!warp_wait(&ms.s_full[sb], (tile / kSBufs) & 1, status, kStatusWaitFull)) return;
      tc_fence_after();
      float x[NHW];
      tmem_ld<NHW>(tmem + lane_base + sb * 16 + col0, x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.s_free[sb]);
      const bool valid = tok < h.ntok;
#pragma unroll
      for (int i = 0; i < NHW; ++i) {
        float y = x[i] * sc;
        if (capped) y = cap_log2e * (1.f - 2.f / (ex2(y * two_log2e_over_cap) + 1.f));
        x[i] = valid ? y : -INFINITY;
      }
      // ---- tile maximum per head over the 128 tokens (four quadrants of this group)
      const float wmax = warp_reduce_cols<false>(x);
      const int jb = tile & 1;
      if (col_writer(lane)) ms.red[jb][q][col0 + reduced_col(lane)] = wmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.join[g][jb]);
      if (!warp_wait(&ms.join[g][jb], (tile >> 1) & 1, status, kStatusWaitFull)) return;
      float tmax[NHW];
#pragma unroll
      for (int i = 0; i < NHW; ++i)
        tmax[i] = fmaxf(fmaxf(ms.red[jb][0][col0 + i], ms.red[jb][1][col0 + i]),
                        fmaxf(ms.red[jb][2][col0 + i], ms.red[jb][3][col0 + i]));
      if (first) {
#pragma unroll
        for (int i = 0; i < NHW; ++i) m_ref[i] = tmax[i], lsum[i] = 0.f;
      } else {
        bool grow = false;
#pragma unroll
        for (int i = 0; i < NHW; ++i) grow |= tmax[i] > m_ref[i] + kRescaleLog2;
        if (grow) {   // uniform over the group (same maxima): rescale its O columns in TMEM
          if (!rescale(a, ms, tmem + lane_base + 64 + (task & 1) * 16 + col0, tile, tmax, m_ref, lsum)) return;
        }
      }
      // ---- P = 2^(x - m): this group's heads of the token's 16-head row of the B operand
      //      (MN-major, no swizzle: token blocks of 8 are 256 bytes apart, heads 8-15 at +128)
      if (!warp_wait(&ms.p_free[tile % kPBufs], ((tile / kPBufs) & 1) ^ 1u, status, kStatusWaitFull)) return;
      uint32_t pk[NHW / 2];
#pragma unroll
      for (int i = 0; i < NHW; i += 2) {
        const float p0 = valid ? ex2(x[i] - m_ref[i]) : 0.f;
        const float p1 = valid ? ex2(x[i + 1] - m_ref[i + 1]) : 0.f;
        lsum[i] += p0;
        lsum[i + 1] += p1;
        pk[i / 2] = Mma<T>::pack(p0, p1);
      }
      unsigned char* prow = smem + kOffP + (tile % kPBufs) * kPBytes + (tok >> 3) * 256 + (tok & 7) * 16 +
                            (col0 >> 3) * 128 + (col0 & 7) * 2;
      if constexpr (NHW == 8) {
        *reinterpret_cast<uint4*>(prow) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      } else if constexpr (NHW == 4) {
        *reinterpret_cast<uint2*>(prow) = make_uint2(pk[0], pk[1]);
      } else {
        *reinterpret_cast<uint32_t*>(prow) = pk[0];
      }
      // Rows of V past the tile's last token must be finite (P = 0 multiplies them): the
      // cp.async path zero-fills them; with tensor-map boxes the two groups clear the row.
      if (a.tma_kv && h.ntok < kTS) {
        if (!warp_wait(&ms.full_v[s], ph_v, status, kStatusWaitFull)) return;
        if (!valid) {
          unsigned char* vt = smem + s * kStage + kTile;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(vt + tile_off<kTS>(tok, g * 8 + c)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.p_full[tile % kPBufs]);
      if (pending) {
        if (!epilogue(a, ms, tmem, ph, ptask, pm, pl)) return;
        pending = false;
      }
      if (h.flags & kFlagLast) {
        pending = true;
        ph = h;
        ptask = task;
#pragma unroll
        for (int i = 0; i < NHW; ++i) pm[i] = m_ref[i], pl[i] = lsum[i];
        ++task;
      }
      ++tile;
      if (++s == kStages) {
        s = 0;
        ph_v ^= 1u;
      }
    }
    if (pending) epilogue(a, ms, tmem, ph, ptask, pm, pl);
  }

  // ------------------------------------------------------------------ entry
  __device__ static void run(const DecodeLaunch& a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
      const int producers = a.tma_kv ? 1 : kProducerWarps;
      for (int i = 0; i < kStages; ++i) {
        mbar_init(&ms.full_k[i], 32 * producers + 1);
        mbar_init(&ms.full_v[i], 32 * producers + 1);
        mbar_init(&ms.empty_k[i], 1);
        mbar_init(&ms.empty_v[i], 1);
      }
      for (int i = 0; i < kSBufs; ++i) {
        mbar_init(&ms.s_full[i], 1);
        mbar_init(&ms.s_free[i], kSoftmaxWarps);
      }
      for (int i = 0; i < kPBufs; ++i) {
        mbar_init(&ms.p_full[i], kSoftmaxWarps);
        mbar_init(&ms.p_free[i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&ms.q_full[i], 1);
        mbar_init(&ms.q_empty[i], 1);
        mbar_init(&ms.o_full[i], 1);
        mbar_init(&ms.o_free[i], kSoftmaxWarps);
        for (int g = 0; g < 2; ++g) {
          mbar_init(&ms.join[g][i], kSoftmaxWarps / 2);
          mbar_init(&ms.join_l[g][i], kSoftmaxWarps / 2);
        }
      }
      for (int i = 0; i < kTaskQ; ++i) {
        mbar_init(&ms.tfull[i], 1);
        mbar_init(&ms.tempty[i], 1);
      }
      for (int i = 0; i < kSD; ++i) {
        mbar_init(&ms.sdfull[i], 1);
        mbar_init(&ms.sdempty[i], producers);
      }
      for (int i = 0; i < kHdrQ; ++i) {
        mbar_init(&ms.hfull[i], 1);
        mbar_init(&ms.hempty[i], kSoftmaxWarps);
      }
      mbar_init(&ms.drain, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // P columns past the heads the softmax writes stay zero for the whole launch.
    for (int i = threadIdx.x; i < kPBufs * kPBytes / 16; i += kThreads)
      reinterpret_cast<uint4*>(smem + kOffP)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    if (warp == kMmaWarp) tmem_alloc(smem_addr(&ms.tmem_base), kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    // Programmatic dependent launch: everything above overlapped the previous kernel.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (warp < kSoftmaxWarps) {
      softmax(a, smem, ms, tmem);
    } else if (warp == kMmaWarp) {
      if (lane == 0) mma_issuer(a, smem, ms, tmem);
      __syncwarp();
    } else if (warp < kIndexerWarp) {
      producer(a, smem, ms);
    } else if (warp == kIndexerWarp) {
      indexer(a, smem, ms);
    } else {
      if (lane == 0) scheduler(a, ms);
      __syncwarp();
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
    // The merge launched after this kernel zeroes the claim words once this grid completes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }
};

template <typename T, int NHW>
__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(const __grid_constant__ DecodeLaunch a) {
  TcKernel<T, NHW>::run(a);
}

template <typename T, int NHW>
cudaError_t launch_tc_typed(const DecodeLaunch& a, cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  static std::atomic<void*> configured[kMaxDevices] = {};   // context the attribute was set in
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  void* ctx = current_context();
  if (ctx == nullptr || configured[device].load(std::memory_order_acquire) != ctx) {
    e = cudaFuncSetAttribute(decode_tc_kernel<T, NHW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[device].store(ctx, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.workers);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_tc_kernel<T, NHW>, a);
}

}  // namespace

cudaError_t launch_decode_tc(const DecodeLaunch& a, cudaStream_t stream) {
  const int g = a.group_size;   // head columns per softmax warp: half the padded group
  if (a.d.dtype == SGLD_DTYPE_BF16) {
    if (g <= 4) return launch_tc_typed<__nv_bfloat16, 2>(a, stream);
    return g <= 8 ? launch_tc_typed<__nv_bfloat16, 4>(a, stream) : launch_tc_typed<__nv_bfloat16, 8>(a, stream);
  }
  if (g <= 4) return launch_tc_typed<__half, 2>(a, stream);
  return g <= 8 ? launch_tc_typed<__half, 4>(a, stream) : launch_tc_typed<__half, 8>(a, stream);
}

}  // namespace sgld
