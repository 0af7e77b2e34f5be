/*
 * sgld_b200.h -- C ABI of the B200 (sm_100a) paged GQA decode hot path.
 *
 * Drop-in replacement for the GPU work of StrongObserver/-SGLang-Decode-
 * (package ``sglang_decode``).  Every entry point below replaces one group of
 * Triton launches of the reference; the comment of each names the reference
 * interface (file:line, paths inside the reference project).
 *
 * Conventions
 *  - All pointers are DEVICE pointers unless stated otherwise; every buffer is
 *    owned by the caller.  No function allocates, frees or synchronises;
 *    sgld_plan_build, sgld_decode_persistent and sgld_merge_splits can be captured
 *    into a CUDA graph.
 *  - `stream` is a cudaStream_t passed as void*; work is enqueued in stream order.
 *  - Return value: an sgld_status.  Non-zero means nothing was enqueued; the
 *    message is available from sgld_last_error() (thread-local).
 *  - Integer metadata is int32, strides are in ELEMENTS (int64).
 *  - Device-side problems never trap: invalid plan metadata sets plan->error
 *    and turns every output row into NaN (as the reference does); a bounded
 *    in-kernel wait that expires sets a non-zero word in `status`.
 */
#ifndef SGLD_B200_H
#define SGLD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SGLD_ABI_VERSION 9

typedef enum sgld_status {
  SGLD_OK = 0,
  SGLD_ERR_INVALID_ARGUMENT = 1, /* shape / capacity / pointer / stride check failed */
  SGLD_ERR_UNSUPPORTED = 2,      /* geometry outside this build (e.g. head_dim 96)   */
  SGLD_ERR_CUDA = 3              /* a launch failed; see sgld_last_error()           */
} sgld_status;

enum { SGLD_DTYPE_F16 = 0, SGLD_DTYPE_BF16 = 1, SGLD_DTYPE_E4M3 = 2 /* K/V only: fp8 e4m3 */ };

/* Execution modes -- reference src/sglang_decode/config.py:6-11. */
enum { SGLD_MODE_R0 = 0, SGLD_MODE_R1 = 1, SGLD_MODE_STATIC = 2, SGLD_MODE_D1 = 3, SGLD_MODE_D4 = 4 };

/* Capacity contract -- reference config.py:14-58 (the fields the planner reads).
 * groups = tasks per record = KV heads owned by this GPU. */
typedef struct sgld_plan_geometry {
  int32_t batch_capacity; /* Bcap                                     */
  int32_t max_splits;     /* Smax                                     */
  int32_t max_context;    /* longest admissible request               */
  int32_t groups;         /* KV heads handled by this plan            */
  int32_t workers;        /* persistent decode CTAs (grid size)       */
} sgld_plan_geometry;

/* Plan buffers -- reference runtime/workspace.py:7-23 (PlanBuffers).
 * Sizes: B = batch_capacity, E = B*max_splits, T = E*groups, W = workers. */
typedef struct sgld_plan_buffers {
  int32_t* lengths;      /* [B]   caller-written context lengths        */
  int32_t* splits;       /* [B]   caller-written requested split counts */
  int32_t* active;       /* [1]   caller-written active batch size      */
  int32_t* counts;       /* [B]   records per request                   */
  int32_t* offsets;      /* [B+1] exclusive prefix of counts            */
  int32_t* chunk;        /* [B]   split chunk per request               */
  int32_t* request;      /* [E]   SoA records ...                       */
  int32_t* split;        /* [E]                                         */
  int32_t* begin;        /* [E]                                         */
  int32_t* end;          /* [E]                                         */
  int32_t* weight;       /* [E]   ceil((end-begin)/128)                 */
  int32_t* order;        /* [E]   record permutation (bucket order)     */
  int32_t* pack_first;   /* [T]   first task of each pack               */
  int32_t* pack_count;   /* [T]   tasks in each pack                    */
  int32_t* record_count; /* [1]                                         */
  int32_t* num_packs;    /* [1]                                         */
  int32_t* mode;         /* [1]   mode chosen for this step             */
  int32_t* error;        /* [1]   non-zero: invalid metadata            */
  int32_t* static_head;  /* [W]   STATIC list heads                     */
  int32_t* static_next;  /* [T]   STATIC list links                     */
  int32_t* arrivals;     /* [B*groups] split arrivals per (request, KV head) of the small-batch
                            kernel's fused merge: zeroed by every plan build and left zero by
                            every decode (an addition: no reference counterpart)            */
} sgld_plan_buffers;

/*
 * One int32 storage for every plan buffer: the number of int32 words it needs, and the
 * sgld_plan_buffers that views it (buffers in declaration order, sizes as above).  Lets a caller
 * allocate and pass the plan as a single array.  No counterpart in the reference (its
 * PlanBuffers are separate tensors, runtime/workspace.py:7-23).
 */
size_t sgld_plan_storage_words(const sgld_plan_geometry* geometry);
int sgld_plan_buffers_in_storage(int32_t* storage, const sgld_plan_geometry* geometry, sgld_plan_buffers* out);

/*
 * Build the step's task table on the GPU (one launch, one CTA).
 * Replaces reference planning/builder.py:6-28 (build_plan: count_scan,
 * emit_records, make_order_and_packs, greedy_lists of kernels/plan.py:7-135).
 *
 *  force_mode      -1 = AUTO (rules, else R1), 0..4 forces a mode.
 *  rules           device int32 [n_rules, 5] rows (min_tasks, max_tasks, min_ratio,
 *                  max_ratio, mode); may be NULL when n_rules == 0.
 *  layer_counters  device int32 words zeroed by this launch (the per-layer claim
 *                  counters of the decode launches that follow); may be NULL.
 */
int sgld_plan_build(const sgld_plan_buffers* plan, const sgld_plan_geometry* geometry,
                    int32_t force_mode, const int32_t* rules, int32_t n_rules,
                    int32_t* layer_counters, int32_t n_counter_words, void* stream);

/* Attention geometry and tensors of one decode launch. */
typedef struct sgld_decode_args {
  const void* q;        /* [B, Hq, D] fp16/bf16, strides q_stride                            */
  const void* k;        /* paged [P, page_size, Hkv, D] / CSR [N, Hkv, D], strides k_stride    */
  const void* v;        /* same shape as k, strides v_stride                                  */
  void* out;            /* [B, Hq, D] contiguous, same dtype as q                             */
  const int32_t* pages; /* paged: page table [B, max_pages] (pt_stride); CSR: kv_indices      */
  const int32_t* indptr;/* CSR: [B+1] row pointers into kv_indices; NULL selects paged       */
  int64_t q_stride[3];  /* elements                                                          */
  int64_t k_stride[4];  /* (page, token-in-page, head, dim); CSR: (token, 0, head, dim)      */
  int64_t v_stride[4];
  int64_t pt_stride[2]; /* page table strides (paged only)                                   */
  int64_t kv_extent;    /* paged: pages in k/v; CSR: token slots in k/v; 0 if unknown. Bounds
                           the tensor-map (TMA) copies of the paged path                      */
  int32_t dtype;        /* SGLD_DTYPE_*                                                      */
  int32_t query_heads;  /* Hq on this GPU                                                    */
  int32_t kv_heads;     /* Hkv on this GPU (== plan groups)                                  */
  int32_t head_dim;     /* 64, 128 or 256                                                    */
  int32_t page_size;    /* 1 for CSR                                                         */
  float scale;          /* softmax scale (reference default head_dim^-0.5)                   */
  float logit_cap;      /* > 0: each scaled score s becomes logit_cap * tanh(s / logit_cap)
                           before the softmax (SGLang's soft cap, upstream
                           decode_attention.py:127-128); 0 disables it; not in the
                           reference's own kernel (its adapter falls back)              */
  int32_t kv_dtype;     /* dtype of k and v: == dtype, or SGLD_DTYPE_E4M3 (fp8 K/V with a
                           fp16/bf16 q; head_dim 128).  The reference has no fp8 path      */
  float k_scale;        /* scores use k_scale * k (0 reads as 1): dequantises fp8 keys      */
  float v_scale;        /* outputs use v_scale * v (0 reads as 1)                           */
  int32_t q_rows;       /* rows of q (and of k_new / v_new / new_loc); 0 means batch_capacity.
                           The plan's active count must not exceed it: a task of a request at
                           or past q_rows reads a zero query and sets status bit 64          */
  /* KV-cache write: SGLang's set_kv_buffer, the step before the decode (reference
     integrations/sglang_backend.py:91-92), chained into this call.  With new_loc
     non-NULL, row r < q_rows of k_new / v_new ([q_rows, Hkv, D] in `dtype`, any strides)
     is stored at token slot new_loc[r] of k / v (paged: page new_loc/page_size, row
     new_loc%page_size) before the decode reads the pool, so the result is exactly the
     write followed by the decode.  An e4m3 pool stores e4m3(x / k_scale) (v: v_scale),
     rounded to nearest even and saturated to +-448.  A slot outside kv_extent is
     skipped and sets status bit 128.                                                     */
  const void* k_new;
  const void* v_new;
  const void* new_loc;  /* [q_rows] int64, or int32 when new_loc_int32 != 0                 */
  int64_t knew_stride[3];  /* elements: (request, head, dim)                               */
  int64_t vnew_stride[3];
  int32_t new_loc_int32;
  /* Layer scratch -- reference runtime/workspace.py:26-40 (LayerBuffers) */
  int32_t* counter;     /* [2]  claim counter + spare word; zero before, zeroed by the merge */
  float* partial;       /* [B, Hq, Smax, D] fp32 normalised split outputs, 16-byte aligned   */
  float* lse;           /* [B, Hq, Smax]    fp32 natural-log LSE per split                   */
  int32_t* status;      /* [1]  0 = ok; otherwise sticky error bits: 1-32 a bounded in-kernel
                           wait expired, 64 q_rows too small, 128 a new_loc slot out of range */
} sgld_decode_args;

/*
 * Persistent paged GQA decode followed by the split merge (two launches: W decode
 * CTAs, then the merge grid as a programmatic dependent launch; with new_loc set, the
 * KV-cache write is a third launch chained right before the decode).
 * Replaces reference runtime/engine.py:62-73: the counter reset, the
 * persistent_decode launch (kernels/attention.py:87-130, task body :12-84) and
 * the merge_splits launch (kernels/merge.py:7-30).  Task dispatch follows
 * plan->mode exactly (R0 prefix search, R1 stride, STATIC lists, D1/D4 atomic
 * pack claims); each task writes its normalised partial and LSE to slot
 * (request*Hq + head)*Smax + split; the merge combines each row's splits in split
 * order into `out`.  Rows with no record are written as zeros, or NaN when
 * plan->error is set.  The merge launch leaves args->counter zero for the next call; a call
 * that returns an error may leave it non-zero (zero it, or pass it to the next
 * sgld_plan_build as a layer counter, before reusing it).
 */
int sgld_decode_persistent(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                           const sgld_plan_geometry* geometry, void* stream);

/*
 * Stand-alone split merge over (partial, lse) -- reference kernels/merge.py:7-30
 * (launched at runtime/engine.py:71-73).  out [B, Hq, D] in `dtype`.
 */
int sgld_merge_splits(const float* partial, const float* lse, const int32_t* counts,
                      const int32_t* error, void* out, int32_t dtype, int32_t batch_capacity,
                      int32_t query_heads, int32_t head_dim, int32_t max_splits, void* stream);

/*
 * Allocation-free variant of sgld_decode_persistent (no counterpart in the reference).
 * For callers that cannot allocate device memory: plugin interfaces that pass only input
 * and output buffers, or servers that give all device memory to their KV-cache pool at
 * start-up (cudaMalloc would also synchronise the device inside the serving loop).  The
 * decode's scratch (two claim words, fp32 partials and LSEs) lives in a 16 MiB
 * device array owned by the library on every GPU that loads it; args->counter, ->partial
 * and ->lse are ignored.  args->status must be a caller-owned device word (NULL is
 * rejected): bounded-wait and slot errors are reported there, as for
 * sgld_decode_persistent.  A geometry is accepted when
 *     256 + round_up(Bcap*Hq*Smax*D*4, 256) + round_up(Bcap*Hq*Smax*4, 256) <= 16 MiB
 * (Bcap = batch_capacity, Hq = query_heads, Smax = max_splits, D = head_dim); larger ones
 * return SGLD_ERR_INVALID_ARGUMENT.  Every argument is checked before anything is
 * enqueued.  Nothing is allocated.  The first call on a device (and the first after a
 * device reset) looks up the array's device address: make it before any stream capture.
 * All calls share the array: calls whose GPU work overlaps race and must be serialised by
 * the caller.
 */
int sgld_decode_persistent_noalloc(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                                   const sgld_plan_geometry* geometry, void* stream);

/* Decode kernels (see sgld_decode_kernel_kind). */
enum {
  SGLD_KERNEL_MMA_SYNC = 0,      /* mma.sync kernel, cp.async or element copies of K/V rows        */
  SGLD_KERNEL_TCGEN05 = 1,       /* tcgen05.mma kernel, TMEM accumulators, cp.async K/V rows        */
  SGLD_KERNEL_TCGEN05_TMA = 2,   /* tcgen05.mma kernel, paged K/V by tensor-map TMA boxes           */
  SGLD_KERNEL_MMA_SYNC_TMA = 3,  /* mma.sync kernel, paged K/V by tensor-map TMA boxes              */
  SGLD_KERNEL_SMALL = 4          /* small-batch kernel: one CTA per task of the task capacity       */
};

/*
 * Which decode kernel sgld_decode_persistent would launch for these arguments (an
 * SGLD_KERNEL_* value), or minus an sgld_status when the arguments are invalid.  Nothing is
 * enqueued.  By default a geometry whose task capacity (batch_capacity * max_splits *
 * kv_heads) is at most 1024 uses the small-batch kernel (head_dim 128, 16-bit K/V, group <= 8,
 * 16-byte aligned rows) and every other one the persistent mma.sync kernel; the environment
 * variable SGLD_DECODE_KERNEL=mma|small|tcgen05 forces a kernel where it applies (the tcgen05
 * kernel: head_dim 128, 16-bit K/V, 16-byte aligned rows).  No counterpart in the reference
 * (its only kernel is the Triton one).
 */
int sgld_decode_kernel_kind(const sgld_decode_args* args, const sgld_plan_buffers* plan,
                            const sgld_plan_geometry* geometry);

/* Bytes of per-layer scratch (counter, partial, lse, status) for one decode
 * layer -- reference runtime/workspace.py:33-40 (LayerBuffers.allocate). */
size_t sgld_layer_workspace_bytes(int32_t batch_capacity, int32_t query_heads, int32_t kv_heads,
                                  int32_t head_dim, int32_t max_splits);

/* Thread-local message of the last non-zero status returned on this host thread. */
const char* sgld_last_error(void);

/* SGLD_ABI_VERSION of the loaded library. */
int32_t sgld_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SGLD_B200_H */
