"""CPU restatement of the reference's task-table planning (test infrastructure only).

Two layers are restated here:

1. The host specification, ``src/sglang_decode/planning/reference.py``:
   ``split_records`` (:15-30), ``bucket_order`` (:33-34), ``make_packs`` (:37-54),
   ``greedy_static`` (:57-67) and ``validate_plan`` (:70-76).
2. The exact device-table semantics of the reference's Triton plan kernels,
   ``src/sglang_decode/kernels/plan.py`` -- ``count_scan`` (:7-27),
   ``emit_records`` (:30-45), ``make_order_and_packs`` (:48-100) and
   ``greedy_lists`` (:103-135) -- as sequenced by ``planning/builder.py:6-28``.
   ``device_tables`` returns every buffer those kernels write, including the
   error flag for invalid metadata, AUTO rule evaluation, the uniform->R1
   override, the forced-mode override and the GPU LPT linked lists.

Everything is pure Python integer arithmetic; int32 wrap-around is emulated where
the Triton kernels compute in int32.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

BLOCK_KV = 128          # config.py:24 -- tile size, also the weight unit
SPLIT_ALIGNMENT = 32    # config.py:25 -- split chunk alignment
INT32_MAX = 2**31 - 1


def _i32(x: int) -> int:
    """Wrap an integer to int32 the way Triton int32 arithmetic does."""
    x &= 0xFFFFFFFF
    return x - (1 << 32) if x & 0x80000000 else x


def _cdiv(a: int, b: int) -> int:
    """tl.cdiv on int32 operands: (a + b - 1) // b with int32 wrap of the sum."""
    return _i32(_i32(a + b - 1) // b) if b > 0 else 0


@dataclass(frozen=True)
class Record:
    """One (request, split) record -- planning/reference.py:6-12."""
    request: int
    split: int
    begin: int
    end: int
    weight: int


@dataclass(frozen=True)
class Geometry:
    """The subset of DecodeConfig the planner reads (config.py:14-58).

    ``groups`` is the number of tasks per record, i.e. the KV heads handled by this
    GPU (``kv_heads`` in the reference config; Hkv/N under head sharding).
    """
    batch_capacity: int
    max_splits: int
    max_context: int
    groups: int
    workers: int

    @property
    def record_capacity(self) -> int:       # config.py:44-46
        return self.batch_capacity * self.max_splits

    @property
    def task_capacity(self) -> int:         # config.py:48-50
        return self.record_capacity * self.groups

    @property
    def buckets(self) -> int:               # config.py:56-58
        return ((self.max_context + BLOCK_KV - 1) // BLOCK_KV - 1).bit_length() + 1


# --------------------------------------------------------------------------------------
# 1. Host specification (planning/reference.py)
# --------------------------------------------------------------------------------------

def split_chunk(length: int, splits: int) -> int:
    """Per-request split chunk: ceil(ceil(L/S)/32)*32 (planning/reference.py:22)."""
    per_split = -(-length // splits)
    return -(-per_split // SPLIT_ALIGNMENT) * SPLIT_ALIGNMENT


def split_records(lengths, requested_splits, geometry):
    """Records, per-request counts and exclusive offsets (planning/reference.py:15-30).

    Raises ValueError on a batch larger than the capacity or an invalid length or
    split count, exactly as the reference's CPU spec does.
    """
    if len(lengths) != len(requested_splits) or len(lengths) > geometry.batch_capacity:
        raise ValueError("batch/split shape exceeds the capture contract")
    records, counts, offsets = [], [], [0]
    for request, (length, splits) in enumerate(zip(lengths, requested_splits)):
        if not (0 <= length <= geometry.max_context) or not (1 <= splits <= geometry.max_splits):
            raise ValueError("invalid length or split count")
        chunk = split_chunk(length, splits)
        count = -(-length // chunk) if chunk else 0
        counts.append(count)
        for split in range(count):
            begin = split * chunk
            end = min(begin + chunk, length)
            records.append(Record(request, split, begin, end, -(-(end - begin) // BLOCK_KV)))
        offsets.append(len(records))
    return records, counts, offsets


def ceil_log2(weight: int) -> int:
    """Bucket of a record: ceil(log2(weight)) == (weight-1).bit_length()."""
    return (weight - 1).bit_length()


def bucket_order(records):
    """Stable heavy-bucket-first permutation (planning/reference.py:33-34)."""
    return sorted(range(len(records)), key=lambda i: -ceil_log2(records[i].weight))


def make_packs(records, order, groups, workers, pack_limit=4):
    """Pack descriptors within each bucket (planning/reference.py:37-54).

    Every bucket keeps one full wave (``workers``) of singleton tasks at its tail; the
    rest is cut into packs of ``width = min(pack_limit, max(1, maxW >> bucket))``.
    """
    packs = []
    max_weight = max((r.weight for r in records), default=1)
    first = 0
    while first < len(order):
        bucket = ceil_log2(records[order[first]].weight)
        end = first
        while end < len(order) and ceil_log2(records[order[end]].weight) == bucket:
            end += 1
        tasks = (end - first) * groups
        width = min(pack_limit, max(1, max_weight // (1 << bucket)))
        packed = max(0, tasks - workers) // width * width
        start = first * groups
        packs += [(start + i, width) for i in range(0, packed, width)]
        packs += [(start + i, 1) for i in range(packed, tasks)]
        first = end
    return packs


def greedy_static(records, groups, workers):
    """Longest-processing-time lists with a (load, worker) heap (planning/reference.py:57-67).

    Tasks are taken in (-weight, task) order; each goes to the least-loaded worker,
    the lowest worker id winning ties.
    """
    tasks = sorted(range(len(records) * groups), key=lambda t: (-records[t // groups].weight, t))
    heap = [(0, w) for w in range(workers)]
    heapq.heapify(heap)
    lists = [[] for _ in range(workers)]
    for task in tasks:
        load, worker = heapq.heappop(heap)
        lists[worker].append(task)
        heapq.heappush(heap, (load + records[task // groups].weight, worker))
    return lists


def validate_plan(records, order, packs, groups):
    """Coverage and slot-uniqueness checks (planning/reference.py:70-76)."""
    assert sorted(order) == list(range(len(records)))
    tasks = [t for first, count in packs for t in range(first, first + count)]
    assert sorted(tasks) == list(range(len(records) * groups))
    slots = {(records[order[t // groups]].request, records[order[t // groups]].split, t % groups)
             for t in tasks}
    assert len(slots) == len(tasks)


def lists_from_links(head, nxt, workers, limit):
    """Walk STATIC linked lists the way the decode claim loop does (attention.py:107-128)."""
    lists = []
    for w in range(workers):
        out, cursor, guard = [], head[w], 0
        while 0 <= cursor < limit:
            out.append(cursor)
            cursor = nxt[cursor]
            guard += 1
            if guard > limit:
                raise AssertionError("cycle in static list")
        lists.append(out)
    return lists


# --------------------------------------------------------------------------------------
# 2. Device-table semantics (kernels/plan.py + planning/builder.py)
# --------------------------------------------------------------------------------------

def _count_scan(lengths_buf, splits_buf, active, geometry):
    """count_scan (kernels/plan.py:7-27): validation, chunk, counts, offsets, total, error."""
    bcap, smax, maxctx = geometry.batch_capacity, geometry.max_splits, geometry.max_context
    counts, chunks, any_invalid = [], [], False
    for r in range(bcap):
        live = r < active
        length = lengths_buf[r] if live else 0
        splits = splits_buf[r] if live else 1
        invalid = live and (length < 0 or length > maxctx or splits < 1 or splits > smax)
        any_invalid |= invalid
        chunk = _i32(_cdiv(_cdiv(max(length, 0), max(splits, 1)), SPLIT_ALIGNMENT) * SPLIT_ALIGNMENT)
        n = _cdiv(length, max(chunk, 1)) if (live and not invalid) else 0
        counts.append(n)
        chunks.append(chunk)
    error = int(active < 0 or active > bcap or any_invalid)
    if error:
        counts = [0] * bcap
    offsets, running = [], 0
    for n in counts:
        offsets.append(running)
        running += n
    offsets.append(running)
    return counts, chunks, offsets, running, error


def _emit_records(lengths_buf, counts, offsets, chunks, geometry):
    """emit_records (kernels/plan.py:30-45): SoA records at offsets[r] + s."""
    e = geometry.record_capacity
    out = {k: [None] * e for k in ("request", "split", "begin", "end", "weight")}
    for r in range(geometry.batch_capacity):
        for s in range(min(counts[r], geometry.max_splits)):
            i = offsets[r] + s
            begin = s * chunks[r]
            end = min(begin + chunks[r], lengths_buf[r])
            out["request"][i], out["split"][i] = r, s
            out["begin"][i], out["end"][i] = begin, end
            out["weight"][i] = _cdiv(end - begin, BLOCK_KV)
    return out


def select_mode(weights, total, groups, rules, force_mode):
    """Mode choice of make_order_and_packs (kernels/plan.py:53-71).

    Returns (mode, max_weight).  Rows are (min_tasks, max_tasks, min_ratio,
    max_ratio, mode); the last matching row wins; a uniform-weight batch is R1;
    ``force_mode >= 0`` overrides everything.
    """
    valid = weights[:total]
    max_weight = max(valid + [1])            # invalid lanes load 1
    min_weight = min(valid) if valid else INT32_MAX
    ratio = max_weight * 100 // max(min_weight, 1)
    mode = 1
    tasks = total * groups
    for lo, hi, rlo, rhi, row_mode in rules:
        if lo <= tasks <= hi and rlo <= ratio <= rhi:
            mode = row_mode
    if max_weight == min_weight:
        mode = 1
    if force_mode >= 0:
        mode = force_mode
    return mode, max_weight


def _bucket(weight, buckets):
    """Saturating integer ceil-log2 of kernels/plan.py:77-79."""
    return sum(1 for b in range(1, buckets) if weight > (1 << (b - 1)))


def _order_and_packs(weights, total, mode, max_weight, geometry):
    """Order and pack descriptors of make_order_and_packs (kernels/plan.py:72-100)."""
    g, w_count, buckets = geometry.groups, geometry.workers, geometry.buckets
    if mode in (0, 1):
        return list(range(total)), [], []
    bucket = [_bucket(w, buckets) for w in weights[:total]]
    order, first, count = [], [], []
    record_base = 0
    for b in range(buckets - 1, -1, -1):
        members = [i for i in range(total) if bucket[i] == b]
        order += members
        tasks = len(members) * g
        width = min(4, max(1, max_weight // (1 << b))) if mode == 4 else 1
        packed_tasks = max(0, tasks - w_count) // width * width
        packed_packs = packed_tasks // width
        for p in range(packed_packs + tasks - packed_tasks):
            if p < packed_packs:
                first.append(record_base * g + p * width)
                count.append(width)
            else:
                first.append(record_base * g + packed_tasks + p - packed_packs)
                count.append(1)
        record_base += len(members)
    return order, first, count


def _greedy_lists(weights, total, geometry):
    """GPU LPT lists of greedy_lists (kernels/plan.py:103-135).

    Records are taken heaviest first (lowest id on ties); each of a record's
    ``groups`` tasks is appended to the least-loaded worker (lowest id on ties).
    Returns (heads[workers], {task: next}) -- only the written ``next`` entries.
    """
    g, workers = geometry.groups, geometry.workers
    heads = [-1] * workers
    links = {}
    tails = [-1] * workers
    # argmin over (load, worker) == the top of a (load, worker) min-heap.
    heap = [(0, w) for w in range(workers)]
    for record in sorted(range(total), key=lambda i: (-weights[i], i)):
        largest = weights[record]
        for group in range(g):
            task = record * g + group
            load, owner = heapq.heappop(heap)
            if tails[owner] < 0:
                heads[owner] = task
            else:
                links[tails[owner]] = task
            links[task] = -1
            tails[owner] = task
            heapq.heappush(heap, (load + largest, owner))
    return heads, links


def device_tables(lengths_buf, splits_buf, active, geometry, force_mode=-1, rules=()):
    """Every plan buffer the reference's build_plan writes (planning/builder.py:6-28).

    ``lengths_buf``/``splits_buf`` are the full capacity-sized device buffers
    (``PlanBuffers.lengths/splits``).  Entries a step leaves untouched on the
    device (stale from an earlier step) are reported as ``None``.  STATIC lists are
    produced whenever the step's mode is STATIC (the reference launches
    ``greedy_lists`` when a STATIC rule or force exists, and that kernel acts
    only when the mode is STATIC).
    """
    counts, chunks, offsets, total, error = _count_scan(lengths_buf, splits_buf, active, geometry)
    out = dict(counts=counts, chunk=chunks, offsets=offsets, record_count=total, error=error,
               request=None, split=None, begin=None, end=None, weight=None, order=None,
               pack_first=None, pack_count=None, num_packs=0, mode=0,
               static_head=None, static_links=None)
    if int(force_mode) == 0:                       # builder.py:11-14 -- R0 stops after count_scan
        return out
    rec = _emit_records(lengths_buf, counts, offsets, chunks, geometry)
    out.update(rec)
    weights = [rec["weight"][i] for i in range(total)]
    mode, max_weight = select_mode(weights, total, geometry.groups, [tuple(r) for r in rules],
                                   int(force_mode))
    order, first, count = _order_and_packs(weights, total, mode, max_weight, geometry)
    out.update(mode=mode, order=order, pack_first=first, pack_count=count, num_packs=len(first))
    if mode == 2:
        out["static_head"], out["static_links"] = _greedy_lists(weights, total, geometry)
    return out


def task_slots(tables, geometry, query_heads, group_size):
    """Map every logical task to its (request, split, kv_head, begin, end) and partial slots.

    Follows ``_attention_task`` (kernels/attention.py:23-47, 81): task -> record via
    the mode's indirection (R0 binary search over offsets, STATIC original ids,
    others through ``order``), slot = (request*Hq + head)*Smax + split.
    """
    g, smax = geometry.groups, geometry.max_splits
    total = tables["record_count"]
    out = []
    for task in range(total * g):
        group, record = task % g, task // g
        if tables["mode"] != 2:
            record = tables["order"][record]
        request = tables["request"][record]
        split = tables["split"][record]
        heads = [group * group_size + h for h in range(group_size)]
        slots = [(request * query_heads + h) * smax + split for h in heads]
        out.append((request, split, group, tables["begin"][record], tables["end"][record], slots))
    return out
