"""Host-side STATIC planner: LPT worker lists built on the CPU and uploaded.

The reference's benchmark keeps this as its strongest static baseline ("STATIC_CPU",
``benchmarks/bench_decode.py:14-30``): a scheduler that already knows the step's lengths
plans the longest-processing-time lists with a heap on the host (O(T log W)) instead of
on the GPU, then uploads them.  The GPU plan build still produces the records (mode R1,
which skips ordering and packing); the uploaded lists replace ``static_head`` /
``static_next`` and the mode word becomes STATIC.

The lists are the reference's LPT exactly (``planning/reference.py:50-60``): tasks in
(weight descending, task id ascending) order, each to the least-loaded worker, lowest
worker id on ties -- the same lists the GPU plan kernel builds in mode STATIC.
"""
from __future__ import annotations

import heapq

import torch

from ..config import Mode


def record_weights(lengths, splits, config):
    """Per-record weights in record order (request-major, split-minor), as the plan emits them."""
    weights = []
    for length, split in zip(lengths, splits):
        if not 0 <= length <= config.max_context or not 1 <= split <= config.max_splits:
            raise ValueError("invalid length or split count")
        chunk = ((length + split - 1) // split + 31) // 32 * 32
        count = (length + chunk - 1) // chunk if chunk else 0
        for s in range(count):
            begin, end = s * chunk, min((s + 1) * chunk, length)
            weights.append((end - begin + config.block_kv - 1) // config.block_kv)
    return weights


def lpt_lists(weights, groups, workers):
    """(static_head [workers], static_next {task: next}) of the heap LPT over record weights."""
    tasks = sorted(range(len(weights) * groups), key=lambda t: (-weights[t // groups], t))
    heap = [(0, w) for w in range(workers)]
    head = [-1] * workers
    tail = [-1] * workers
    links = {}
    for task in tasks:
        load, worker = heapq.heappop(heap)
        if tail[worker] < 0:
            head[worker] = task
        else:
            links[tail[worker]] = task
        links[task] = -1
        tail[worker] = task
        heapq.heappush(heap, (load + weights[task // groups], worker))
    return head, links


def prepare_host_static(engine, lengths, splits):
    """Plan one step with host LPT lists (the engine's plan inputs must hold this step).

    Issues the GPU plan build in mode R1 (records only), then uploads the lists and sets
    the mode word to STATIC.  Host work: O(T log W) for T = records x groups tasks.
    """
    c, p = engine.config, engine.plan
    weights = record_weights(lengths, splits, c)
    head, links = lpt_lists(weights, c.kv_heads, c.workers)
    saved = engine.force_mode
    engine.force_mode = int(Mode.R1)
    try:
        engine.prepare()
    finally:
        engine.force_mode = saved
    nxt = torch.full((c.task_capacity,), -1, dtype=torch.int32)
    if links:
        keys = torch.tensor(list(links.keys()), dtype=torch.int64)
        nxt[keys] = torch.tensor(list(links.values()), dtype=torch.int32)
    p.static_head.copy_(torch.tensor(head, dtype=torch.int32), non_blocking=False)
    p.static_next.copy_(nxt, non_blocking=False)
    p.mode.fill_(int(Mode.STATIC))
