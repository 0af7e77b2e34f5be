"""Seeded decode workloads: the reference's fixtures and the BASELINE configs.

* ``split_hints`` / ``make_inputs`` / ``update_plan`` follow the reference's
  ``benchmarks/workloads.py:14-50`` (same split rule; same generator call sequence,
  so the same seed on the same device gives the same tensors).
* ``baseline(name)`` builds the five benchmark configurations (C1..C5): shapes,
  dtype, KV layout (paged or CSR), length distribution and page/slot permutation.
  Values are N(0,1), sm_scale = 1/sqrt(head_dim), splits = split_hints(lengths, 16).
  There is no dataset: every input is synthetic and seeded.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

import torch

from .config import DecodeConfig

WORKLOADS = {
    "A": [512] * 24 + [8192] * 8,
    "B": [256] * 24 + [1536] * 4 + [16384] * 4,
    "B64": ([256] * 24 + [1536] * 4 + [16384] * 4) * 2,
    "uniform": [1024] * 32,
    "holdout": [33, 255, 513, 1025, 3073, 8191, 16383],
}


def split_hints(lengths, maximum=16):
    """Fixture split rule: chunk = ceil(max(L)/maximum); splits = ceil(L/chunk) in [1, maximum]."""
    chunk = max(1, math.ceil(max(lengths, default=0) / maximum))
    return [max(1, min(maximum, math.ceil(n / chunk))) for n in lengths]


def make_inputs(config, lengths, seed=17, device="cuda", dtype=torch.bfloat16):
    """Paged fixture: permuted physical pages, page table padded with -1, randn Q/K/V."""
    generator = torch.Generator(device=device).manual_seed(seed)
    pages_per_request = [math.ceil(n / config.page_size) for n in lengths]
    physical_pages = max(1, sum(pages_per_request))
    permutation = torch.randperm(physical_pages, generator=generator, device=device)
    table = torch.full((config.batch_capacity, config.max_pages), -1, dtype=torch.int32, device=device)
    cursor = 0
    for row, count in enumerate(pages_per_request):
        table[row, :count] = permutation[cursor:cursor + count].int()
        cursor += count
    shape = (physical_pages, config.page_size, config.kv_heads, config.head_dim)
    k = torch.randn(shape, generator=generator, device=device, dtype=dtype)
    v = torch.randn(shape, generator=generator, device=device, dtype=dtype)
    q = torch.randn((config.batch_capacity, config.query_heads, config.head_dim),
                    generator=generator, device=device, dtype=dtype)
    return q, k, v, table


def make_csr_inputs(config, lengths, seed=17, device="cuda", dtype=torch.bfloat16, pool=None):
    """CSR fixture (page_size 1): kv_indices are consecutive slices of a slot permutation.

    Returns q [Bcap,Hq,D], k/v [pool,Hkv,D], kv_indices [sum L] int32, kv_indptr [Bcap+1]
    int32 (rows past len(lengths) repeat the total).
    """
    generator = torch.Generator(device=device).manual_seed(seed)
    total = sum(lengths)
    pool = max(1, total if pool is None else pool)
    if pool < total:
        raise ValueError("pool smaller than the total context")
    indices = torch.randperm(pool, generator=generator, device=device)[:total].int()
    pointers = [0]
    for n in lengths:
        pointers.append(pointers[-1] + n)
    pointers += [pointers[-1]] * (config.batch_capacity + 1 - len(pointers))
    indptr = torch.tensor(pointers, dtype=torch.int32, device=device)
    shape = (pool, config.kv_heads, config.head_dim)
    k = torch.randn(shape, generator=generator, device=device, dtype=dtype)
    v = torch.randn(shape, generator=generator, device=device, dtype=dtype)
    q = torch.randn((config.batch_capacity, config.query_heads, config.head_dim),
                    generator=generator, device=device, dtype=dtype)
    return q, k, v, indices, indptr


def update_plan(engine, lengths, splits=None):
    """Write one step's lengths / splits / active into the plan inputs (H2D copies)."""
    p = engine.plan
    splits = split_hints(lengths, engine.config.max_splits) if splits is None else splits
    p.lengths.zero_()
    p.splits.fill_(1)
    p.active.fill_(len(lengths))
    if lengths:
        p.lengths[:len(lengths)].copy_(torch.tensor(lengths, dtype=torch.int32))
        p.splits[:len(lengths)].copy_(torch.tensor(splits, dtype=torch.int32))


@dataclass
class Baseline:
    """One benchmark configuration (C1..C5): shapes, dtype, KV layout and seeded lengths.

    Inputs follow the reference fixture recipe (``benchmarks/workloads.py:14-40``):
    N(0,1) values from a seeded generator, splits = ``split_hints(lengths, 16)``."""
    name: str
    config: DecodeConfig
    dtype: torch.dtype
    csr: bool
    lengths: list
    layers: int = 1
    pool_tokens: int = 0          # CSR pool slots (>= sum of lengths)
    pool_pages: int = 0           # paged pool pages
    modes: tuple = (-1,)
    replay_batches: tuple = ()
    notes: dict = field(default_factory=dict)

    @property
    def splits(self):
        return split_hints(self.lengths, 16)

    def kv_bytes(self, kv_heads=None):
        """Algorithmic K+V bytes of one layer (every token's K and V row read once)."""
        hkv = self.config.kv_heads if kv_heads is None else kv_heads
        elem = torch.finfo(self.dtype).bits // 8
        return sum(self.lengths) * hkv * self.config.head_dim * 2 * elem


def _randint(rng, lo, hi, n):
    return [rng.randint(lo, hi) for _ in range(n)]


def baseline(name, seed=17, workers=148):
    """Build one of C1..C5 (lengths drawn from a seeded Python RNG)."""
    rng = random.Random(seed)
    if name == "C1":    # Llama-3-8B, B=8, CSR over a 16384-slot pool
        lengths = _randint(rng, 64, 1024, 8)
        cfg = DecodeConfig(batch_capacity=8, max_splits=16, max_context=1024, query_heads=32,
                           kv_heads=8, head_dim=128, page_size=1, workers=workers)
        return Baseline(name, cfg, torch.bfloat16, True, lengths, pool_tokens=16384)
    if name == "C2":    # skewed B=64, page_size 16, 10% long requests
        lengths = _randint(rng, 128, 1024, 64)
        for i in rng.sample(range(64), round(0.1 * 64)):
            lengths[i] = rng.randint(16384, 32768)
        cfg = DecodeConfig(batch_capacity=64, max_splits=16, max_context=32768, query_heads=32,
                           kv_heads=8, head_dim=128, page_size=16, workers=workers)
        pages = sum(math.ceil(n / 16) for n in lengths)
        return Baseline(name, cfg, torch.bfloat16, False, lengths, pool_pages=pages,
                        modes=(1, 2, 3, 4))
    if name == "C3":    # Llama-3-70B, B=256, fp16, CSR; heads sharded over 1/2/4/8 GPUs
        lengths = _randint(rng, 1024, 8192, 256)
        cfg = DecodeConfig(batch_capacity=256, max_splits=16, max_context=8192, query_heads=64,
                           kv_heads=8, head_dim=128, page_size=1, workers=workers)
        return Baseline(name, cfg, torch.float16, True, lengths, pool_tokens=sum(lengths))
    if name == "C4":    # long context, page_size 64, pool = total pages + 10%
        lengths = _randint(rng, 32768, 131072, 16)
        cfg = DecodeConfig(batch_capacity=16, max_splits=16, max_context=131072, query_heads=32,
                           kv_heads=8, head_dim=128, page_size=64, workers=workers)
        pages = math.ceil(1.1 * sum(math.ceil(n / 64) for n in lengths))
        return Baseline(name, cfg, torch.bfloat16, False, lengths, pool_pages=pages)
    if name == "C5":    # Qwen2-7B, 28 layers, G=7, CSR, CUDA graph at capacity 128
        lengths = _randint(rng, 256, 4096, 128)
        cfg = DecodeConfig(batch_capacity=128, max_splits=16, max_context=8192, query_heads=28,
                           kv_heads=4, head_dim=128, page_size=1, workers=workers)
        return Baseline(name, cfg, torch.bfloat16, True, lengths, layers=28,
                        pool_tokens=sum(lengths) + 5 * 128, replay_batches=(128, 96, 64, 33, 1))
    raise KeyError(name)


def subset(b: Baseline, requests: int) -> Baseline:
    """The first ``requests`` requests of a Baseline (pool sized for them), same config."""
    import dataclasses
    lengths = b.lengths[:requests]
    c = b.config
    if b.csr:
        pool_tokens = b.pool_tokens if b.name == "C1" else sum(lengths) + (b.pool_tokens - sum(b.lengths))
        return dataclasses.replace(b, lengths=lengths, pool_tokens=max(pool_tokens, sum(lengths), 1))
    pages = sum(math.ceil(n / c.page_size) for n in lengths)
    if b.name == "C4":
        pages = math.ceil(1.1 * pages)
    return dataclasses.replace(b, lengths=lengths, pool_pages=max(pages, 1))


def paged_tables(config, lengths, pool_pages, generator, device):
    """Page table [Bcap, max_pages] from consecutive slices of a page permutation."""
    perm = torch.randperm(pool_pages, generator=generator, device=device)
    table = torch.full((config.batch_capacity, config.max_pages), -1, dtype=torch.int32, device=device)
    cursor = 0
    for row, n in enumerate(lengths):
        count = math.ceil(n / config.page_size)
        table[row, :count] = perm[cursor:cursor + count].int()
        cursor += count
    return table


def generate(b: Baseline, device="cuda", seed=17, kv_heads=None, head_offset=0):
    """Materialise one layer of a Baseline on ``device``.

    ``kv_heads``/``head_offset`` select a head shard (tensor-parallel sharding by KV
    head): the returned K/V pool holds only heads [offset, offset+kv_heads) and Q only
    the matching query heads.  Every shard draws the FULL tensors' values from the
    same seed, so shards of a sharded run equal slices of the unsharded run.
    Returns dict(q, k, v, pages, indptr).
    """
    c = b.config
    hkv = c.kv_heads if kv_heads is None else kv_heads
    group = c.group_size
    gen = torch.Generator(device=device).manual_seed(seed)
    if b.csr:
        total = sum(b.lengths)
        pages = torch.randperm(b.pool_tokens, generator=gen, device=device)[:total].int()
        pointers = [0]
        for n in b.lengths:
            pointers.append(pointers[-1] + n)
        pointers += [pointers[-1]] * (c.batch_capacity + 1 - len(pointers))
        indptr = torch.tensor(pointers, dtype=torch.int32, device=device)
        rows = b.pool_tokens
        shape_full = (rows, c.kv_heads, c.head_dim)
    else:
        pages = paged_tables(c, b.lengths, b.pool_pages, gen, device)
        indptr = None
        shape_full = (b.pool_pages, c.page_size, c.kv_heads, c.head_dim)
    k = _sharded_randn(shape_full, gen, device, b.dtype, hkv, head_offset)
    v = _sharded_randn(shape_full, gen, device, b.dtype, hkv, head_offset)
    q_full_shape = (c.batch_capacity, c.query_heads, c.head_dim)
    q = torch.randn(q_full_shape, generator=gen, device=device, dtype=b.dtype)
    q = q[:, head_offset * group:(head_offset + hkv) * group].contiguous()
    return dict(q=q, k=k, v=v, pages=pages, indptr=indptr)


def graph_layer(b: Baseline, layer: int, device="cuda"):
    """One layer of a graph Baseline (C5): its K/V pool and the full slot permutation.

    Layer ``layer`` is seeded 17 + layer.  Request r's first L0_r tokens live in slots
    perm[offset_r : offset_r + L0_r]; the token a request appends at replay step s
    (s = 1, 2, ...) lives in slot perm[sum(L0) + (s - 1) * capacity + r].
    Returns dict(k, v, perm, q) with q at the graph capacity.
    """
    c = b.config
    gen = torch.Generator(device=device).manual_seed(17 + layer)
    perm = torch.randperm(b.pool_tokens, generator=gen, device=device).int()
    shape = (b.pool_tokens, c.kv_heads, c.head_dim)
    k = _sharded_randn(shape, gen, device, b.dtype, c.kv_heads, 0)
    v = _sharded_randn(shape, gen, device, b.dtype, c.kv_heads, 0)
    q = torch.randn((c.batch_capacity, c.query_heads, c.head_dim), generator=gen, device=device, dtype=b.dtype)
    return dict(k=k, v=v, perm=perm, q=q)


def graph_step(b: Baseline, step: int, batch: int):
    """Lengths and slot positions (into a layer's permutation) of replay step ``step``.

    The batch is the first ``batch`` requests; each has appended ``step`` tokens.  The
    positions are the same for every layer (each layer applies its own permutation).
    Returns (lengths, positions) with positions a CPU int64 tensor of sum(lengths) entries.
    """
    cap = b.config.batch_capacity
    total0 = sum(b.lengths)
    if (step) * cap > b.pool_tokens - total0:
        raise ValueError("the pool has no room for that many appended tokens")
    lengths, parts, offset = [], [], 0
    for r in range(batch):
        n0 = b.lengths[r]
        lengths.append(n0 + step)
        parts.append(torch.arange(offset, offset + n0, dtype=torch.int64))
        if step:
            parts.append(total0 + r + cap * torch.arange(step, dtype=torch.int64))
        offset += n0
    positions = torch.cat(parts) if parts else torch.zeros(0, dtype=torch.int64)
    return lengths, positions


def _sharded_randn(shape, gen, device, dtype, hkv, head_offset, chunk_rows=1 << 16):
    """randn of the full [..., Hkv, D] pool, keeping heads [offset, offset+hkv) only.

    Draws chunk by chunk (the same chunking for every shard, so a shard equals the
    matching slice of the unsharded pool) and never materialises the full pool.
    """
    out = torch.empty((*shape[:-2], hkv, shape[-1]), device=device, dtype=dtype)
    rows = shape[0]
    for start in range(0, rows, chunk_rows):
        stop = min(rows, start + chunk_rows)
        block = torch.randn((stop - start, *shape[1:]), generator=gen, device=device, dtype=dtype)
        out[start:stop] = block[..., head_offset:head_offset + hkv, :]
    return out
