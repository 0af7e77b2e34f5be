#!/usr/bin/env python3
"""Generate golden vectors for the decode hot path FROM THE REFERENCE ITSELF.

Run in a container where the reference checkout is available (read-only) and
torch + triton are importable:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

It writes, next to this script:

* ``plan_spec.json.gz``    -- the reference CPU specification
  (``src/sglang_decode/planning/reference.py``) on the documented workloads and
  extra cases: records, counts, offsets, bucket order, D1/D4 packs and heap-LPT
  static lists.
* ``plan_device.json.gz``  -- every buffer written by the reference's Triton plan
  kernels (``src/sglang_decode/kernels/plan.py`` via ``planning/builder.py``),
  executed on the CPU by the Triton interpreter (``TRITON_INTERPRET=1``), for
  forced modes, AUTO rules, uniform batches, zero lengths and invalid metadata.
* ``attention.npz``     -- small seeded decode cases: inputs (raw fp16/bf16 bits),
  the reference FP32 oracle (``src/sglang_decode/reference/attention.py``), and
  for fp16 the reference Triton decode + merge outputs run by the interpreter
  (``kernels/attention.py``, ``kernels/merge.py``), plus its partial/LSE slots.

The tests never import the reference; they only read these files.
"""
from __future__ import annotations

import argparse
import gzip
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"      # must precede the triton import

HERE = Path(__file__).resolve().parent


def _load_reference(root: Path):
    sys.path.insert(0, str(root / "src"))
    sys.path.insert(0, str(root))
    import torch  # noqa: F401
    from sglang_decode.config import DecodeConfig, Mode
    from sglang_decode.planning import reference as spec
    from sglang_decode.planning.policy import PolicyRule
    from sglang_decode.reference.attention import paged_attention
    from sglang_decode.runtime.engine import DecodeEngine
    from benchmarks.workloads import split_hints, WORKLOADS
    return dict(DecodeConfig=DecodeConfig, Mode=Mode, spec=spec, PolicyRule=PolicyRule,
                paged_attention=paged_attention, DecodeEngine=DecodeEngine,
                split_hints=split_hints, WORKLOADS=WORKLOADS)


def spec_cases(ref):
    """CPU-spec goldens on the reference's documented and fixture workloads."""
    DecodeConfig, spec, split_hints, W = (ref["DecodeConfig"], ref["spec"], ref["split_hints"],
                                          ref["WORKLOADS"])
    cases = []
    documented = [
        ("A", W["A"], [1] * 24 + [16] * 8),
        ("B", W["B"], [1] * 24 + [2] * 4 + [16] * 4),
        ("B64", W["B64"], ([1] * 24 + [2] * 4 + [16] * 4) * 2),
        ("tail", [0, 1, 33, 513], [16, 16, 16, 2]),
        ("hint_A", W["A"], split_hints(W["A"])),
        ("hint_B", W["B"], split_hints(W["B"])),
        ("hint_B64", W["B64"], split_hints(W["B64"])),
        ("hint_uniform", W["uniform"], split_hints(W["uniform"])),
        ("hint_holdout", W["holdout"], split_hints(W["holdout"])),
        ("mixed6", [0, 1, 17, 33, 257, 513], split_hints([0, 1, 17, 33, 257, 513])),
    ]
    for name, lengths, splits in documented:
        for workers, kv_heads in ((108, 8), (148, 8), (148, 4), (4, 8), (148, 1), (7, 2)):
            c = DecodeConfig(workers=workers, kv_heads=kv_heads, query_heads=kv_heads * 4)
            records, counts, offsets = spec.split_records(lengths, splits, c)
            order = spec.bucket_order(records)
            packs4 = spec.make_packs(records, order, c.kv_heads, c.workers, pack_limit=4)
            packs1 = spec.make_packs(records, order, c.kv_heads, c.workers, pack_limit=1)
            lists = spec.greedy_static(records, c.kv_heads, c.workers)
            cases.append(dict(
                name=name, lengths=lengths, splits=splits, workers=workers, groups=kv_heads,
                batch_capacity=c.batch_capacity, max_splits=c.max_splits, max_context=c.max_context,
                records=[[r.request, r.split, r.begin, r.end, r.weight] for r in records],
                counts=counts, offsets=offsets, order=order,
                packs_d4=[list(p) for p in packs4], packs_d1=[list(p) for p in packs1],
                static_lists=lists))
    rejected = []
    for lengths, splits in ([32769], [1]), ([1], [0]), ([1] * 65, [1] * 65), ([-1], [1]), ([5], [17]):
        try:
            spec.split_records(lengths, splits, DecodeConfig())
            rejected.append(dict(lengths=lengths, splits=splits, raised=False))
        except ValueError:
            rejected.append(dict(lengths=lengths, splits=splits, raised=True))
    return dict(cases=cases, rejected=rejected)


def _plan_run(ref, config, lengths_buf, splits_buf, active, force, rules):
    import torch
    engine = ref["DecodeEngine"](config, device="cpu", dtype=torch.float16, rules=rules,
                                 force_mode=force)
    p = engine.plan
    p.lengths.copy_(torch.tensor(lengths_buf, dtype=torch.int32))
    p.splits.copy_(torch.tensor(splits_buf, dtype=torch.int32))
    p.active.fill_(active)
    # Poison every output so stale entries are recognisable (-7 never occurs naturally).
    for name in ("counts", "offsets", "chunk", "request", "split", "begin", "end", "weight",
                 "order", "pack_first", "pack_count", "record_count", "num_packs", "mode",
                 "error", "static_head", "static_next"):
        getattr(p, name).fill_(-7)
    engine.prepare()
    out = {}
    for name in ("record_count", "num_packs", "mode", "error"):
        out[name] = int(getattr(p, name).item())
    for name in ("counts", "offsets", "chunk", "static_head"):
        out[name] = getattr(p, name).tolist()
    # Record arrays: the written prefix, plus whether everything past it kept the poison.
    total = max(out["record_count"], 0) if out["record_count"] != -7 else 0
    for name in ("request", "split", "begin", "end", "weight", "order"):
        full = getattr(p, name).tolist()
        out[name] = full[:total]
        out[name + "_tail_untouched"] = all(x == -7 for x in full[total:])
    packs = max(out["num_packs"], 0) if out["num_packs"] != -7 else 0
    for name in ("pack_first", "pack_count"):
        full = getattr(p, name).tolist()
        out[name] = full[:packs]
        out[name + "_tail_untouched"] = all(x == -7 for x in full[packs:])
    # Linked-list links: only the written entries, as [task, next] pairs.
    out["static_next"] = [[t, x] for t, x in enumerate(p.static_next.tolist()) if x != -7]
    return out


def device_cases(ref):
    """Reference Triton plan kernels under the interpreter, every buffer recorded."""
    DecodeConfig, Mode, PolicyRule, split_hints, W = (
        ref["DecodeConfig"], ref["Mode"], ref["PolicyRule"], ref["split_hints"], ref["WORKLOADS"])

    def pad(values, n, fill):
        return list(values) + [fill] * (n - len(values))

    cases = []

    def add(name, cfg, lengths, splits, active=None, force=-1, rules=(), lengths_buf=None,
            splits_buf=None):
        b = cfg["batch_capacity"]
        lengths_buf = lengths_buf or pad(lengths, b, 0)
        splits_buf = splits_buf or pad(splits, b, 1)
        active = len(lengths) if active is None else active
        config = DecodeConfig(**cfg)
        rule_objs = [PolicyRule(*r) for r in rules]
        out = _plan_run(ref, config, lengths_buf, splits_buf, active, force, rule_objs)
        cases.append(dict(name=name, config=cfg, lengths_buf=lengths_buf, splits_buf=splits_buf,
                          active=active, force=force, rules=[list(r) for r in rules],
                          buckets=config.buckets, outputs=out))

    base = dict(batch_capacity=64, max_splits=16, max_context=32768, query_heads=32, kv_heads=8,
                head_dim=128, page_size=16, workers=148)
    mixed = [0, 1, 17, 33, 257, 513]
    for force in (0, 1, 2, 3, 4):
        add(f"B_force{force}", base, W["B"], split_hints(W["B"]), force=force)
        add(f"mixed_force{force}", base, mixed, split_hints(mixed), force=force)
        add(f"B64_force{force}", base, W["B64"], split_hints(W["B64"]), force=force)
    add("A_auto", base, W["A"], split_hints(W["A"]))
    add("uniform_auto", base, W["uniform"], split_hints(W["uniform"]))
    add("uniform_force4", base, W["uniform"], split_hints(W["uniform"]), force=4)
    d4_rule = [(1, 8 * 64 * 16, 101, 10000, 4)]
    add("rule_d4", base, W["B"], split_hints(W["B"]), rules=d4_rule)
    add("rule_d4_uniform", base, W["uniform"], split_hints(W["uniform"]), rules=d4_rule)
    add("rule_static", base, W["B"], split_hints(W["B"]), rules=[(0, 100000, 100, 100000, 2)])
    add("rule_two_rows", base, W["B"], split_hints(W["B"]),
        rules=[(0, 100000, 100, 100000, 3), (0, 100000, 150, 100000, 4)])
    add("rule_no_match", base, W["B"], split_hints(W["B"]), rules=[(0, 10, 100, 100000, 4)])
    add("rule_ratio_miss", base, W["B"], split_hints(W["B"]), rules=[(0, 100000, 100, 120, 3)])
    add("empty_batch", base, [], [], active=0)
    add("all_zero_len", base, [0, 0, 0], [1, 1, 1], force=4)
    # Invalid metadata: the device zeroes all tasks and raises the error word.
    add("bad_negative_len", base, [5, -1, 7], [1, 1, 1], force=4)
    add("bad_long_len", base, [5, 40000, 7], [1, 1, 1], force=1)
    add("bad_split0", base, [5, 9, 7], [1, 0, 1], force=3)
    add("bad_split_big", base, [5, 9, 7], [1, 17, 1], force=2)
    add("bad_active_big", base, [5, 9], [1, 1], active=65, force=4)
    add("bad_active_neg", base, [5, 9], [1, 1], active=-1, force=4)
    # Stale rows beyond `active` must be ignored even when they hold invalid values.
    add("stale_rows", base, [300, 40], [2, 1], active=2, force=4,
        lengths_buf=pad([300, 40], 64, 99999), splits_buf=pad([2, 1], 64, 0))
    # Shapes of the BASELINE configs (planning only depends on these fields).
    c1 = dict(batch_capacity=8, max_splits=16, max_context=1024, query_heads=32, kv_heads=8,
              head_dim=128, page_size=1, workers=148)
    l1 = [64, 1024, 700, 333, 129, 900, 1000, 65]
    for force in (-1, 1, 2, 3, 4, 0):
        add(f"c1_force{force}", c1, l1, split_hints(l1), force=force)
    import random
    rng = random.Random(5)
    c2 = dict(batch_capacity=64, max_splits=16, max_context=32768, query_heads=32, kv_heads=8,
              head_dim=128, page_size=16, workers=148)
    l2 = [rng.randint(128, 1024) for _ in range(64)]
    for i in rng.sample(range(64), 6):
        l2[i] = rng.randint(16384, 32768)
    for force in (1, 2, 3, 4):
        add(f"c2_force{force}", c2, l2, split_hints(l2), force=force)
    c5 = dict(batch_capacity=128, max_splits=16, max_context=8192, query_heads=4, kv_heads=4,
              head_dim=128, page_size=1, workers=148)
    l5 = [rng.randint(256, 4096) for _ in range(33)]
    for force in (1, 3, 4):
        add(f"c5_force{force}", c5, l5, split_hints(l5), force=force)
    small_w = dict(base, workers=5, kv_heads=2, query_heads=8)
    l3 = [rng.randint(1, 3000) for _ in range(40)]
    for force in (2, 3, 4):
        add(f"smallw_force{force}", small_w, l3, split_hints(l3), force=force)
    g1 = dict(base, kv_heads=1, query_heads=16, workers=16)
    for force in (2, 4):
        add(f"g1_force{force}", g1, l3, split_hints(l3), force=force)
    return dict(cases=cases)


def attention_cases(ref, out_path):
    """Small seeded decode cases with the reference oracle (and interpreter) outputs."""
    import numpy as np
    import torch
    DecodeConfig, Mode, split_hints = ref["DecodeConfig"], ref["Mode"], ref["split_hints"]
    paged_attention, DecodeEngine = ref["paged_attention"], ref["DecodeEngine"]
    arrays = {}
    meta = []

    def bits(t):
        return t.contiguous().view(torch.int16).numpy()

    def make(cfg, lengths, seed, dtype):
        g = torch.Generator().manual_seed(seed)
        ps = cfg["page_size"]
        per = [-(-n // ps) for n in lengths]
        npages = max(1, sum(per))
        perm = torch.randperm(npages, generator=g)
        maxp = -(-cfg["max_context"] // ps)
        table = torch.full((cfg["batch_capacity"], maxp), -1, dtype=torch.int32)
        cur = 0
        for row, cnt in enumerate(per):
            table[row, :cnt] = perm[cur:cur + cnt].int()
            cur += cnt
        shape = (npages, ps, cfg["kv_heads"], cfg["head_dim"])
        k = torch.randn(shape, generator=g).to(dtype)
        v = torch.randn(shape, generator=g).to(dtype)
        q = torch.randn((cfg["batch_capacity"], cfg["query_heads"], cfg["head_dim"]),
                        generator=g).to(dtype)
        return q, k, v, table

    specs = [
        ("paged_g4_f16", dict(batch_capacity=6, max_splits=4, max_context=1024, query_heads=8,
                              kv_heads=2, head_dim=64, page_size=16, workers=7),
         [0, 1, 17, 33, 257, 513], torch.float16, True),
        ("paged_g8_bf16", dict(batch_capacity=4, max_splits=8, max_context=2048, query_heads=16,
                               kv_heads=2, head_dim=128, page_size=16, workers=9),
         [700, 129, 31, 333], torch.bfloat16, False),
        ("paged_g1_f16", dict(batch_capacity=3, max_splits=4, max_context=512, query_heads=4,
                              kv_heads=4, head_dim=64, page_size=8, workers=5),
         [300, 0, 77], torch.float16, True),
        ("paged_g16_f16", dict(batch_capacity=2, max_splits=4, max_context=512, query_heads=32,
                               kv_heads=2, head_dim=64, page_size=32, workers=6),
         [511, 96], torch.float16, True),
    ]
    for name, cfg, lengths, dtype, run_triton in specs:
        q, k, v, table = make(cfg, lengths, 17, dtype)
        c = DecodeConfig(**cfg)
        expected = paged_attention(q, k, v, table, lengths, c.page_size)
        splits = split_hints(lengths, c.max_splits)
        arrays[f"{name}/q"], arrays[f"{name}/k"], arrays[f"{name}/v"] = bits(q), bits(k), bits(v)
        arrays[f"{name}/pages"] = table.numpy()
        arrays[f"{name}/oracle"] = expected.numpy()
        entry = dict(name=name, config=cfg, lengths=lengths, splits=splits,
                     dtype="float16" if dtype == torch.float16 else "bfloat16",
                     triton_modes=[])
        if run_triton:
            for mode in (Mode.R0, Mode.R1, Mode.STATIC, Mode.D1, Mode.D4):
                engine = DecodeEngine(c, device="cpu", dtype=dtype, force_mode=int(mode))
                p = engine.plan
                p.lengths.zero_()
                p.splits.fill_(1)
                p.active.fill_(len(lengths))
                p.lengths[:len(lengths)].copy_(torch.tensor(lengths, dtype=torch.int32))
                p.splits[:len(lengths)].copy_(torch.tensor(splits, dtype=torch.int32))
                engine.layers[0].partial.fill_(float("nan"))
                engine.layers[0].lse.fill_(float("nan"))
                engine.prepare()
                out = engine.execute(q, k, v, table)
                arrays[f"{name}/triton_{int(mode)}"] = out.float().numpy()
                if mode == Mode.R1:
                    arrays[f"{name}/triton_partial"] = engine.layers[0].partial.numpy()
                    arrays[f"{name}/triton_lse"] = engine.layers[0].lse.numpy()
                entry["triton_modes"].append(int(mode))
        meta.append(entry)
    # Group size 7 (Qwen2-7B shape): the reference config rejects it, its FP32 oracle does not.
    cfg7 = dict(batch_capacity=3, max_splits=4, max_context=512, query_heads=28, kv_heads=4,
                head_dim=128, page_size=1, workers=5)
    lengths7 = [200, 1, 150]
    q, k, v, table = make(cfg7, lengths7, 23, torch.bfloat16)
    expected = paged_attention(q, k, v, table, lengths7, 1)
    arrays["csr_g7_bf16/q"], arrays["csr_g7_bf16/k"], arrays["csr_g7_bf16/v"] = bits(q), bits(k), bits(v)
    arrays["csr_g7_bf16/pages"] = table.numpy()
    arrays["csr_g7_bf16/oracle"] = expected.numpy()
    meta.append(dict(name="csr_g7_bf16", config=cfg7, lengths=lengths7,
                     splits=split_hints(lengths7, 4), dtype="bfloat16", triton_modes=[]))
    np.savez_compressed(out_path, **arrays)
    return meta


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    ref = _load_reference(args.reference)
    with gzip.open(HERE / "plan_spec.json.gz", "wt") as f:
        json.dump(spec_cases(ref), f)
    with gzip.open(HERE / "plan_device.json.gz", "wt") as f:
        json.dump(device_cases(ref), f)
    meta = attention_cases(ref, HERE / "attention.npz")
    (HERE / "attention.json").write_text(json.dumps(meta, indent=1))
    print("wrote golden vectors to", HERE)


if __name__ == "__main__":
    main()
