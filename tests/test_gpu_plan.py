"""GPU task tables vs the reference (bit-exact), through the C ABI.

Every case of tests/golden/plan_device.json.gz was produced by the reference's own
Triton plan kernels; the sm_100a plan kernel must reproduce every buffer exactly,
including stale (untouched) entries, error handling and AUTO rules.  Random cases
and the BASELINE shapes are checked against the CPU oracle.
"""
import random

import pytest
import torch

from oracle import planning as P
from sglang_decode.config import DecodeConfig
from sglang_decode.planning.policy import PolicyRule
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import baseline, split_hints
from tests.golden import plan_device
from tests.helpers import capture_tables, geometry_of, oracle_tables_in_golden_format, poison_plan

pytestmark = pytest.mark.gpu


def run_plan(config, lengths_buf, splits_buf, active, force, rules):
    engine = DecodeEngine(config, device="cuda", dtype=torch.float16, force_mode=force,
                          rules=[PolicyRule(*r) for r in rules])
    p = engine.plan
    p.lengths.copy_(torch.tensor(lengths_buf, dtype=torch.int32))
    p.splits.copy_(torch.tensor(splits_buf, dtype=torch.int32))
    p.active.fill_(active)
    poison_plan(p)
    engine.counters.fill_(12345)
    engine.prepare()
    torch.cuda.synchronize()
    assert engine.counters.eq(0).all(), "plan build must reset the layer claim counters"
    return capture_tables(p)


CASES = plan_device()["cases"]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_plan_matches_reference_triton_tables(case, cuda_device):
    cfg = DecodeConfig(**case["config"])
    got = run_plan(cfg, case["lengths_buf"], case["splits_buf"], case["active"], case["force"],
                   case["rules"])
    assert got == case["outputs"]


def _random_case(rng):
    bcap = rng.choice([1, 3, 8, 17, 64, 256])
    smax = rng.choice([1, 2, 4, 16])
    while bcap * smax > 4096:
        smax //= 2
    maxctx = rng.choice([64, 1000, 8192, 131072])
    hkv = rng.choice([1, 2, 4, 8])
    workers = rng.choice([1, 5, 108, 148, 296, 1500])
    n = rng.randint(0, bcap)
    lengths = [rng.choice([0, 1, rng.randint(1, maxctx), maxctx]) for _ in range(n)]
    splits = [rng.randint(1, smax) for _ in range(n)]
    force = rng.choice([-1, 0, 1, 2, 3, 4])
    rules = []
    if force == -1 and rng.random() < 0.7:
        for _ in range(rng.randint(1, 3)):
            lo = rng.randint(0, 200)
            rules.append((lo, lo + rng.randint(0, 10**5), 100 + rng.randint(0, 300),
                          100 + rng.randint(300, 10**5), rng.choice([1, 2, 3, 4])))
    cfg = DecodeConfig(batch_capacity=bcap, max_splits=smax, max_context=maxctx,
                       query_heads=hkv * 2, kv_heads=hkv, head_dim=128, page_size=16, workers=workers)
    lb = lengths + [0] * (bcap - n)
    sb = splits + [1] * (bcap - n)
    if rng.random() < 0.15:       # invalid metadata: the error path (tasks zeroed, error word)
        i = rng.randrange(bcap)
        if rng.random() < 0.5:
            lb[i] = rng.choice([-1, maxctx + 1])
        else:
            sb[i] = rng.choice([0, smax + 1])
        n = max(n, i + 1) if rng.random() < 0.8 else n
    return cfg, lb, sb, n, force, rules


@pytest.mark.parametrize("seed", range(40))
def test_plan_random_cases_match_oracle(seed, cuda_device):
    cfg, lb, sb, active, force, rules = _random_case(random.Random(1000 + seed))
    g = geometry_of(cfg)
    want = oracle_tables_in_golden_format(P.device_tables(lb, sb, active, g, force, rules), g)
    got = run_plan(cfg, lb, sb, active, force, rules)
    assert got == want


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4", "C5"])
@pytest.mark.parametrize("force", [-1, 0, 1, 2, 3, 4])
def test_plan_baseline_shapes_match_oracle(name, force, cuda_device):
    b = baseline(name)
    cfg = b.config
    g = geometry_of(cfg)
    lb = b.lengths + [0] * (cfg.batch_capacity - len(b.lengths))
    sb = b.splits + [1] * (cfg.batch_capacity - len(b.lengths))
    want = oracle_tables_in_golden_format(P.device_tables(lb, sb, len(b.lengths), g, force), g)
    got = run_plan(cfg, lb, sb, len(b.lengths), force, [])
    assert got == want


@pytest.mark.parametrize("workers", [7, 148, 1023, 1024, 1025])
@pytest.mark.parametrize("maxctx", [8192, 1 << 21])
def test_plan_static_lists_all_worker_and_weight_ranges(workers, maxctx, cuda_device):
    """STATIC lists on the kernel's three LPT paths: weights up to 4096 (run table,
    32-bit rank keys), heavier weights (contexts above 512K tokens: per-run max
    reduction, 64-bit keys) and more than 1024 workers (serial LPT)."""
    rng = random.Random(workers * 7 + maxctx)
    bcap, smax, hkv = 64, 4, 4
    for _ in range(3):
        n = rng.randint(1, bcap)
        lengths = [rng.choice([1, 33, 128, 129, rng.randint(1, maxctx), maxctx]) for _ in range(n)]
        splits = [rng.randint(1, smax) for _ in range(n)]
        cfg = DecodeConfig(batch_capacity=bcap, max_splits=smax, max_context=maxctx, query_heads=hkv * 2,
                           kv_heads=hkv, head_dim=128, page_size=16, workers=workers)
        g = geometry_of(cfg)
        lb = lengths + [0] * (bcap - n)
        sb = splits + [1] * (bcap - n)
        want = oracle_tables_in_golden_format(P.device_tables(lb, sb, n, g, 2), g)
        assert run_plan(cfg, lb, sb, n, 2, []) == want


@pytest.mark.parametrize("shards", [1, 2, 4, 8])
def test_plan_head_sharded_groups_match_oracle(shards, cuda_device):
    """Under KV-head sharding each GPU plans with groups = Hkv/N (C3)."""
    b = baseline("C3")
    c = b.config
    cfg = DecodeConfig(batch_capacity=c.batch_capacity, max_splits=c.max_splits,
                       max_context=c.max_context, query_heads=c.query_heads // shards,
                       kv_heads=c.kv_heads // shards, head_dim=c.head_dim, page_size=1,
                       workers=c.workers)
    g = geometry_of(cfg)
    for force in (1, 2, 4):
        want = oracle_tables_in_golden_format(
            P.device_tables(b.lengths, b.splits, len(b.lengths), g, force), g)
        assert run_plan(cfg, b.lengths, b.splits, len(b.lengths), force, []) == want


def test_plan_tables_stable_across_repeated_builds(cuda_device):
    cfg = DecodeConfig(workers=148)
    lengths = [256] * 24 + [1536] * 4 + [16384] * 4
    splits = split_hints(lengths)
    lb = lengths + [0] * (64 - 32)
    sb = splits + [1] * (64 - 32)
    first = run_plan(cfg, lb, sb, 32, 2, [])
    for _ in range(3):
        assert run_plan(cfg, lb, sb, 32, 2, []) == first
