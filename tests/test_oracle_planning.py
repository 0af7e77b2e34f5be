"""Pin the CPU planning oracle to the reference (golden vectors + its known answers).

The goldens come from the reference's own CPU spec and from its Triton plan
kernels executed by the Triton CPU interpreter (tests/golden/make_golden.py).
"""
import pytest

from oracle import planning as P
from tests.golden import plan_device, plan_spec


def _geometry(case):
    return P.Geometry(case["batch_capacity"], case["max_splits"], case["max_context"],
                      case["groups"], case["workers"])


@pytest.mark.parametrize("index", range(len(plan_spec()["cases"])))
def test_spec_matches_reference_cpu_spec(index):
    case = plan_spec()["cases"][index]
    g = _geometry(case)
    records, counts, offsets = P.split_records(case["lengths"], case["splits"], g)
    assert [[r.request, r.split, r.begin, r.end, r.weight] for r in records] == case["records"]
    assert counts == case["counts"] and offsets == case["offsets"]
    order = P.bucket_order(records)
    assert order == case["order"]
    assert [list(p) for p in P.make_packs(records, order, g.groups, g.workers, 4)] == case["packs_d4"]
    assert [list(p) for p in P.make_packs(records, order, g.groups, g.workers, 1)] == case["packs_d1"]
    assert P.greedy_static(records, g.groups, g.workers) == case["static_lists"]
    P.validate_plan(records, order, P.make_packs(records, order, g.groups, g.workers), g.groups)


@pytest.mark.parametrize("index", range(len(plan_spec()["rejected"])))
def test_spec_rejections_match_reference(index):
    case = plan_spec()["rejected"][index]
    g = P.Geometry(64, 16, 32768, 8, 108)
    if case["raised"]:
        with pytest.raises(ValueError):
            P.split_records(case["lengths"], case["splits"], g)
    else:
        P.split_records(case["lengths"], case["splits"], g)


# Known answers restated from the reference's tests/unit/test_planning.py:9-54.
@pytest.mark.parametrize("lengths,splits,records_count,pack_count", [
    ([512] * 24 + [8192] * 8, [1] * 24 + [16] * 8, 152, 1216),
    ([256] * 24 + [1536] * 4 + [16384] * 4, [1] * 24 + [2] * 4 + [16] * 4, 96, 705),
    (([256] * 24 + [1536] * 4 + [16384] * 4) * 2, ([1] * 24 + [2] * 4 + [16] * 4) * 2, 192, 1329),
])
def test_documented_task_geometry(lengths, splits, records_count, pack_count):
    g = P.Geometry(64, 16, 32768, 8, 108)
    records, counts, offsets = P.split_records(lengths, splits, g)
    order = P.bucket_order(records)
    packs = P.make_packs(records, order, g.groups, g.workers)
    assert len(records) == records_count == sum(counts) == offsets[-1]
    assert len(packs) == pack_count
    P.validate_plan(records, order, packs, g.groups)
    longest = max(r.weight for r in records)
    for first, count in packs:
        assert 1 <= count <= 4
        assert sum(records[order[t // g.groups]].weight for t in range(first, first + count)) <= longest


def test_tail_and_zero_lengths_preserve_original_split_slots():
    records, counts, _ = P.split_records([0, 1, 33, 513], [16, 16, 16, 2], P.Geometry(64, 16, 32768, 8, 108))
    assert counts == [0, 1, 2, 2]
    assert [(r.begin, r.end) for r in records if r.request == 3] == [(0, 288), (288, 513)]
    assert all(r.begin < r.end for r in records)


def test_small_bucket_remains_singletons():
    g = P.Geometry(64, 16, 32768, 8, 108)
    records, _, _ = P.split_records([128, 1024], [1, 1], g)
    assert all(count == 1 for _, count in P.make_packs(records, P.bucket_order(records), 8, 108))


def test_static_lists_cover_tasks_and_balance_uniform_work():
    g = P.Geometry(64, 16, 32768, 8, 4)
    records, _, _ = P.split_records([512] * 8, [1] * 8, g)
    lists = P.greedy_static(records, g.groups, g.workers)
    assert sorted(t for w in lists for t in w) == list(range(64))
    assert {len(w) for w in lists} == {16}


def _device_case(case):
    cfg = case["config"]
    g = P.Geometry(cfg["batch_capacity"], cfg["max_splits"], cfg["max_context"], cfg["kv_heads"],
                   cfg["workers"])
    assert g.buckets == case["buckets"]
    return g, P.device_tables(case["lengths_buf"], case["splits_buf"], case["active"], g,
                              case["force"], case["rules"])


def assert_tables_match(got, golden, geometry):
    """Compare oracle tables with a reference device capture (stale entries = untouched)."""
    for name in ("record_count", "num_packs", "mode", "error", "counts", "offsets", "chunk"):
        assert got[name] == golden[name], name
    total = golden["record_count"]
    for name in ("request", "split", "begin", "end", "weight", "order"):
        if got[name] is None:
            assert golden[name] == [-7] * len(golden[name]), name
        else:
            assert got[name][:total] == golden[name], name
        assert golden[name + "_tail_untouched"], name
    if got["pack_first"] is not None:
        assert got["pack_first"] == golden["pack_first"]
        assert got["pack_count"] == golden["pack_count"]
    else:
        assert golden["pack_first"] == [-7] * len(golden["pack_first"])
    if got["static_head"] is None:
        assert all(h == -7 for h in golden["static_head"])
        assert golden["static_next"] == []
    else:
        assert got["static_head"] == golden["static_head"]
        assert sorted(got["static_links"].items()) == [tuple(x) for x in golden["static_next"]]


@pytest.mark.parametrize("index", range(len(plan_device()["cases"])))
def test_device_tables_match_reference_kernels(index):
    case = plan_device()["cases"][index]
    g, got = _device_case(case)
    assert_tables_match(got, case["outputs"], g)


def test_device_goldens_cover_every_mode_and_the_error_path():
    cases = plan_device()["cases"]
    assert {c["outputs"]["mode"] for c in cases} >= {0, 1, 2, 3, 4}
    assert any(c["outputs"]["error"] for c in cases)
    assert any(c["rules"] for c in cases)


def test_device_tables_agree_with_cpu_spec_on_valid_input():
    """GPU table semantics restate the CPU spec on valid metadata (spec <-> device bridge)."""
    for case in plan_spec()["cases"][:40]:
        g = _geometry(case)
        n = len(case["lengths"])
        buf_l = case["lengths"] + [0] * (g.batch_capacity - n)
        buf_s = case["splits"] + [1] * (g.batch_capacity - n)
        for force, packs in ((3, case["packs_d1"]), (4, case["packs_d4"])):
            t = P.device_tables(buf_l, buf_s, n, g, force)
            if t["record_count"] == 0:
                continue
            assert t["order"] == case["order"]
            assert [list(p) for p in zip(t["pack_first"], t["pack_count"])] == packs
        t = P.device_tables(buf_l, buf_s, n, g, 2)
        links = [t["static_links"].get(i, -1) for i in range(g.task_capacity)]
        walked = P.lists_from_links(t["static_head"], links, g.workers, t["record_count"] * g.groups)
        assert walked == case["static_lists"]
