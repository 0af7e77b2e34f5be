"""Host STATIC planner and AUTO policy calibration (CPU): the host LPT lists equal the
reference LPT the GPU plan kernel reproduces, and ``freeze`` publishes a rule only when the
reference's adoption gates pass."""
import csv
import json
import random

import pytest

from oracle import planning as P
from sglang_decode.config import DecodeConfig
from sglang_decode.planning import calibrate as C
from sglang_decode.planning.host_static import lpt_lists, record_weights
from sglang_decode.planning.policy import load_policy
from sglang_decode.workloads import split_hints


@pytest.mark.parametrize("seed", range(30))
def test_host_lpt_lists_equal_the_reference_lpt(seed):
    rng = random.Random(seed)
    n = rng.randint(0, 48)
    maxctx = rng.choice([1000, 8192, 131072])
    lengths = [rng.choice([0, 1, 129, rng.randint(1, maxctx), maxctx]) for _ in range(n)]
    splits = split_hints(lengths, 16) if lengths else []
    groups, workers = rng.choice([1, 4, 7, 8]), rng.choice([1, 5, 148])
    cfg = DecodeConfig(batch_capacity=64, max_splits=16, max_context=maxctx, query_heads=groups * 2,
                       kv_heads=groups, head_dim=128, page_size=16, workers=workers)
    g = P.Geometry(cfg.batch_capacity, cfg.max_splits, cfg.max_context, groups, workers)
    want = P.device_tables(lengths + [0] * (64 - n), splits + [1] * (64 - n), n, g, 2)
    weights = record_weights(lengths, splits, cfg)
    assert weights == want["weight"][:want["record_count"]]
    head, links = lpt_lists(weights, groups, workers)
    assert head == want["static_head"][:workers]
    assert sorted(links.items()) == sorted(want["static_links"].items())


def _csv(path, medians, rounds=5, spread=0.01, status="ok"):
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["variant", "round", "status", "wall_us"])
        w.writeheader()
        for r in range(rounds):
            for name, m in medians.items():
                w.writerow({"variant": name, "round": r, "status": status,
                            "wall_us": m * (1 + spread * (r - rounds // 2) / rounds)})
    return path


def test_freeze_adopts_a_clear_dynamic_win_and_load_policy_accepts_it(tmp_path):
    times = {"R1": 200.0, "STATIC_CPU": 230.0, "D1": 185.0, "D4": 175.0}
    cal, hold = _csv(tmp_path / "cal.csv", times), _csv(tmp_path / "hold.csv", times)
    out = tmp_path / "policy.json"
    art = C.freeze(cal, hold, out, (512, 32768), (400, 10**6))
    assert art["rules"][0]["mode"] == 4 and art["status"] == "validated" and len(art["evidence"]) == 2
    rules = load_policy(out)
    assert rules[0].mode == 4 and rules[0].min_tasks == 512 and rules[0].max_ratio == 10**6
    with pytest.raises(FileExistsError):               # a published policy is never overwritten
        C.freeze(cal, hold, out, (512, 32768), (400, 10**6))


@pytest.mark.parametrize("d4", [197.0, 199.0])         # gains below 3%: R1 is kept
def test_freeze_keeps_round_robin_for_small_gains(tmp_path, d4):
    times = {"R1": 200.0, "STATIC_CPU": 230.0, "D1": 210.0, "D4": d4}
    art = C.freeze(_csv(tmp_path / "c.csv", times), _csv(tmp_path / "h.csv", times), tmp_path / "p.json",
                   (0, 100), (100, 200))
    assert art["rules"][0]["mode"] == 1


def test_freeze_rejects_overlapping_samples_for_dynamic_modes(tmp_path):
    times = {"R1": 200.0, "STATIC_CPU": 230.0, "D1": 210.0, "D4": 190.0}
    cal = _csv(tmp_path / "c.csv", times, spread=0.5)   # wide spread: D4's slowest >= R1's fastest
    art = C.freeze(cal, _csv(tmp_path / "h.csv", times), tmp_path / "p.json", (0, 100), (100, 200))
    assert art["rules"][0]["mode"] == 1


@pytest.mark.parametrize("case", ["holdout_regression", "holdout_small_gain", "host_static_wins",
                                  "failed_row", "few_rounds", "same_file"])
def test_freeze_publishes_nothing_when_a_gate_fails(tmp_path, case):
    cal_t = {"R1": 200.0, "STATIC_CPU": 230.0, "D1": 185.0, "D4": 175.0}
    hold_t = dict(cal_t)
    kwargs = {}
    if case == "holdout_regression":
        hold_t["D4"] = 210.0
    if case == "holdout_small_gain":
        hold_t["D4"] = 198.0
    if case == "host_static_wins":
        cal_t = hold_t = {"R1": 200.0, "STATIC_CPU": 150.0, "D1": 185.0, "D4": 175.0}
    cal = _csv(tmp_path / "c.csv", cal_t, status="failed" if case == "failed_row" else "ok",
               rounds=3 if case == "few_rounds" else 5)
    hold = cal if case == "same_file" else _csv(tmp_path / "h.csv", hold_t)
    with pytest.raises(C.CalibrationError):
        C.freeze(cal, hold, tmp_path / "p.json", (0, 100), (100, 200))
    assert not (tmp_path / "p.json").exists()


def test_shipped_b200_policy_is_validated_by_its_evidence():
    import hashlib
    from pathlib import Path

    import sglang_decode
    root = Path(sglang_decode.__file__).parent / "policies"
    art = json.loads((root / "b200_skewed.json").read_text())
    for ev in art["evidence"]:
        assert hashlib.sha256((root / ev["path"]).read_bytes()).hexdigest() == ev["sha256"]
    rules = load_policy(root / "b200_skewed.json")
    # With R1's claimed tail, D1 no longer clears the 3% gate on the C2 skew: R1 is published.
    assert [r.mode for r in rules] == [1]
    cal, hold = (C.read_rows(root / ev["path"]) for ev in art["evidence"])
    assert C.choose(cal, hold) == "R1"                    # the gates reproduce the published choice
