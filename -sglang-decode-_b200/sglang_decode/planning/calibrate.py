"""Calibrate an AUTO policy rule from measurements, with the reference's adoption gates.

Two steps, as in the reference (``scripts/calibrate_policy.py``):

* ``measure`` (GPU) times one workload under R1, STATIC_CPU (host LPT lists, see
  ``host_static.py``), D1 and D4, in rotating order, for several rounds, and writes one CSV
  row per (round, variant): ``variant, round, status, wall_us`` -- the host wall time of a
  whole step (plan build + decode + merge; host planning included for STATIC_CPU).
* ``freeze`` (CPU, never runs a kernel) reads a calibration CSV and an independent holdout
  CSV and publishes at most one rule for a stated task-count / weight-ratio range:
  a dynamic mode (D1/D4) is adopted only if its median beats the better static mode by at
  least 3% and its slowest round is faster than the static mode's fastest, and only if the
  holdout confirms it (median <= 97% of the holdout's better static mode, no overlap);
  any candidate that regresses the holdout by more than 2% publishes nothing; a winning
  host-static planner is reported and not replaced by the GPU LPT.  The artefact has the
  format ``load_policy`` accepts (``status: validated`` with the evidence files' SHA-256).

    python -m sglang_decode.planning.calibrate measure --workload C2 --seed 17 --output cal.csv
    python -m sglang_decode.planning.calibrate freeze cal.csv hold.csv --output policy.json \\
        --tasks 512 32768 --ratio 400 1000000
"""
from __future__ import annotations

import argparse
import csv
import hashlib
import json
import statistics
import time
from pathlib import Path

MODES = {"R1": 1, "STATIC_CPU": 2, "D1": 3, "D4": 4}
MIN_ROUNDS = 5


class CalibrationError(RuntimeError):
    """The measurements do not support publishing a rule."""


# ----------------------------------------------------------------------------- measure (GPU)
def measure(workload="C2", seed=17, rounds=5, iterations=50, warmup=5, device="cuda"):
    """Rows (variant, round, status, wall_us) for the four variants on one workload."""
    import torch

    from ..runtime.engine import DecodeEngine
    from ..workloads import baseline, generate, update_plan
    from .host_static import prepare_host_static

    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    torch.cuda.set_device(device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    b = baseline(workload, seed=seed, workers=sms)
    data = generate(b, device=device, seed=seed)
    args = (data["q"], data["k"], data["v"], data["pages"])
    engines = {}
    for name, mode in MODES.items():
        e = DecodeEngine(b.config, device=device, dtype=b.dtype, force_mode=-1 if name == "STATIC_CPU" else mode)
        update_plan(e, b.lengths, b.splits)
        engines[name] = e

    def step(name):
        e = engines[name]
        if name == "STATIC_CPU":
            prepare_host_static(e, b.lengths, b.splits)
        else:
            e.prepare()
        return e.execute(*args, indptr=data["indptr"])

    for name in MODES:
        for _ in range(warmup):
            step(name)
    torch.cuda.synchronize()
    rows, names = [], list(MODES)
    for r in range(rounds):
        for name in names[r % len(names):] + names[:r % len(names)]:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(iterations):
                out = step(name)
            torch.cuda.synchronize()
            wall = (time.perf_counter() - t0) / iterations * 1e6
            ok = engines[name].layers[0].status.item() == 0 and bool(torch.isfinite(out[:len(b.lengths)].float()).all())
            rows.append({"variant": name, "round": r, "status": "ok" if ok else "failed",
                         "wall_us": f"{wall:.3f}"})
    return rows


def write_rows(rows, path):
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["variant", "round", "status", "wall_us"])
        w.writeheader()
        w.writerows(rows)


# ----------------------------------------------------------------------------- freeze (CPU)
def read_rows(path):
    groups = {}
    with open(path, newline="") as f:
        for row in csv.DictReader(f):
            if row["status"] != "ok":
                raise CalibrationError(f"{path}: a failed sample must be investigated, not dropped")
            groups.setdefault(row["variant"], []).append(float(row["wall_us"]))
    for name in MODES:
        if len(groups.get(name, [])) < MIN_ROUNDS:
            raise CalibrationError(f"{path}: at least {MIN_ROUNDS} rounds of {name} are required")
    return groups


def choose(calibration, holdout):
    """The mode the measurements support (raises CalibrationError when none may be published)."""
    med = statistics.median
    best_static = min(("R1", "STATIC_CPU"), key=lambda n: med(calibration[n]))
    candidate = min(MODES, key=lambda n: med(calibration[n]))
    if candidate in ("D1", "D4"):
        gain = 1 - med(calibration[candidate]) / med(calibration[best_static])
        if gain < 0.03 or max(calibration[candidate]) >= min(calibration[best_static]):
            candidate = best_static
    hold_static = min(("R1", "STATIC_CPU"), key=lambda n: med(holdout[n]))
    if med(holdout[candidate]) > 1.02 * med(holdout[hold_static]):
        raise CalibrationError("holdout regression above 2%: no policy published")
    if candidate in ("D1", "D4") and (med(holdout[candidate]) > 0.97 * med(holdout[hold_static])
                                      or max(holdout[candidate]) >= min(holdout[hold_static])):
        raise CalibrationError("the dynamic mode's holdout benefit is below the adoption gate")
    if candidate == "STATIC_CPU":
        raise CalibrationError("the host static planner wins: keep it as the baseline; the GPU LPT "
                               "is not substituted for it in AUTO")
    return candidate


def freeze(calibration_csv, holdout_csv, output, tasks, ratio):
    calibration_csv, holdout_csv = Path(calibration_csv), Path(holdout_csv)
    if calibration_csv.resolve() == holdout_csv.resolve():
        raise CalibrationError("an independent holdout file is required")
    mode = choose(read_rows(calibration_csv), read_rows(holdout_csv))
    evidence = [{"path": p.name, "sha256": hashlib.sha256(p.read_bytes()).hexdigest()}
                for p in (calibration_csv, holdout_csv)]
    artefact = {"status": "validated", "evidence": evidence,
                "rules": [{"min_tasks": tasks[0], "max_tasks": tasks[1], "min_ratio": ratio[0],
                           "max_ratio": ratio[1], "mode": MODES[mode]}]}
    with open(output, "x") as f:          # never overwrite a published policy
        json.dump(artefact, f, indent=2)
    return artefact


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = parser.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("measure")
    m.add_argument("--workload", default="C2")
    m.add_argument("--seed", type=int, default=17)
    m.add_argument("--rounds", type=int, default=5)
    m.add_argument("--iterations", type=int, default=50)
    m.add_argument("--output", type=Path, required=True)
    f = sub.add_parser("freeze")
    f.add_argument("calibration", type=Path)
    f.add_argument("holdout", type=Path)
    f.add_argument("--output", type=Path, required=True)
    f.add_argument("--tasks", nargs=2, type=int, required=True)
    f.add_argument("--ratio", nargs=2, type=int, required=True)
    args = parser.parse_args(argv)
    if args.cmd == "measure":
        write_rows(measure(args.workload, args.seed, args.rounds, args.iterations), args.output)
        print(f"wrote {args.output}")
        return
    try:
        artefact = freeze(args.calibration, args.holdout, args.output, args.tasks, args.ratio)
    except CalibrationError as exc:
        raise SystemExit(str(exc)) from None
    print(json.dumps(artefact, indent=2))


if __name__ == "__main__":
    main()
