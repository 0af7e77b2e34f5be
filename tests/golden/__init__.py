"""Golden vectors produced by the reference (see make_golden.py) and their loaders."""
import gzip
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


@lru_cache(maxsize=None)
def plan_spec():
    with gzip.open(HERE / "plan_spec.json.gz", "rt") as f:
        return json.load(f)


@lru_cache(maxsize=None)
def plan_device():
    with gzip.open(HERE / "plan_device.json.gz", "rt") as f:
        return json.load(f)


@lru_cache(maxsize=None)
def attention_meta():
    return json.loads((HERE / "attention.json").read_text())


def attention_arrays():
    return np.load(HERE / "attention.npz")
