"""Shared helpers for the GPU parity tests (device tables, oracle comparisons)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import attention as A
from oracle import planning as P

PLAN_ARRAYS = ("counts", "offsets", "chunk", "request", "split", "begin", "end", "weight", "order",
               "pack_first", "pack_count", "record_count", "num_packs", "mode", "error",
               "static_head", "static_next")
POISON = -7


def geometry_of(config):
    return P.Geometry(config.batch_capacity, config.max_splits, config.max_context,
                      config.kv_heads, config.workers)


def poison_plan(plan):
    for name in PLAN_ARRAYS:
        getattr(plan, name).fill_(POISON)


def capture_tables(plan):
    """Read a device plan into the golden format (written prefixes + untouched flags)."""
    get = lambda name: getattr(plan, name).cpu().tolist()
    out = {name: int(getattr(plan, name).item()) for name in ("record_count", "num_packs", "mode", "error")}
    for name in ("counts", "offsets", "chunk", "static_head"):
        out[name] = get(name)
    total = max(out["record_count"], 0) if out["record_count"] != POISON else 0
    for name in ("request", "split", "begin", "end", "weight", "order"):
        full = get(name)
        out[name] = full[:total]
        out[name + "_tail_untouched"] = all(x == POISON for x in full[total:])
    packs = max(out["num_packs"], 0) if out["num_packs"] != POISON else 0
    for name in ("pack_first", "pack_count"):
        full = get(name)
        out[name] = full[:packs]
        out[name + "_tail_untouched"] = all(x == POISON for x in full[packs:])
    out["static_next"] = [[t, x] for t, x in enumerate(get("static_next")) if x != POISON]
    return out


def oracle_tables_in_golden_format(tables, geometry):
    """Convert oracle.planning.device_tables output to the golden/capture format."""
    e, t = geometry.record_capacity, geometry.task_capacity
    total = tables["record_count"]
    out = {name: tables[name] for name in ("record_count", "num_packs", "mode", "error", "counts",
                                           "chunk")}
    out["offsets"] = tables["offsets"]
    for name in ("request", "split", "begin", "end", "weight", "order"):
        vals = tables[name]
        out[name] = [POISON] * total if vals is None else list(vals[:total])
        out[name + "_tail_untouched"] = True
    for name in ("pack_first", "pack_count"):
        vals = tables[name]
        out[name] = [] if vals is None else list(vals)
        out[name + "_tail_untouched"] = True
    if tables["static_head"] is None:
        out["static_head"] = [POISON] * geometry.workers
        out["static_next"] = []
    else:
        out["static_head"] = list(tables["static_head"])
        out["static_next"] = sorted([list(kv) for kv in tables["static_links"].items()])
    del e, t
    return out


def f32(t):
    return t.detach().float().cpu().numpy()


def oracle_paged(q, k, v, pages, lengths, page_size, scale=None, logit_cap=0.0):
    return A.paged_attention(f32(q), f32(k), f32(v), pages.cpu().numpy(), lengths, page_size, scale,
                             logit_cap)


def oracle_csr(q, k, v, indptr, indices, lengths, scale=None, logit_cap=0.0):
    return A.csr_attention(f32(q), f32(k), f32(v), indptr.cpu().numpy(), indices.cpu().numpy(),
                           lengths, scale, logit_cap)


def assert_within_tolerance(actual, expected, n, max_abs=2e-2, mean_abs=2e-3):
    """max-abs <= 2e-2 and mean-abs <= 2e-3 vs the FP32 oracle."""
    got = f32(actual)[:n] if isinstance(actual, torch.Tensor) else np.asarray(actual)[:n]
    exp = np.asarray(expected)[:n]
    assert np.isfinite(got).all(), "non-finite output"
    worst, mean = A.tolerance_report(got, exp)
    assert worst <= max_abs and mean <= mean_abs, (worst, mean)
    return worst, mean


def oracle_requests(q, k, v, lengths, *, indptr=None, indices=None, pages=None, page_size=1,
                    requests=None, scale=None, logit_cap=0.0):
    """FP32 oracle rows [len(lengths), Hq, D] for ``requests`` (default: every request).

    Each request's K/V rows are gathered on their own device in token order (CSR:
    ``indices[indptr[r] + t]``; paged: ``pages[r, t // page_size]``, row ``t % page_size``)
    and only those rows are upcast and copied to the host, so pools of many GB can be
    checked.  Rows of requests not selected stay zero."""
    wanted = range(len(lengths)) if requests is None else requests
    out = np.zeros((len(lengths), q.shape[1], q.shape[2]), dtype=np.float32)
    starts = indptr.cpu().tolist() if indptr is not None else None
    for r in wanted:
        n = int(lengths[r])
        if n == 0:
            continue
        if starts is not None:
            rows = indices[starts[r]:starts[r] + n].long()
            key, value = k[rows], v[rows]
        else:
            t = torch.arange(n, device=k.device)
            phys = pages[r, t // page_size].long()
            key, value = k[phys, t % page_size], v[phys, t % page_size]
        out[r] = A.request_attention(f32(q[r]), f32(key), f32(value), scale, logit_cap)
    return out


def assert_rows_within_tolerance(actual, expected, rows, max_abs=2e-2, mean_abs=2e-3):
    """The tolerance bar on the selected request rows only."""
    rows = list(rows)
    got = f32(actual)[rows]
    exp = np.asarray(expected)[rows]
    assert np.isfinite(got).all(), "non-finite output"
    worst, mean = A.tolerance_report(got, exp)
    assert worst <= max_abs and mean <= mean_abs, (worst, mean)
    return worst, mean
