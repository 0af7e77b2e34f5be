"""Pin the FP32 attention oracle and split/merge restatement to the reference.

Goldens (tests/golden/attention.npz) hold the reference's FP32 ``paged_attention``
outputs, and for fp16 cases its Triton decode + merge run by the Triton CPU
interpreter, including the partial/LSE slots of R1.
"""
import numpy as np
import pytest

from oracle import attention as A
from oracle import planning as P
from tests.golden import attention_arrays, attention_meta
from tests.golden.inputs import as_f32, load_case

CASES = attention_meta()


def _geometry(cfg):
    return P.Geometry(cfg["batch_capacity"], cfg["max_splits"], cfg["max_context"],
                      cfg["kv_heads"], cfg["workers"])


@pytest.mark.parametrize("meta", CASES, ids=[m["name"] for m in CASES])
def test_paged_oracle_matches_reference_fp32(meta):
    arrays = attention_arrays()
    q, k, v, pages = load_case(arrays, meta)
    got = A.paged_attention(as_f32(q), as_f32(k), as_f32(v), pages.numpy(), meta["lengths"],
                            meta["config"]["page_size"])
    np.testing.assert_allclose(got, arrays[f"{meta['name']}/oracle"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("meta", [m for m in CASES if m["config"]["page_size"] == 1],
                         ids=lambda m: m["name"])
def test_csr_oracle_equals_paged_oracle_for_page_size_one(meta):
    arrays = attention_arrays()
    q, k, v, pages = load_case(arrays, meta)
    lengths = meta["lengths"]
    indptr = np.concatenate([[0], np.cumsum(lengths)])
    indices = np.concatenate([pages.numpy()[r, :n] for r, n in enumerate(lengths)])
    got = A.csr_attention(as_f32(q), as_f32(k)[:, 0], as_f32(v)[:, 0], indptr, indices, lengths)
    np.testing.assert_allclose(got, arrays[f"{meta['name']}/oracle"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("meta", [m for m in CASES if m["triton_modes"]], ids=lambda m: m["name"])
def test_reference_kernels_agree_with_oracle_within_north_star_tolerance(meta):
    """The reference's own Triton path (interpreted, fp16) sits inside the 2e-2/2e-3 bar."""
    arrays = attention_arrays()
    n = len(meta["lengths"])
    expected = arrays[f"{meta['name']}/oracle"][:n]
    for mode in meta["triton_modes"]:
        got = arrays[f"{meta['name']}/triton_{mode}"][:n]
        max_abs, mean_abs = A.tolerance_report(got, expected)
        assert max_abs <= 2e-2 and mean_abs <= 2e-3, (mode, max_abs, mean_abs)


@pytest.mark.parametrize("meta", [m for m in CASES if m["triton_modes"]], ids=lambda m: m["name"])
def test_split_partials_and_merge_match_reference_slots(meta):
    """Slot assignment (request*Hq + head)*Smax + split and the LSE merge (merge.py)."""
    arrays = attention_arrays()
    cfg = meta["config"]
    g = _geometry(cfg)
    q, k, v, pages = load_case(arrays, meta)
    records, counts, _ = P.split_records(meta["lengths"], meta["splits"], g)
    rec = [(r.request, r.split, r.begin, r.end) for r in records]
    partial, lse = A.split_partials(as_f32(q), as_f32(k), as_f32(v), rec, cfg["max_splits"],
                                    pages=pages.numpy(), page_size=cfg["page_size"])
    ref_partial = arrays[f"{meta['name']}/triton_partial"]
    ref_lse = arrays[f"{meta['name']}/triton_lse"]
    written = ~np.isnan(ref_lse)
    assert np.array_equal(written, ~np.isnan(lse)), "slot sets differ"
    np.testing.assert_allclose(lse[written], ref_lse[written], atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(partial[written], ref_partial[written], atol=2e-2, rtol=1e-2)
    full_counts = counts + [0] * (cfg["batch_capacity"] - len(counts))
    merged = A.merge_splits(np.nan_to_num(partial), np.nan_to_num(lse), full_counts)
    np.testing.assert_allclose(merged, arrays[f"{meta['name']}/oracle"], atol=2e-5, rtol=1e-4)


def test_merge_error_flag_poisons_every_row():
    partial = np.zeros((2, 3, 4, 8), np.float32)
    lse = np.zeros((2, 3, 4), np.float32)
    assert np.isnan(A.merge_splits(partial, lse, [1, 0], error=1)).all()
    assert (A.merge_splits(partial, lse, [0, 0]) == 0).all()
