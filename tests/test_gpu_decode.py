"""GPU decode outputs vs the FP32 oracle and the reference's own kernel outputs.

Ports the reference's tests/gpu/test_decode.py (every Mode x mixed/B lengths,
NaN-poisoned partial/LSE, GPU records vs the CPU spec, non-contiguous K/V) and adds
CSR indexing, group sizes 1..16 (incl. 7), head dims 64/128/256, fp16/bf16, slot-level
partial/LSE checks, the stand-alone merge, the error path and mode invariance.
Tolerance (north star): max-abs <= 2e-2 and mean-abs <= 2e-3 against FP32.
"""
import numpy as np
import pytest
import torch

from oracle import attention as A
from oracle import planning as P
from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.runtime.engine import DecodeEngine, merge_splits
from sglang_decode.workloads import make_csr_inputs, make_inputs, split_hints, update_plan
from tests.golden import attention_arrays, attention_meta
from tests.golden.inputs import load_case
from tests.helpers import assert_within_tolerance, f32, geometry_of, oracle_csr, oracle_paged

pytestmark = pytest.mark.gpu

MIXED = [0, 1, 17, 33, 257, 513]
B = [256] * 24 + [1536] * 4 + [16384] * 4


def run(engine, inputs, lengths, splits=None, indptr=None, layer=0, scale=None, logit_cap=0.0, k_scale=1.0,
        v_scale=1.0):
    update_plan(engine, lengths, splits)
    lb = engine.layers[layer]
    lb.partial.fill_(float("nan"))
    lb.lse.fill_(float("nan"))
    engine.prepare()
    q, k, v, pages = inputs
    out = engine.execute(q, k, v, pages, layer=layer, indptr=indptr, scale=scale, logit_cap=logit_cap,
                         k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    assert lb.status.item() == 0, "bounded in-kernel wait expired"
    assert engine.counters.eq(0).all(), "claim words not left at zero"
    return out


@pytest.mark.parametrize("mode", list(Mode))
@pytest.mark.parametrize("lengths", [MIXED, B], ids=["mixed", "B"])
def test_outputs_and_gpu_records(mode, lengths, cuda_device):
    c = DecodeConfig()
    engine = DecodeEngine(c, force_mode=mode)
    inputs = make_inputs(c, lengths, device="cpu")
    inputs = tuple(t.cuda() for t in inputs)
    out = run(engine, inputs, lengths)
    expected = oracle_paged(*inputs, lengths, c.page_size)
    assert_within_tolerance(out, expected, len(lengths))
    assert (f32(out)[len(lengths):] == 0).all(), "inactive rows must be zero"
    assert engine.plan.error.item() == 0
    records, counts, _ = P.split_records(lengths, split_hints(lengths), geometry_of(c))
    assert engine.plan.record_count.item() == len(records)
    assert engine.plan.counts[:len(lengths)].tolist() == counts
    if mode != Mode.R0:
        assert engine.plan.request[:len(records)].tolist() == [r.request for r in records]
        assert engine.plan.begin[:len(records)].tolist() == [r.begin for r in records]
    if mode in (Mode.D1, Mode.D4):
        order = P.bucket_order(records)
        packs = P.make_packs(records, order, c.kv_heads, c.workers, pack_limit=1 if mode == Mode.D1 else 4)
        assert engine.plan.order[:len(records)].tolist() == order
        count = engine.plan.num_packs.item()
        assert list(zip(engine.plan.pack_first[:count].tolist(),
                        engine.plan.pack_count[:count].tolist())) == packs
    if mode == Mode.STATIC:
        lists = P.greedy_static(records, c.kv_heads, c.workers)
        walked = P.lists_from_links(engine.plan.static_head.tolist(), engine.plan.static_next.tolist(),
                                    c.workers, len(records) * c.kv_heads)
        assert walked == lists


def test_noncontiguous_kv_strides(cuda_device):
    c = DecodeConfig()
    lengths = [17, 513]
    q, k, v, pages = (t.cuda() for t in make_inputs(c, lengths, device="cpu"))

    def strided(x):
        storage = torch.empty((*x.shape[:-1], x.shape[-1] * 2), device=x.device, dtype=x.dtype)
        storage[..., ::2].copy_(x)
        return storage[..., ::2]

    k, v = strided(k), strided(v)
    engine = DecodeEngine(c, force_mode=Mode.D4)
    out = run(engine, (q, k, v, pages), lengths)
    assert_within_tolerance(out, oracle_paged(q, k, v, pages, lengths, c.page_size), 2)


@pytest.mark.parametrize("mode", list(Mode))
def test_modes_are_bit_identical(mode, cuda_device):
    """Dispatch order never changes a slot's arithmetic, so every mode gives the same bits."""
    c = DecodeConfig()
    lengths = B
    inputs = tuple(t.cuda() for t in make_inputs(c, lengths, device="cpu"))
    base = run(DecodeEngine(c, force_mode=Mode.R1), inputs, lengths).clone()
    got = run(DecodeEngine(c, force_mode=mode), inputs, lengths)
    assert torch.equal(base, got)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("group,head_dim", [(1, 128), (2, 64), (4, 128), (7, 128), (8, 128), (8, 64),
                                            (8, 256), (16, 128), (12, 64), (16, 256), (3, 256)])
@pytest.mark.parametrize("mode", [Mode.R1, Mode.D4])
def test_csr_group_sizes_and_head_dims(dtype, group, head_dim, mode, cuda_device):
    hkv = 2 if group > 4 else 4
    lengths = [1, 65, 300, 0, 1000, 129, 64]
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=hkv * group,
                     kv_heads=hkv, head_dim=head_dim, page_size=1, workers=37)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", dtype=dtype,
                                                               pool=4000))
    engine = DecodeEngine(c, dtype=dtype, force_mode=mode)
    out = run(engine, (q, k, v, idx), lengths, indptr=indptr)
    expected = oracle_csr(q, k, v, indptr, idx, lengths)
    assert_within_tolerance(out, expected, len(lengths))


@pytest.mark.parametrize("cap", [2.0, 20.0, 50.0])
@pytest.mark.parametrize("layout", ["csr_g8", "csr_g7", "paged64_g4", "paged16_g16_d256"])
def test_logit_soft_cap_matches_oracle_in_every_mode(cap, layout, cuda_device):
    """SGLang's soft cap (s -> cap * tanh(s / cap)); Q scaled up so that the cap bites."""
    lengths = [1, 65, 300, 0, 1000, 129, 700]
    group, hkv, d = {"csr_g8": (8, 2, 128), "csr_g7": (7, 2, 128), "paged64_g4": (4, 4, 128),
                     "paged16_g16_d256": (16, 1, 256)}[layout]
    ps = {"paged64_g4": 64, "paged16_g16_d256": 16}.get(layout, 1)
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=hkv * group,
                     kv_heads=hkv, head_dim=d, page_size=ps, workers=37)
    if ps == 1:
        q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=4000))
        inputs = (4.0 * q, k, v, idx)
        expected = oracle_csr(4.0 * q, k, v, indptr, idx, lengths, logit_cap=cap)
        plain = oracle_csr(4.0 * q, k, v, indptr, idx, lengths)
    else:
        indptr = None
        q, k, v, pages = (t.cuda() for t in make_inputs(c, lengths, device="cpu"))
        inputs = (4.0 * q, k, v, pages)
        expected = oracle_paged(4.0 * q, k, v, pages, lengths, ps, logit_cap=cap)
        plain = oracle_paged(4.0 * q, k, v, pages, lengths, ps)
    assert np.abs(expected - plain).max() > 1e-2, "the cap must change the result in this case"
    outs = []
    for mode in (Mode.R0, Mode.R1, Mode.STATIC, Mode.D1, Mode.D4):
        out = run(DecodeEngine(c, force_mode=mode), inputs, lengths, indptr=indptr, logit_cap=cap)
        assert_within_tolerance(out, expected, len(lengths))
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every dispatch mode gives identical outputs"


FP8 = getattr(torch, "float8_e4m3fn", None)


@pytest.mark.skipif(FP8 is None, reason="torch without float8_e4m3fn")
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("layout", ["csr_g8", "csr_g7", "csr_g16", "paged16_g4", "paged64_g8", "csr_strided_g4"])
@pytest.mark.parametrize("scales", [(1.0, 1.0), (0.5, 2.0)], ids=["unscaled", "scaled"])
def test_fp8_kv_matches_oracle_in_every_mode(qdtype, layout, scales, cuda_device):
    """e4m3 K/V with a fp16/bf16 Q: the oracle sees the same fp8 values (dequantised, times
    k_scale / v_scale); every dispatch mode gives identical outputs."""
    lengths = [1, 65, 300, 0, 1000, 129, 700]
    group, hkv = {"csr_g8": (8, 2), "csr_g7": (7, 2), "csr_g16": (16, 1), "paged16_g4": (4, 4),
                  "paged64_g8": (8, 2), "csr_strided_g4": (4, 2)}[layout]
    ps = {"paged16_g4": 16, "paged64_g8": 64}.get(layout, 1)
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=hkv * group,
                     kv_heads=hkv, head_dim=128, page_size=ps, workers=37)
    ks, vs = scales
    if ps == 1:
        q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", dtype=qdtype,
                                                                   pool=4000))
        k8, v8 = k.to(FP8), v.to(FP8)
        if layout == "csr_strided_g4":                 # rows 160 bytes apart: the element-copy path
            wide_k = torch.zeros(k.shape[0], hkv, 160, device="cuda", dtype=FP8)
            wide_v = torch.zeros_like(wide_k)
            wide_k[..., :128], wide_v[..., :128] = k8, v8
            k8, v8 = wide_k[..., :128], wide_v[..., :128]
        pages = idx
        expected = oracle_csr(q, k8.float() * ks, v8.float() * vs, indptr, idx, lengths)
    else:
        indptr = None
        q, k, v, pages = (t.cuda() for t in make_inputs(c, lengths, device="cpu", dtype=qdtype))
        k8, v8 = k.to(FP8), v.to(FP8)
        expected = oracle_paged(q, k8.float() * ks, v8.float() * vs, pages, lengths, ps)
    outs = []
    for mode in (Mode.R0, Mode.R1, Mode.STATIC, Mode.D1, Mode.D4):
        out = run(DecodeEngine(c, dtype=qdtype, force_mode=mode), (q, k8, v8, pages), lengths, indptr=indptr,
                  k_scale=ks, v_scale=vs)
        assert_within_tolerance(out, expected, len(lengths))
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every dispatch mode gives identical outputs"


@pytest.mark.skipif(FP8 is None, reason="torch without float8_e4m3fn")
def test_fp8_kv_rejects_other_head_dims_and_mixed_kv(cuda_device):
    lengths = [10, 20]
    c = DecodeConfig(batch_capacity=2, max_splits=2, max_context=64, query_heads=8, kv_heads=2,
                     head_dim=64, page_size=1, workers=4)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=64))
    engine = DecodeEngine(c)
    update_plan(engine, lengths)
    engine.prepare()
    with pytest.raises(ValueError):                    # fp8 K/V: head_dim 128 only
        engine.execute(q, k.to(FP8), v.to(FP8), idx, indptr=indptr)
    with pytest.raises(ValueError):                    # K and V must share a dtype
        engine.execute(q, k.to(FP8), v, idx, indptr=indptr)
    with pytest.raises(ValueError):
        engine.execute(q, k, v, idx, indptr=indptr, k_scale=0.0)


def test_logit_cap_must_be_finite_and_non_negative(cuda_device):
    c = DecodeConfig(batch_capacity=2, max_splits=2, max_context=64, query_heads=8, kv_heads=2,
                     head_dim=128, page_size=1, workers=4)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, [10, 20], device="cpu", pool=64))
    engine = DecodeEngine(c)
    update_plan(engine, [10, 20])
    engine.prepare()
    for bad in (-1.0, float("nan"), float("inf")):
        with pytest.raises(ValueError):
            engine.execute(q, k, v, idx, indptr=indptr, logit_cap=bad)


@pytest.mark.parametrize("page_size", [1, 8, 16, 64])
def test_paged_page_sizes(page_size, cuda_device):
    lengths = [700, 3, 64, 129, 2000]
    c = DecodeConfig(batch_capacity=6, max_splits=4, max_context=2048, query_heads=16, kv_heads=2,
                     head_dim=128, page_size=page_size, workers=148)
    inputs = tuple(t.cuda() for t in make_inputs(c, lengths, device="cpu"))
    out = run(DecodeEngine(c, force_mode=Mode.D4), inputs, lengths)
    assert_within_tolerance(out, oracle_paged(*inputs, lengths, page_size), len(lengths))


def test_partial_and_lse_slots_match_oracle(cuda_device):
    """Merge slot assignment (request*Hq + head)*Smax + split, exact set of written slots."""
    c = DecodeConfig(workers=148)
    lengths = MIXED + [2048, 4095]
    inputs = tuple(t.cuda() for t in make_inputs(c, lengths, device="cpu"))
    for mode in Mode:
        engine = DecodeEngine(c, force_mode=mode)
        run(engine, inputs, lengths)
        records, _, _ = P.split_records(lengths, split_hints(lengths), geometry_of(c))
        rec = [(r.request, r.split, r.begin, r.end) for r in records]
        q, k, v, pages = inputs
        partial, lse = A.split_partials(f32(q), f32(k), f32(v), rec, c.max_splits,
                                        pages=pages.cpu().numpy(), page_size=c.page_size)
        got_lse = f32(engine.layers[0].lse)
        got_partial = f32(engine.layers[0].partial)
        written = ~np.isnan(lse)
        assert np.array_equal(written, ~np.isnan(got_lse)), "slot sets differ"
        np.testing.assert_allclose(got_lse[written], lse[written], atol=2e-2, rtol=0)
        assert np.abs(got_partial[written] - partial[written]).max() <= 2e-2


def test_standalone_merge_matches_oracle(cuda_device):
    rng = np.random.default_rng(3)
    b, hq, smax, d = 5, 6, 7, 128
    partial = rng.standard_normal((b, hq, smax, d)).astype(np.float32)
    lse = (rng.standard_normal((b, hq, smax)) * 4).astype(np.float32)
    counts = [0, 1, 3, 7, 2]
    partial_t = torch.from_numpy(partial).cuda()
    partial_t[0].fill_(float("nan"))             # slots >= counts must never be read
    partial_t[2, :, 3:].fill_(float("nan"))
    lse_t = torch.from_numpy(lse).cuda()
    counts_t = torch.tensor(counts, dtype=torch.int32, device="cuda")
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    for dtype in (torch.bfloat16, torch.float16):
        out = torch.empty((b, hq, d), dtype=dtype, device="cuda")
        merge_splits(partial_t, lse_t, counts_t, error, out)
        want = A.merge_splits(np.nan_to_num(partial), lse, counts)
        assert_within_tolerance(out, want, b, max_abs=1e-2, mean_abs=1e-3)
        error.fill_(1)
        merge_splits(partial_t, lse_t, counts_t, error, out)
        assert torch.isnan(out.float()).all()
        error.fill_(0)


@pytest.mark.parametrize("bad", ["negative_length", "long_length", "zero_splits", "active_over"])
def test_invalid_metadata_turns_every_output_nan(bad, cuda_device):
    c = DecodeConfig(batch_capacity=4, max_splits=4, max_context=512, query_heads=8, kv_heads=2,
                     head_dim=64, page_size=16, workers=9)
    lengths = [100, 200, 300]
    inputs = tuple(t.cuda() for t in make_inputs(c, lengths, device="cpu"))
    engine = DecodeEngine(c, force_mode=Mode.D4)
    update_plan(engine, lengths)
    p = engine.plan
    if bad == "negative_length":
        p.lengths[1] = -5
    elif bad == "long_length":
        p.lengths[2] = 513
    elif bad == "zero_splits":
        p.splits[0] = 0
    else:
        p.active.fill_(5)
    engine.prepare()
    out = engine.execute(*inputs)
    torch.cuda.synchronize()
    assert p.error.item() == 1
    assert p.record_count.item() == 0
    assert torch.isnan(out.float()).all()
    assert engine.layers[0].status.item() == 0


def test_empty_batch_writes_zeros(cuda_device):
    c = DecodeConfig(batch_capacity=4, max_splits=4, max_context=512, query_heads=8, kv_heads=2,
                     head_dim=64, page_size=16, workers=9)
    inputs = tuple(t.cuda() for t in make_inputs(c, [1], device="cpu"))
    engine = DecodeEngine(c)
    engine.layers[0].output.fill_(float("nan"))
    out = run(engine, inputs, [])
    assert (out.float() == 0).all()


GOLDEN = attention_meta()


@pytest.mark.parametrize("meta", GOLDEN, ids=[m["name"] for m in GOLDEN])
def test_golden_cases_match_reference(meta, cuda_device):
    """Reference-produced inputs: FP32 oracle and (fp16) the reference's Triton outputs."""
    arrays = attention_arrays()
    q, k, v, pages = (t.cuda() for t in load_case(arrays, meta))
    cfg = DecodeConfig(**meta["config"])
    lengths, splits = meta["lengths"], meta["splits"]
    if cfg.page_size == 1:
        # Golden K/V are paged with one token per page; run them through CSR indexing too.
        table = pages.cpu().numpy()
        rows = [table[r, :n] for r, n in enumerate(lengths)]
        indices = torch.tensor(np.concatenate(rows) if rows else [], dtype=torch.int32, device="cuda")
        indptr = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]).tolist()
                              + [sum(lengths)] * (cfg.batch_capacity + 1 - len(lengths) - 1),
                              dtype=torch.int32, device="cuda")
        k3, v3 = k[:, 0], v[:, 0]
    for mode in Mode:
        engine = DecodeEngine(cfg, dtype=q.dtype, force_mode=mode)
        out = run(engine, (q, k, v, pages), lengths, splits)
        n = len(lengths)
        assert_within_tolerance(out, arrays[f"{meta['name']}/oracle"], n)
        if int(mode) in meta["triton_modes"]:
            assert_within_tolerance(out, arrays[f"{meta['name']}/triton_{int(mode)}"], n)
        if cfg.page_size == 1:
            out2 = run(engine, (q, k3, v3, indices), lengths, splits, indptr=indptr)
            assert torch.equal(out, out2), "CSR and one-token paged indexing must agree bitwise"
