"""Every decode kernel against the FP32 oracle: the persistent mma.sync kernel, the small-batch
kernel (one CTA per task) and the tcgen05 kernel (QK and PV on tcgen05.mma with tensor-memory
accumulators, head_dim 128, 16-bit K/V).

SGLD_DECODE_KERNEL selects the kernel per call ("mma" / "small" / "tcgen05"); each case asserts
which kernel actually ran (sgld_decode_kernel_kind), so a silent fallback cannot pass for
coverage (the small-batch kernel serves groups of at most 8).
Tolerance: max-abs 2e-2, mean-abs 2e-3 against FP32; every dispatch mode bit-identical.
"""
import numpy as np
import pytest
import torch

from oracle import attention as A
from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import baseline, generate, make_csr_inputs, make_inputs, subset, update_plan
from tests.helpers import assert_rows_within_tolerance, assert_within_tolerance, oracle_csr, oracle_paged, oracle_requests

pytestmark = pytest.mark.gpu

KERNELS = {"mma": {"mma.sync", "mma.sync+tma"}, "small": {"small"}, "tcgen05": {"tcgen05", "tcgen05+tma"}}


def _expect(kernel, group=8):
    """Kernels a call may take: the small-batch kernel only serves groups of at most 8."""
    return KERNELS["mma"] if kernel == "small" and group > 8 else KERNELS[kernel]


@pytest.fixture(params=sorted(KERNELS))
def kernel(request, monkeypatch):
    monkeypatch.setenv("SGLD_DECODE_KERNEL", request.param)
    return request.param


def _run(engine, inputs, lengths, indptr=None, **kw):
    update_plan(engine, lengths)
    engine.layers[0].partial.fill_(float("nan"))
    engine.prepare()
    q, k, v, pages = inputs
    out = engine.execute(q, k, v, pages, indptr=indptr, **kw)
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() == 0, "bounded in-kernel wait expired"
    assert engine.counters.eq(0).all()
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("group", [1, 3, 4, 7, 8, 12, 16])
def test_csr_groups(kernel, dtype, group):
    hkv = 2 if group > 4 else 4
    lengths = [1, 65, 300, 0, 1000, 129, 64, 128]
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=hkv * group, kv_heads=hkv,
                     head_dim=128, page_size=1, workers=37)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", dtype=dtype, pool=4000))
    expected = oracle_csr(q, k, v, indptr, idx, lengths)
    outs = []
    for mode in Mode:
        engine = DecodeEngine(c, dtype=dtype, force_mode=mode)
        out = _run(engine, (q, k, v, idx), lengths, indptr=indptr)
        assert engine.kernel_kind() in _expect(kernel, group)
        assert_within_tolerance(out, expected, len(lengths))
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every mode gives the same bits"


@pytest.mark.parametrize("page_size", [1, 16, 32, 64])
def test_paged_page_sizes(kernel, page_size):
    lengths = [700, 3, 64, 129, 2000, 32]
    c = DecodeConfig(batch_capacity=6, max_splits=4, max_context=2048, query_heads=16, kv_heads=2, head_dim=128,
                     page_size=page_size, workers=148)
    inputs = tuple(t.cuda() for t in make_inputs(c, lengths, device="cpu"))
    engine = DecodeEngine(c, force_mode=Mode.D4)
    out = _run(engine, inputs, lengths)
    assert engine.kernel_kind() in KERNELS[kernel]
    assert_within_tolerance(out, oracle_paged(*inputs, lengths, page_size), len(lengths))


@pytest.mark.parametrize("cap", [0.0, 5.0, 30.0])
def test_logit_cap_and_large_scores(kernel, cap):
    """Q scaled up so scores reach tens of units: the running maximum grows across tiles, which
    exercises the tcgen05 kernel's in-place rescale of the output in tensor memory."""
    lengths = [1000, 300, 900]
    c = DecodeConfig(batch_capacity=3, max_splits=2, max_context=1024, query_heads=16, kv_heads=2, head_dim=128,
                     page_size=1, workers=20)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=3000))
    # Later tokens of each request get larger keys, so tile maxima keep rising.
    position = torch.zeros(k.shape[0], device="cuda")
    position[idx.long()] = torch.arange(idx.numel(), device="cuda", dtype=position.dtype) / idx.numel()
    k = (k.float() * (0.2 + 2.8 * position).view(-1, 1, 1)).to(torch.bfloat16)
    q = (4.0 * q.float()).to(torch.bfloat16)
    expected = oracle_csr(q, k, v, indptr, idx, lengths, logit_cap=cap)
    engine = DecodeEngine(c, force_mode=Mode.R1)
    out = _run(engine, (q, k, v, idx), lengths, indptr=indptr, logit_cap=cap)
    assert engine.kernel_kind() in KERNELS[kernel]
    assert_within_tolerance(out, expected, len(lengths))


def test_strided_q_falls_back_to_the_mma_kernel(monkeypatch):
    """A Q whose rows are not 16-byte aligned cannot be loaded by a TMA box: the call still
    succeeds on the mma.sync kernel even when tcgen05 is requested."""
    monkeypatch.setenv("SGLD_DECODE_KERNEL", "tcgen05")
    lengths = [100, 300]
    c = DecodeConfig(batch_capacity=2, max_splits=2, max_context=512, query_heads=8, kv_heads=2, head_dim=128,
                     page_size=1, workers=8)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=512))
    storage = torch.zeros(2, 8, 129, dtype=q.dtype, device="cuda")
    storage[..., :128] = q
    q_odd = storage[..., :128]
    engine = DecodeEngine(c)
    out = _run(engine, (q_odd, k, v, idx), lengths, indptr=indptr)
    assert engine.kernel_kind() == "mma.sync"
    assert_within_tolerance(out, oracle_csr(q, k, v, indptr, idx, lengths), len(lengths))


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4"])
def test_baseline_shapes_on_the_tcgen05_kernel(monkeypatch, name):
    """The benchmark configurations' real shapes (C3: 16-request prefix, C4: 3 requests)."""
    monkeypatch.setenv("SGLD_DECODE_KERNEL", "tcgen05")
    b = baseline(name, workers=torch.cuda.get_device_properties(0).multi_processor_count)
    b = {"C3": subset(b, 16), "C4": subset(b, 3)}.get(name, b)
    data = generate(b, device="cuda", seed=17)
    c = b.config
    expected = oracle_requests(data["q"], data["k"], data["v"], b.lengths, indptr=data["indptr"],
                               indices=data["pages"], pages=data["pages"], page_size=c.page_size)
    outs = []
    for mode in ((Mode.R1, Mode.D1) if name != "C2" else (Mode.R1, Mode.STATIC, Mode.D1, Mode.D4)):
        engine = DecodeEngine(c, device="cuda", dtype=b.dtype, force_mode=mode)
        update_plan(engine, b.lengths, b.splits)
        engine.prepare()
        out = engine.execute(data["q"], data["k"], data["v"], data["pages"], indptr=data["indptr"])
        torch.cuda.synchronize()
        assert engine.layers[0].status.item() == 0
        assert engine.kernel_kind() in KERNELS["tcgen05"]
        assert_rows_within_tolerance(out, expected, range(len(b.lengths)))
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("window_left", [0, 63, 500, 4096])
def test_sliding_window_csr(kernel, window_left):
    """SGLang / FlashInfer window_left: the query attends to the last min(L, window_left + 1)
    tokens; the window is the unchanged kernel on shifted CSR bases and windowed lengths."""
    from sglang_decode.window import window_bases, window_lengths
    lengths = [1, 65, 300, 0, 1000, 129]
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=16, kv_heads=2, head_dim=128,
                     page_size=1, workers=37)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=4000))
    full = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    wl = window_lengths(lengths, window_left)
    bases = window_bases(indptr, full, window_left)
    starts = indptr.cpu().tolist()
    want = np.zeros((len(lengths), c.query_heads, c.head_dim), dtype=np.float32)
    for r, (n, w) in enumerate(zip(lengths, wl)):
        if w:
            rows = idx[starts[r] + n - w:starts[r] + n].long()
            want[r] = A.request_attention(q[r].float().cpu().numpy(), k[rows].float().cpu().numpy(),
                                          v[rows].float().cpu().numpy())
    engine = DecodeEngine(c, force_mode=Mode.D4)
    out = _run(engine, (q, k, v, idx), wl, indptr=bases)
    assert engine.kernel_kind() in KERNELS[kernel]
    assert_within_tolerance(out, want, len(lengths))


def test_small_kernel_is_bitwise_equal_to_the_persistent_kernel_on_single_stage_tasks(monkeypatch):
    """C1's tasks are at most 64 tokens (one stage): the small-batch kernel runs the persistent
    kernel's fragment code, softmax and combine on them, so the outputs agree bit for bit."""
    b = baseline("C1", workers=torch.cuda.get_device_properties(0).multi_processor_count)
    data = generate(b, device="cuda", seed=17)
    outs = {}
    for kernel in ("mma", "small"):
        monkeypatch.setenv("SGLD_DECODE_KERNEL", kernel)
        engine = DecodeEngine(b.config, device="cuda", dtype=b.dtype)
        update_plan(engine, b.lengths, b.splits)
        engine.prepare()
        out = engine.execute(data["q"], data["k"], data["v"], data["pages"], indptr=data["indptr"])
        torch.cuda.synchronize()
        assert engine.layers[0].status.item() == 0
        assert engine.kernel_kind() in KERNELS[kernel]
        n = engine.plan.record_count.item()
        assert (engine.plan.end[:n] - engine.plan.begin[:n]).max().item() <= 64
        outs[kernel] = out.clone()
    assert torch.equal(outs["mma"], outs["small"])


def test_small_kernel_fused_merge_edges(monkeypatch):
    """The small-batch kernel merges the splits itself (the last split CTA of a request's KV
    head merges its rows).  Zero-length and inactive requests give zero rows, the arrival
    counters are left at zero so several layers run on one plan, invalid metadata turns every
    row NaN, and an empty batch writes zeros -- the stand-alone merge kernel's rules."""
    monkeypatch.setenv("SGLD_DECODE_KERNEL", "small")
    lengths = [0, 65, 300, 0, 1000, 1]
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=16, kv_heads=2, head_dim=128,
                     page_size=1, workers=37)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=2000))
    expected = oracle_csr(q, k, v, indptr, idx, lengths)
    engine = DecodeEngine(c, layers=3, force_mode=Mode.D1)
    update_plan(engine, lengths)
    engine.prepare()
    for layer in range(3):
        engine.layers[layer].output.fill_(float("nan"))
        engine.layers[layer].partial.fill_(float("nan"))
        engine.execute(q, k, v, idx, layer=layer, indptr=indptr)
    torch.cuda.synchronize()
    assert engine.kernel_kind() == "small"
    assert engine.plan.arrivals.eq(0).all(), "arrival counters not left at zero"
    for layer in range(3):
        out = engine.layers[layer].output
        assert engine.layers[layer].status.item() == 0
        assert_within_tolerance(out, expected, len(lengths))
        assert (out[len(lengths):].float() == 0).all(), "inactive rows must be zero"
        assert (out[0].float() == 0).all() and (out[3].float() == 0).all(), "zero-length rows must be zero"

    engine.plan.lengths[2] = c.max_context + 1                       # invalid metadata
    engine.prepare()
    out = engine.execute(q, k, v, idx, indptr=indptr)
    torch.cuda.synchronize()
    assert engine.plan.error.item() == 1
    assert torch.isnan(out.float()).all()

    update_plan(engine, [])                                          # empty batch
    engine.layers[0].output.fill_(float("nan"))
    engine.prepare()
    out = engine.execute(q, k, v, idx, indptr=indptr)
    torch.cuda.synchronize()
    assert (out.float() == 0).all()
    assert engine.plan.arrivals.eq(0).all()
