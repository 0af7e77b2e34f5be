"""KV-cache write chained into the decode call, and Q with fewer rows than the capacity (GPU).

SGLang's decode step writes the new token's K/V into the pool (``set_kv_buffer``) and
then decodes; the reference adapter also copies Q into a capacity-sized buffer first
(reference ``integrations/sglang_backend.py:91-92,102-103``).  The engine does both in
its own call (a write kernel chained before the decode; Q read in place).  The call must
give exactly what "write the rows, then decode" gives, in every dispatch mode: the same
output bits and the same pool, for any slots.
"""
import pytest
import torch

from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import make_csr_inputs, make_inputs, update_plan
from tests.helpers import assert_within_tolerance, oracle_csr, oracle_paged

pytestmark = pytest.mark.gpu

LENGTHS = [1, 65, 300, 0, 1000, 129, 700]   # the empty request's row is written too
CASES = {  # name: (kv_heads, group, head_dim, page_size)
    "csr_g8": (2, 8, 128, 1),
    "csr_g7": (4, 7, 128, 1),
    "paged16_d64_g4": (2, 4, 64, 16),
    "paged32_g8": (2, 8, 128, 32),
    "paged64_d256_g16": (1, 16, 256, 64),   # the tensor-map (TMA) kernel
}


def _setup(name, dtype):
    hkv, group, d, ps = CASES[name]
    c = DecodeConfig(batch_capacity=8, max_splits=8, max_context=1024, query_heads=hkv * group,
                     kv_heads=hkv, head_dim=d, page_size=ps, workers=37)
    rows = len(LENGTHS)
    if ps == 1:
        q, k, v, idx, indptr = make_csr_inputs(c, LENGTHS, device="cpu", dtype=dtype, pool=4000)
        used = set(idx.tolist())
        spare = next(s for s in range(4000) if s not in used)
        ends = torch.tensor(LENGTHS).cumsum(0)
        loc = [int(idx[int(ends[r]) - 1]) if n else spare for r, n in enumerate(LENGTHS)]
        pages = idx
    else:
        q, k, v, pages = make_inputs(c, LENGTHS, device="cpu", dtype=dtype)
        indptr = None
        # request 0 (one token) leaves rows 1.. of its page unread: the empty request's slot
        spare = int(pages[0, 0]) * ps + 1
        loc = [int(pages[r, (n - 1) // ps]) * ps + (n - 1) % ps if n else spare for r, n in enumerate(LENGTHS)]
    g = torch.Generator().manual_seed(5)
    k_new = torch.randn(rows, hkv, d, generator=g, dtype=dtype)
    v_new = torch.randn(rows, hkv, d, generator=g, dtype=dtype)
    cuda = lambda t: None if t is None else t.cuda()
    return c, cuda(q[:rows]), cuda(k), cuda(v), cuda(pages), cuda(indptr), cuda(k_new), cuda(v_new), loc


def _written(c, pool, loc, rows):
    """The pool after set_kv_buffer: rows stored at their token slots."""
    out = pool.clone()
    out.view(-1, c.kv_heads, c.head_dim)[torch.tensor(loc, device="cuda")] = rows
    return out


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("loc_dtype", [torch.int64, torch.int32], ids=["i64", "i32"])
def test_fused_kv_write_equals_write_then_decode(name, dtype, loc_dtype, cuda_device):
    c, q, k, v, pages, indptr, k_new, v_new, loc = _setup(name, dtype)
    k_ref, v_ref = _written(c, k, loc, k_new), _written(c, v, loc, v_new)
    new_loc = torch.tensor(loc, dtype=loc_dtype, device="cuda")
    outs = []
    for mode in Mode:
        engine = DecodeEngine(c, dtype=dtype, force_mode=mode)
        update_plan(engine, LENGTHS)
        engine.prepare()
        want = engine.execute(q, k_ref, v_ref, pages, indptr=indptr).clone()
        k_got, v_got = k.clone(), v.clone()          # stale rows at the new slots
        engine.prepare()
        got = engine.execute(q, k_got, v_got, pages, indptr=indptr, k_new=k_new, v_new=v_new, new_loc=new_loc)
        torch.cuda.synchronize()
        assert engine.layers[0].status.item() == 0
        assert torch.equal(got, want), f"{mode}: fused write differs from write-then-decode"
        assert torch.equal(k_got, k_ref) and torch.equal(v_got, v_ref), f"{mode}: pool differs"
        outs.append(got.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every dispatch mode gives identical outputs"
    if indptr is None:
        expected = oracle_paged(q, k_ref, v_ref, pages, LENGTHS, c.page_size)
    else:
        expected = oracle_csr(q, k_ref, v_ref, indptr, pages, LENGTHS)
    assert_within_tolerance(outs[0], expected, len(LENGTHS))


def test_write_to_slots_that_other_requests_read(cuda_device):
    """Slots anywhere in the pool, including positions in the middle of other requests'
    contexts: every reader sees the new row (write first, then decode)."""
    c, q, k, v, pages, indptr, k_new, v_new, _ = _setup("csr_g8", torch.bfloat16)
    g = torch.Generator().manual_seed(9)
    picks = torch.randperm(pages.numel(), generator=g)[:q.shape[0]]
    loc = [int(pages[int(i)]) for i in picks]          # slots that some request reads
    k_ref, v_ref = _written(c, k, loc, k_new), _written(c, v, loc, v_new)
    for mode in (Mode.R1, Mode.D4):
        engine = DecodeEngine(c, dtype=torch.bfloat16, force_mode=mode)
        update_plan(engine, LENGTHS)
        engine.prepare()
        want = engine.execute(q, k_ref, v_ref, pages, indptr=indptr).clone()
        k_got, v_got = k.clone(), v.clone()
        engine.prepare()
        got = engine.execute(q, k_got, v_got, pages, indptr=indptr, k_new=k_new, v_new=v_new,
                             new_loc=torch.tensor(loc, device="cuda"))
        torch.cuda.synchronize()
        assert engine.layers[0].status.item() == 0
        assert torch.equal(got, want) and torch.equal(k_got, k_ref) and torch.equal(v_got, v_ref)


FP8 = getattr(torch, "float8_e4m3fn", None)


@pytest.mark.skipif(FP8 is None, reason="torch without float8_e4m3fn")
def test_write_into_an_fp8_pool(cuda_device):
    """An e4m3 pool stores e4m3(x / scale) (fp32 quotient, one rounding); the decode then
    reads the quantised rows.  Values stay inside the e4m3 range here."""
    c, q, k, v, pages, indptr, k_new, v_new, loc = _setup("csr_g8", torch.bfloat16)
    ks, vs = 0.5, 2.0
    k8, v8 = (k / ks).to(FP8), (v / vs).to(FP8)
    k_ref, v_ref = k8.clone(), v8.clone()
    slots = torch.tensor(loc, device="cuda")
    k_ref.view(-1, c.kv_heads, c.head_dim)[slots] = (k_new.float() / ks).to(FP8)
    v_ref.view(-1, c.kv_heads, c.head_dim)[slots] = (v_new.float() / vs).to(FP8)
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, LENGTHS)
    engine.prepare()
    want = engine.execute(q, k_ref, v_ref, pages, indptr=indptr, k_scale=ks, v_scale=vs).clone()
    k_got, v_got = k8.clone(), v8.clone()
    engine.prepare()
    got = engine.execute(q, k_got, v_got, pages, indptr=indptr, k_scale=ks, v_scale=vs,
                         k_new=k_new, v_new=v_new, new_loc=slots)
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() == 0
    assert torch.equal(k_got.view(torch.uint8), k_ref.view(torch.uint8))
    assert torch.equal(v_got.view(torch.uint8), v_ref.view(torch.uint8))
    assert torch.equal(got, want)


def test_strided_q_and_new_rows_from_one_qkv_tensor(cuda_device):
    """Q, K and V as views of one projection output [rows, (Hq + 2 Hkv) * D], as SGLang
    hands them to the backend: nothing is copied and the result is unchanged."""
    c, q, k, v, pages, indptr, k_new, v_new, loc = _setup("csr_g7", torch.bfloat16)
    rows, hq, hkv, d = q.shape[0], c.query_heads, c.kv_heads, c.head_dim
    qkv = torch.cat([q.reshape(rows, -1), k_new.reshape(rows, -1), v_new.reshape(rows, -1)], dim=1)
    q_view = qkv[:, :hq * d].view(rows, hq, d)
    k_view = qkv[:, hq * d:(hq + hkv) * d].view(rows, hkv, d)
    v_view = qkv[:, (hq + hkv) * d:].view(rows, hkv, d)
    assert not q_view.is_contiguous()
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, LENGTHS)
    engine.prepare()
    want = engine.execute(q, _written(c, k, loc, k_new), _written(c, v, loc, v_new), pages, indptr=indptr).clone()
    engine.prepare()
    k_got, v_got = k.clone(), v.clone()
    got = engine.execute(q_view, k_got, v_got, pages, indptr=indptr, k_new=k_view, v_new=v_view,
                         new_loc=torch.tensor(loc, device="cuda"))
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() == 0
    assert torch.equal(got, want)
    assert torch.equal(k_got, _written(c, k, loc, k_new))


def test_q_with_fewer_rows_than_active_requests_is_flagged(cuda_device):
    """A plan whose active count exceeds Q's rows reads a zero query for the extra
    requests (never past Q) and sets status bit 64."""
    c, q, k, v, pages, indptr, *_ = _setup("csr_g8", torch.bfloat16)
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, LENGTHS)                     # 7 active requests
    engine.prepare()
    engine.execute(q[:5], k, v, pages, indptr=indptr)
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() & 64


def test_out_of_range_slot_is_skipped_and_flagged(cuda_device):
    """A slot outside the pool is not written (status bit 128); the other rows are, and
    nothing is read or written out of bounds."""
    c, q, k, v, pages, indptr, k_new, v_new, loc = _setup("csr_g8", torch.bfloat16)
    bad = list(loc)
    bad[2] = k.shape[0]                               # one past the last token slot
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, LENGTHS)
    engine.prepare()
    k_got, v_got = k.clone(), v.clone()
    engine.execute(q, k_got, v_got, pages, indptr=indptr, k_new=k_new, v_new=v_new,
                   new_loc=torch.tensor(bad, device="cuda"))
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() & 128
    good = [r for r in range(len(loc)) if r != 2]
    assert torch.equal(k_got, _written(c, k, [loc[r] for r in good], k_new[good]))
    assert torch.equal(v_got, _written(c, v, [loc[r] for r in good], v_new[good]))


def test_fused_write_host_checks(cuda_device):
    c, q, k, v, pages, indptr, k_new, v_new, loc = _setup("csr_g8", torch.bfloat16)
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, LENGTHS)
    engine.prepare()
    new_loc = torch.tensor(loc, device="cuda")
    with pytest.raises(ValueError):                  # rows without slots
        engine.execute(q, k, v, pages, indptr=indptr, k_new=k_new, v_new=v_new)
    with pytest.raises(ValueError):                  # one new row short
        engine.execute(q, k, v, pages, indptr=indptr, k_new=k_new[:-1], v_new=v_new, new_loc=new_loc)
    with pytest.raises(ValueError):                  # non-contiguous slots
        engine.execute(q, k, v, pages, indptr=indptr, k_new=k_new, v_new=v_new,
                       new_loc=torch.stack([new_loc, new_loc], 1)[:, 0])
    with pytest.raises(ValueError):                  # more Q rows than the capacity
        engine.execute(torch.cat([q, q]), k, v, pages, indptr=indptr)
