"""GPU test of sgld_decode_persistent_noalloc, the allocation-free decode entry point.

Callers that cannot allocate device memory at the call site (plugin interfaces that pass
only inputs and outputs, servers that gave all device memory to their KV-cache pool) use
this entry point: the decode's scratch lives in a fixed 16 MiB device array inside the
library.  This file is collected last so that a run stopping at its first failure has run
every other test; it also passes on its own in a fresh process.

Every call goes through the C ABI and must agree with sgld_decode_persistent (which uses
caller-owned scratch) and with the FP32 oracle, within the suite's tolerance: max-abs
2e-2, mean-abs 2e-3.  The two calls in a row use different batches, lengths and split
counts, so state the first call leaves in the shared array cannot pass for the second
call's result.
"""
import ctypes

import numpy as np
import pytest
import torch

from sglang_decode import _native
from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import make_csr_inputs, update_plan
from tests.helpers import assert_within_tolerance, oracle_csr

pytestmark = pytest.mark.gpu

TOL = dict(max_abs=2e-2, mean_abs=2e-3)


def _entry_point():
    lib = _native.load()
    return lib, lib.sgld_decode_persistent_noalloc


def _config():
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return DecodeConfig(batch_capacity=8, max_splits=16, max_context=1024, query_heads=32, kv_heads=8,
                        head_dim=128, page_size=1, workers=sms)


def _noalloc_call(fn, engine, out, status, **override):
    """Call the entry point with the engine's last sgld_decode_persistent arguments, the
    scratch pointers cleared (the library supplies them) and the given fields replaced."""
    args = engine.c_args(0)
    args.out = out.data_ptr()
    args.counter = args.partial = args.lse = None
    args.status = status.data_ptr() if status is not None else None
    for name, value in override.items():
        setattr(args, name, value)
    return fn(ctypes.byref(args), ctypes.byref(engine.plan.c_buffers), ctypes.byref(engine.plan.c_geometry),
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_caller_scratch_and_oracle_on_two_different_calls(cuda_device):
    c = _config()
    lib, fn = _entry_point()
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, [1024] * 8, device="cpu", pool=16384))
    # Call 1: all eight requests, up to 16 splits each.  Call 2: five requests with other
    # lengths and few splits, so most slots call 1 wrote are stale for call 2.
    cases = [([64, 1024, 700, 333, 129, 900, 1000, 65], None),
             ([17, 200, 511, 1, 96], [1, 2, 3, 1, 1])]
    for call, (lengths, splits) in enumerate(cases):
        n = len(lengths)
        csr_ptr = torch.tensor([0] + np.cumsum(lengths).tolist() + [sum(lengths)] * (c.batch_capacity - n),
                               dtype=torch.int32, device="cuda")
        rows = idx[:sum(lengths)].contiguous()
        engine = DecodeEngine(c, dtype=torch.bfloat16, force_mode=Mode.D4)
        update_plan(engine, lengths, splits)
        engine.prepare()
        expected = engine.execute(q, k, v, rows, indptr=csr_ptr).clone()
        torch.cuda.synchronize()
        assert engine.layers[0].status.item() == 0
        out = torch.full_like(expected, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = _noalloc_call(fn, engine, out, status)
        assert rc == 0, lib.sgld_last_error()
        torch.cuda.synchronize()
        assert status.item() == 0, f"call {call}: bounded in-kernel wait expired"
        assert_within_tolerance(out, expected.float().cpu().numpy(), n, **TOL)
        assert_within_tolerance(out, oracle_csr(q, k, v, csr_ptr, rows, lengths), n, **TOL)
        assert (out[n:].float() == 0).all(), f"call {call}: rows without a request must be zero"


def test_noalloc_fused_kv_write_matches_caller_scratch(cuda_device):
    c = _config()
    lib, fn = _entry_point()
    lengths = [300, 17, 1000, 64]
    n = len(lengths)
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=4096))
    gen = torch.Generator(device="cpu").manual_seed(5)
    k_new = torch.randn(n, c.kv_heads, c.head_dim, generator=gen).to(torch.bfloat16).cuda()
    v_new = torch.randn(n, c.kv_heads, c.head_dim, generator=gen).to(torch.bfloat16).cuda()
    new_loc = idx[indptr[1:n + 1].long() - 1].long()          # each request's newest token slot
    engine = DecodeEngine(c, dtype=torch.bfloat16, force_mode=Mode.R1)
    update_plan(engine, lengths)
    engine.prepare()
    expected = engine.execute(q[:n], k, v, idx, indptr=indptr, k_new=k_new, v_new=v_new,
                              new_loc=new_loc).clone()
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() == 0
    out = torch.full_like(expected, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _noalloc_call(fn, engine, out, status)            # rewrites the same rows, then decodes
    assert rc == 0, lib.sgld_last_error()
    torch.cuda.synchronize()
    assert status.item() == 0
    assert_within_tolerance(out, expected.float().cpu().numpy(), n, **TOL)
    assert_within_tolerance(out, oracle_csr(q[:n], k, v, indptr, idx, lengths), n, **TOL)


def test_noalloc_rejects_null_status_and_oversized_geometry(cuda_device):
    lib, fn = _entry_point()
    c = _config()
    lengths = [10, 20]
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=64))
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    update_plan(engine, lengths)
    engine.prepare()
    engine.execute(q, k, v, idx, indptr=indptr)
    torch.cuda.synchronize()
    out = torch.zeros_like(engine.layers[0].output)
    assert _noalloc_call(fn, engine, out, None) == 1
    assert b"status is NULL" in lib.sgld_last_error()
    assert _noalloc_call(fn, engine, out, torch.zeros(1, dtype=torch.int32, device="cuda"), head_dim=96) == 2

    big = DecodeConfig(batch_capacity=64, max_splits=16, max_context=32768, query_heads=32, kv_heads=8,
                       head_dim=256, page_size=16, workers=148)
    engine = DecodeEngine(big, dtype=torch.bfloat16)
    args = _native.DecodeArgs()
    args.query_heads, args.kv_heads, args.head_dim = big.query_heads, big.kv_heads, big.head_dim
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    args.status = status.data_ptr()
    rc = fn(ctypes.byref(args), ctypes.byref(engine.plan.c_buffers), ctypes.byref(engine.plan.c_geometry),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"16 MiB" in lib.sgld_last_error()
