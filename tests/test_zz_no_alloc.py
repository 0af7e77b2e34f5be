"""GPU test of sgld_decode_persistent_noalloc, the allocation-free decode entry point.

Callers that cannot allocate device memory at the call site (plugin interfaces that pass
only inputs and outputs, servers that gave all device memory to their KV-cache pool) use
this entry point: the decode's scratch lives in a fixed 16 MiB device array inside the
library.  This file is collected last so that a run stopping at its first failure has run
every other test; it also passes on its own in a fresh process.

Both calls below go through the C ABI and must agree with sgld_decode_persistent (which
uses caller-owned scratch) within the suite's tolerance: max-abs 2e-2, mean-abs 2e-3.
The second call checks that the state the first call leaves in the shared array does
not leak into the next result.
"""
import ctypes

import numpy as np
import pytest
import torch

from sglang_decode import _native
from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import make_csr_inputs, update_plan

pytestmark = pytest.mark.gpu


def _entry_point():
    lib = _native.load()
    fn = lib.sgld_decode_persistent_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_native.DecodeArgs), ctypes.POINTER(_native.PlanBuffersC),
                   ctypes.POINTER(_native.PlanGeometry), ctypes.c_void_p]
    return lib, fn


def test_noalloc_matches_caller_scratch_entry_point_on_two_calls(cuda_device):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    c = DecodeConfig(batch_capacity=8, max_splits=16, max_context=1024, query_heads=32, kv_heads=8,
                     head_dim=128, page_size=1, workers=sms)
    lengths = [64, 1024, 700, 333, 129, 900, 1000, 65]
    q, k, v, idx, indptr = (t.cuda() for t in make_csr_inputs(c, lengths, device="cpu", pool=16384))
    engine = DecodeEngine(c, dtype=torch.bfloat16, force_mode=Mode.D4)
    update_plan(engine, lengths)
    engine.prepare()
    expected = engine.execute(q, k, v, idx, indptr=indptr).clone()
    torch.cuda.synchronize()
    assert engine.layers[0].status.item() == 0

    lib, fn = _entry_point()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(expected, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        args = _native.DecodeArgs()                                 # same tensors and geometry
        ctypes.memmove(ctypes.byref(args), ctypes.byref(engine.layers[0].c_args), ctypes.sizeof(args))
        args.out = out.data_ptr()
        args.counter = args.partial = args.lse = None               # scratch comes from the library
        args.status = status.data_ptr()
        rc = fn(ctypes.byref(args), ctypes.byref(engine.plan.c_buffers),
                ctypes.byref(engine.plan.c_geometry), stream)
        assert rc == 0, lib.sgld_last_error()
        torch.cuda.synchronize()
        assert status.item() == 0, f"call {call}: bounded in-kernel wait expired"
        got = out.float().cpu().numpy()
        want = expected.float().cpu().numpy()
        assert np.isfinite(got).all()
        diff = np.abs(got - want)
        assert diff.max() <= 2e-2 and diff.mean() <= 2e-3, (call, diff.max(), diff.mean())


def test_noalloc_rejects_geometries_beyond_its_scratch(cuda_device):
    lib, fn = _entry_point()
    c = DecodeConfig(batch_capacity=64, max_splits=16, max_context=32768, query_heads=32, kv_heads=8,
                     head_dim=256, page_size=16, workers=148)
    engine = DecodeEngine(c, dtype=torch.bfloat16)
    args = _native.DecodeArgs()
    args.query_heads, args.kv_heads, args.head_dim = c.query_heads, c.kv_heads, c.head_dim
    rc = fn(ctypes.byref(args), ctypes.byref(engine.plan.c_buffers), ctypes.byref(engine.plan.c_geometry),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"16 MiB" in lib.sgld_last_error()
