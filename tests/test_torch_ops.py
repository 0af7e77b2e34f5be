"""The torch operator library over the C ABI (no GPU needed): it loads, registers
torch.ops.sglang_decode.{plan_build, decode, merge} with their mutation annotations, and its
Meta kernels run on meta tensors (what tracing tools call), touching no memory."""
import torch

from sglang_decode import _native
from sglang_decode.config import DecodeConfig


def test_ops_library_registers_schemas():
    ops = _native.ops()
    schemas = {name: str(getattr(ops, name).default._schema) for name in ("plan_build", "decode", "merge")}
    assert "Tensor(a!) plan" in schemas["plan_build"]
    for arg in ("Tensor(c!) out", "Tensor(d!) partial", "Tensor(e!) lse", "Tensor(f!) counter", "Tensor(g!) status"):
        assert arg in schemas["decode"]
    assert "Tensor(a!) out" in schemas["merge"]


def test_ops_meta_kernels_accept_the_engine_argument_layout():
    ops = _native.ops()
    c = DecodeConfig(batch_capacity=4, max_splits=2, max_context=256, query_heads=8, kv_heads=2, head_dim=128,
                     page_size=1, workers=4)
    m = dict(device="meta")
    words = sum(_native.plan_field_words(c.batch_capacity, c.max_splits, c.kv_heads, c.workers))
    plan = torch.empty(words, dtype=torch.int32, **m)
    geometry = [c.batch_capacity, c.max_splits, c.max_context, c.kv_heads, c.workers]
    ops.plan_build(plan, geometry, -1, None, 0, torch.empty(2, dtype=torch.int32, **m))
    q = torch.empty(4, 8, 128, dtype=torch.bfloat16, **m)
    kv = torch.empty(64, 2, 128, dtype=torch.bfloat16, **m)
    out = torch.empty_like(q)
    partial = torch.empty(4, 8, 2, 128, **m)
    lse = torch.empty(4, 8, 2, **m)
    ops.decode(q, kv, kv, torch.empty(64, dtype=torch.int32, **m), torch.empty(5, dtype=torch.int32, **m), out,
               partial, lse, torch.empty(2, dtype=torch.int32, **m), torch.empty(1, dtype=torch.int32, **m), plan,
               geometry, 1, 128 ** -0.5, 0.0, 1.0, 1.0, None, None, None)
    ops.merge(partial, lse, plan[:4], plan[:1], out)


def test_plan_storage_layout_matches_the_c_abi():
    """PlanBuffers views one int32 storage; the C library's sgld_plan_buffers_in_storage must
    place every buffer at the same offset (pure pointer arithmetic: nothing is dereferenced)."""
    import ctypes
    lib = _native.load()
    for geometry in ((8, 16, 1024, 8, 148), (3, 1, 64, 1, 5), (256, 16, 8192, 8, 148)):
        b, smax, _, groups, workers = geometry
        g = _native.PlanGeometry(*geometry)
        sizes = _native.plan_field_words(b, smax, groups, workers)
        assert lib.sgld_plan_storage_words(ctypes.byref(g)) == sum(sizes)
        base = 1 << 20
        out = _native.PlanBuffersC()
        assert lib.sgld_plan_buffers_in_storage(base, ctypes.byref(g), ctypes.byref(out)) == 0
        offset = 0
        for name, n in zip(_native.PLAN_FIELDS, sizes):
            assert getattr(out, name) == base + 4 * offset, name
            offset += n
    assert lib.sgld_plan_storage_words(ctypes.byref(_native.PlanGeometry(0, 1, 1, 1, 1))) == 0
    assert lib.sgld_plan_buffers_in_storage(None, ctypes.byref(_native.PlanGeometry(1, 1, 1, 1, 1)),
                                            ctypes.byref(_native.PlanBuffersC())) == 1
