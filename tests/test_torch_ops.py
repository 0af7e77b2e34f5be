"""The torch operator library over the C ABI (no GPU needed): it loads, registers
torch.ops.sglang_decode.{plan_build, decode, merge} with their mutation annotations, and its
Meta kernels run on meta tensors (what tracing tools call), touching no memory."""
import torch

from sglang_decode import _native
from sglang_decode.config import DecodeConfig


def test_ops_library_registers_schemas():
    ops = _native.ops()
    schemas = {name: str(getattr(ops, name).default._schema) for name in ("plan_build", "decode", "merge")}
    assert "Tensor(a!)[] plan" in schemas["plan_build"]
    for arg in ("Tensor(c!) out", "Tensor(d!) partial", "Tensor(e!) lse", "Tensor(f!) counter", "Tensor(g!) status"):
        assert arg in schemas["decode"]
    assert "Tensor(a!) out" in schemas["merge"]


def test_ops_meta_kernels_accept_the_engine_argument_layout():
    ops = _native.ops()
    c = DecodeConfig(batch_capacity=4, max_splits=2, max_context=256, query_heads=8, kv_heads=2, head_dim=128,
                     page_size=1, workers=4)
    m = dict(device="meta")
    plan = [torch.empty(8, dtype=torch.int32, **m) for _ in _native.PLAN_FIELDS]
    geometry = [c.batch_capacity, c.max_splits, c.max_context, c.kv_heads, c.workers]
    ops.plan_build(plan, geometry, -1, None, 0, torch.empty(2, dtype=torch.int32, **m))
    q = torch.empty(4, 8, 128, dtype=torch.bfloat16, **m)
    kv = torch.empty(64, 2, 128, dtype=torch.bfloat16, **m)
    out = torch.empty_like(q)
    partial = torch.empty(4, 8, 2, 128, **m)
    lse = torch.empty(4, 8, 2, **m)
    ops.decode(q, kv, kv, torch.empty(64, dtype=torch.int32, **m), torch.empty(5, dtype=torch.int32, **m), out,
               partial, lse, torch.empty(2, dtype=torch.int32, **m), torch.empty(1, dtype=torch.int32, **m), plan,
               geometry, 8, 2, 128, 1, 128 ** -0.5, 0.0, 1.0, 1.0, None, None, None)
    ops.merge(partial, lse, plan[3], plan[17], out)
