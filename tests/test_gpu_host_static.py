"""GPU: the host STATIC planner gives the GPU plan kernel's STATIC tables and outputs, and the
calibration measurement runs (one round set on a small workload)."""
import pytest
import torch

from sglang_decode.planning.calibrate import MODES, measure
from sglang_decode.planning.host_static import prepare_host_static
from sglang_decode.runtime.engine import DecodeEngine
from sglang_decode.workloads import baseline, generate, subset, update_plan

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["C1", "C2", "C4"])
def test_host_static_lists_and_outputs_equal_the_gpu_static_plan(name, cuda_device):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    b = baseline(name, workers=sms)
    if name == "C4":
        b = subset(b, 4)
    data = generate(b, device="cuda")
    args = (data["q"], data["k"], data["v"], data["pages"])
    gpu = DecodeEngine(b.config, device="cuda", dtype=b.dtype, force_mode=2)
    host = DecodeEngine(b.config, device="cuda", dtype=b.dtype, force_mode=-1)
    for e in (gpu, host):
        update_plan(e, b.lengths, b.splits)
    gpu.prepare()
    prepare_host_static(host, b.lengths, b.splits)
    torch.cuda.synchronize()
    tasks = int(gpu.plan.record_count.item()) * b.config.kv_heads
    assert int(host.plan.mode.item()) == 2
    assert torch.equal(gpu.plan.static_head, host.plan.static_head)
    assert torch.equal(gpu.plan.static_next[:tasks], host.plan.static_next[:tasks])
    out_gpu = gpu.execute(*args, indptr=data["indptr"]).clone()
    out_host = host.execute(*args, indptr=data["indptr"]).clone()
    torch.cuda.synchronize()
    assert gpu.layers[0].status.item() == 0 and host.layers[0].status.item() == 0
    assert torch.equal(out_gpu, out_host)


def test_calibration_measure_reports_every_variant(cuda_device):
    rows = measure("C1", rounds=5, iterations=3, warmup=1)
    assert len(rows) == 5 * len(MODES)
    assert {r["variant"] for r in rows} == set(MODES)
    assert all(r["status"] == "ok" and float(r["wall_us"]) > 0 for r in rows)
