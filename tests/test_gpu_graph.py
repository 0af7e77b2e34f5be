"""CUDA-graph lifecycle on the GPU (port of the reference's tests/gpu/test_graph.py).

Paged graphs shrink and regrow 32 -> 7 -> 1 -> 32 under a D4 rule with every layer's
partial/LSE NaN-poisoned and its claim counter poisoned before each replay; a CSR
graph (the Qwen2-7B shape, group 7) replays a shrinking batch 128 -> 96 -> 64 -> 33 -> 1
with one token appended per request per step.
"""
import pytest
import torch

from sglang_decode.config import DecodeConfig, Mode
from sglang_decode.planning.policy import PolicyRule
from sglang_decode.runtime.engine import DecodeEngine, PlanKey
from sglang_decode.runtime.graph import DecodeGraph
from sglang_decode.workloads import make_inputs, split_hints
from tests.helpers import assert_within_tolerance, oracle_csr, oracle_paged

pytestmark = pytest.mark.gpu


def test_graph_shrink_regrow_switch_modes_and_reset_layers(cuda_device):
    c = DecodeConfig(batch_capacity=32, max_context=1024)
    # Explicit test-only rules exercise a device branch; not production calibration.
    rules = [PolicyRule(1, c.task_capacity, 101, 10000, int(Mode.D4))]
    engine = DecodeEngine(c, layers=2, rules=rules)
    fixtures = [tuple(t.cuda() for t in make_inputs(c, [1024] * 32, seed=40 + i, device="cpu"))
                for i in range(2)]
    key = PlanKey("shared-sequence-order", "test-splits", (32, 8, 128))
    graph = DecodeGraph(engine, [key] * 2, [(x[1], x[2]) for x in fixtures])
    pointers = [(x.counter.data_ptr(), x.partial.data_ptr(), x.output.data_ptr()) for x in engine.layers]
    for step, batch in enumerate([32, 7, 1, 32]):
        lengths = [1024 if i % 3 == 0 else 33 for i in range(batch)]
        splits = [1] * batch  # ensure nonuniform per-split work for mode switching
        graph.update([x[0][:batch] for x in fixtures], [x[3][:batch] for x in fixtures], lengths, splits)
        if step == 0:
            graph.capture()
        # Poison everything, not just padding: every valid result must be overwritten.
        for layer in engine.layers:
            layer.partial.fill_(float("nan"))
            layer.lse.fill_(float("nan"))
            layer.counter.fill_(100000)
        outputs = graph.replay()
        torch.cuda.synchronize()
        for layer, x in enumerate(fixtures):
            expected = oracle_paged(*x[:3], x[3], lengths, c.page_size)
            assert_within_tolerance(outputs[layer], expected, batch)
            assert engine.layers[layer].status.item() == 0
        assert pointers == [(x.counter.data_ptr(), x.partial.data_ptr(), x.output.data_ptr())
                            for x in engine.layers]
        assert engine.plan.mode.item() == (Mode.R1 if batch == 1 else Mode.D4)


def test_capacity_and_layer_compatibility_before_capture(cuda_device):
    c = DecodeConfig(batch_capacity=2, max_context=1024)
    engine = DecodeEngine(c, layers=2)
    x = tuple(t.cuda() for t in make_inputs(c, [17, 33], device="cpu"))
    first = PlanKey("a", "s", (32, 8, 128))
    second = PlanKey("b", "s", (32, 8, 128))
    with pytest.raises(ValueError):
        DecodeGraph(engine, [first, second], [(x[1], x[2])] * 2)
    graph = DecodeGraph(engine, [first] * 2, [(x[1], x[2])] * 2)
    with pytest.raises(ValueError):
        graph.update([], [], [1, 1, 1], [1, 1, 1])
    with pytest.raises(RuntimeError):
        graph.replay()


@pytest.mark.parametrize("mode", [-1, int(Mode.D4)])
def test_csr_graph_group7_shrinking_batch(mode, cuda_device):
    """Qwen2-7B shape (Hq=28, Hkv=4, G=7) under a CSR graph, batch 128->96->64->33->1."""
    layers, cap, steps = 3, 128, (128, 96, 64, 33, 1)
    c = DecodeConfig(batch_capacity=cap, max_splits=16, max_context=2048, query_heads=28, kv_heads=4,
                     head_dim=128, page_size=1, workers=148)
    gen = torch.Generator().manual_seed(11)
    base = torch.randint(256, 1024, (cap,), generator=gen).tolist()
    pool = sum(base) + len(steps) * cap
    kv = [(torch.randn((pool, 4, 128), generator=gen).to(torch.bfloat16).cuda(),
           torch.randn((pool, 4, 128), generator=gen).to(torch.bfloat16).cuda()) for _ in range(layers)]
    qs = [torch.randn((cap, 28, 128), generator=gen).to(torch.bfloat16).cuda() for _ in range(layers)]
    perm = [torch.randperm(pool, generator=gen).int() for _ in range(layers)]
    engine = DecodeEngine(c, layers=layers, force_mode=mode)
    key = PlanKey("seq", "hints", (28, 4, 128))
    graph = DecodeGraph(engine, [key] * layers, kv, csr=True, index_capacity=pool)
    # Request r owns slots base_offset[r] .. + current length (one appended per step).
    starts = [0]
    for n in base:
        starts.append(starts[-1] + n + len(steps))
    for step, batch in enumerate(steps):
        lengths = [base[r] + step + 1 for r in range(batch)]
        splits = split_hints(lengths, c.max_splits)
        indices = [torch.cat([perm[i][starts[r]:starts[r] + lengths[r]] for r in range(batch)]).cuda()
                   for i in range(layers)]
        graph.update([q[:batch] for q in qs], indices, lengths, splits)
        if step == 0:
            graph.capture()
        for layer in engine.layers:
            layer.partial.fill_(float("nan"))
            layer.counter.fill_(7)
        outputs = graph.replay()
        torch.cuda.synchronize()
        indptr = graph.indptr
        for i in range(layers):
            expected = oracle_csr(qs[i], kv[i][0], kv[i][1], indptr, graph.pages[i], lengths)
            assert_within_tolerance(outputs[i], expected, batch)
            assert engine.layers[i].status.item() == 0
