"""Decode outputs at the benchmark configurations' real shapes vs the FP32 oracle.

The inputs are the bench's own (``sglang_decode.workloads.baseline(name)`` and
``generate``, seed 17): the reference's fixture recipe at the C1..C5 shapes.  Like the
reference's ``tests/gpu/test_decode.py:12-39`` every run compares the output with the FP32
oracle and the device task table with the CPU specification, here at full size:

* C1 in full, under AUTO and every mode;
* C2 in full under R1, STATIC, D1 and D4 (outputs and bit-exact tables);
* C3 (Hq=64, Hkv=8, fp16, CSR) on a 16-request prefix, on one GPU and as the eight
  one-KV-head shards of an 8-way tensor-parallel run, each shard bit-identical to the
  matching heads of the unsharded output;
* C4 on its first three requests (32K-131K tokens, page size 64, 16 splits: 16-way merges);
* C5 as a four-layer CSR CUDA graph at the real lengths (L0 ~ U[256, 4096], group 7) over
  the whole replay 128 -> 96 -> 64 -> 33 -> 1 with one appended token per request per step.

Tolerance (the bar every parity test uses): max-abs 2e-2 and mean-abs 2e-3 against FP32.
"""
import pytest
import torch

from oracle import planning as P
from sglang_decode.config import Mode
from sglang_decode.runtime.engine import DecodeEngine, PlanKey
from sglang_decode.runtime.graph import DecodeGraph
from sglang_decode.sharding import head_shard, shard_config
from sglang_decode.workloads import baseline, generate, graph_layer, graph_step, split_hints, subset, update_plan
from tests.helpers import (assert_rows_within_tolerance, capture_tables, geometry_of, oracle_requests,
                           oracle_tables_in_golden_format, poison_plan)

pytestmark = pytest.mark.gpu


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def _run(b, cfg, data, mode):
    """Plan + decode + merge of one layer; returns (engine, output) after checking the
    status word, the claim counters and the device tables against the CPU spec."""
    engine = DecodeEngine(cfg, device="cuda", dtype=b.dtype, force_mode=mode)
    update_plan(engine, b.lengths, b.splits)
    poison_plan(engine.plan)
    layer = engine.layers[0]
    layer.partial.fill_(float("nan"))
    layer.lse.fill_(float("nan"))
    engine.prepare()
    out = engine.execute(data["q"], data["k"], data["v"], data["pages"], indptr=data["indptr"])
    torch.cuda.synchronize()
    assert layer.status.item() == 0, "bounded in-kernel wait expired"
    assert engine.counters.eq(0).all(), "claim words not left at zero"
    n = len(b.lengths)
    lb = b.lengths + [0] * (cfg.batch_capacity - n)
    sb = b.splits + [1] * (cfg.batch_capacity - n)
    g = geometry_of(cfg)
    assert capture_tables(engine.plan) == oracle_tables_in_golden_format(
        P.device_tables(lb, sb, n, g, int(mode)), g), "device task table differs from the CPU spec"
    return engine, out


def _oracle(b, data):
    c = b.config
    return oracle_requests(data["q"], data["k"], data["v"], b.lengths, indptr=data["indptr"],
                           indices=data["pages"], pages=data["pages"], page_size=c.page_size)


def _check(out, expected, b):
    rows = range(len(b.lengths))
    assert_rows_within_tolerance(out, expected, rows)
    assert (out[len(b.lengths):].float() == 0).all(), "rows past the batch must be zero"


def test_c1_full_every_mode(cuda_device):
    b = baseline("C1", workers=_sms())
    data = generate(b, device="cuda", seed=17)
    expected = _oracle(b, data)
    outs = []
    for mode in (-1, *[int(m) for m in Mode]):
        _, out = _run(b, b.config, data, mode)
        _check(out, expected, b)
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every mode gives the same bits"


def test_c2_full_r1_static_d1_d4(cuda_device):
    b = baseline("C2", workers=_sms())
    data = generate(b, device="cuda", seed=17)
    expected = _oracle(b, data)
    outs = []
    for mode in (Mode.R1, Mode.STATIC, Mode.D1, Mode.D4):
        engine, out = _run(b, b.config, data, int(mode))
        assert engine.plan.mode.item() == int(mode)
        _check(out, expected, b)
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:]), "every mode gives the same bits"


def test_c3_prefix_one_gpu_and_eight_head_shards(cuda_device):
    b = subset(baseline("C3", workers=_sms()), 16)
    c = b.config
    data = generate(b, device="cuda", seed=17)
    expected = _oracle(b, data)
    _, full = _run(b, c, data, -1)
    _check(full, expected, b)
    full = full.clone()
    _, d1 = _run(b, c, data, int(Mode.D1))
    assert torch.equal(full, d1)
    del data
    world = 8
    for rank in range(world):
        shard = head_shard(c, rank, world)
        cfg = shard_config(c, shard)
        part = generate(b, device="cuda", seed=17, kv_heads=shard.kv_heads, head_offset=shard.kv_offset)
        _, out = _run(b, cfg, part, -1)
        heads = slice(shard.q_offset, shard.q_offset + shard.query_heads)
        assert torch.equal(out, full[:, heads]), f"shard {rank} differs from the unsharded heads"
        assert_rows_within_tolerance(out, expected[:, heads], range(len(b.lengths)))


def test_c4_long_context_three_requests(cuda_device):
    b = subset(baseline("C4", workers=_sms()), 3)
    assert min(b.lengths) >= 32768 and max(b.splits) == 16
    data = generate(b, device="cuda", seed=17)
    expected = _oracle(b, data)
    outs = []
    for mode in (Mode.R1, Mode.STATIC, Mode.D4):
        _, out = _run(b, b.config, data, int(mode))
        _check(out, expected, b)
        outs.append(out.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("mode", [-1, int(Mode.D4)])
def test_c5_four_layer_graph_full_replay(mode, cuda_device):
    full = baseline("C5", workers=_sms())
    layers = 4
    b = full
    c = b.config
    data = [graph_layer(b, i, device="cuda") for i in range(layers)]
    engine = DecodeEngine(c, device="cuda", dtype=b.dtype, layers=layers, force_mode=mode)
    key = PlanKey("csr", "split_hints16", (c.query_heads, c.kv_heads))
    graph = DecodeGraph(engine, [key] * layers, [(x["k"], x["v"]) for x in data], csr=True,
                        index_capacity=b.pool_tokens)
    for step, batch in enumerate(b.replay_batches):
        lengths, pos = graph_step(b, step, batch)
        pos = pos.cuda()
        graph.update([x["q"][:batch] for x in data], [x["perm"][pos] for x in data], lengths,
                     split_hints(lengths, c.max_splits))
        if step == 0:
            graph.capture()
        for layer in engine.layers:
            layer.partial.fill_(float("nan"))
            layer.lse.fill_(float("nan"))
        outputs = graph.replay()
        torch.cuda.synchronize()
        for i in range(layers):
            assert engine.layers[i].status.item() == 0
            expected = oracle_requests(data[i]["q"][:batch], data[i]["k"], data[i]["v"], lengths,
                                       indptr=graph.indptr, indices=graph.pages[i])
            assert_rows_within_tolerance(outputs[i], expected, range(batch))
