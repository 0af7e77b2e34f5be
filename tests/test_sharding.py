"""KV-head sharding of the decode path on CPU: host logic and a world-size-2 gloo run.

The N>1 path has no collective on the attention itself; these tests check that each rank's
shard (heads, plan geometry, seeded inputs) is the matching slice of the unsharded problem,
that the rank outputs reassemble to the unsharded FP32 oracle output, and that the timing
reduction takes the max over ranks (as bench.py does).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as A
from oracle import planning as P
from sglang_decode.config import DecodeConfig
from sglang_decode.sharding import assemble, head_shard, shard_config, shard_kv, shard_q
from sglang_decode.workloads import Baseline, generate, split_hints


def _small_c3():
    lengths = [130, 1, 257, 64, 511, 0, 33, 200]
    cfg = DecodeConfig(batch_capacity=8, max_splits=16, max_context=512, query_heads=16, kv_heads=4,
                       head_dim=64, page_size=1, workers=9)
    return Baseline("C3small", cfg, torch.float16, True, lengths, pool_tokens=sum(lengths) + 50)


def test_head_shard_ranges_and_validation():
    c = DecodeConfig(query_heads=64, kv_heads=8)
    shards = [head_shard(c, r, 4) for r in range(4)]
    assert [(s.kv_offset, s.kv_heads, s.q_offset, s.query_heads) for s in shards] == [
        (0, 2, 0, 16), (2, 2, 16, 16), (4, 2, 32, 16), (6, 2, 48, 16)]
    assert shard_config(c, shards[1]).kv_heads == 2 and shard_config(c, shards[1]).group_size == 8
    with pytest.raises(ValueError):
        head_shard(c, 0, 3)
    with pytest.raises(ValueError):
        head_shard(c, 4, 4)


def test_generated_shards_are_slices_of_the_unsharded_inputs():
    b = _small_c3()
    full = generate(b, device="cpu")
    for world in (2, 4):
        for rank in range(world):
            s = head_shard(b.config, rank, world)
            part = generate(b, device="cpu", kv_heads=s.kv_heads, head_offset=s.kv_offset)
            assert torch.equal(part["k"], shard_kv(full["k"], s))
            assert torch.equal(part["v"], shard_kv(full["v"], s))
            assert torch.equal(part["q"], shard_q(full["q"], s))
            assert torch.equal(part["pages"], full["pages"]) and torch.equal(part["indptr"], full["indptr"])


def test_plan_tables_per_shard_only_change_the_group_count():
    b = _small_c3()
    c = b.config
    for world in (1, 2, 4):
        g = P.Geometry(c.batch_capacity, c.max_splits, c.max_context, c.kv_heads // world, c.workers)
        t = P.device_tables(b.lengths + [0] * 0, b.splits, len(b.lengths), g, 4)
        records, _, _ = P.split_records(b.lengths, split_hints(b.lengths), g)
        assert t["record_count"] == len(records)
        assert sum(cnt for cnt in t["pack_count"]) == len(records) * (c.kv_heads // world)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        b = _small_c3()
        s = head_shard(b.config, rank, world)
        data = generate(b, device="cpu", kv_heads=s.kv_heads, head_offset=s.kv_offset)
        out = A.csr_attention(data["q"].float().numpy(), data["k"].float().numpy(),
                              data["v"].float().numpy(), data["indptr"].numpy(), data["pages"].numpy(),
                              b.lengths)
        parts = [torch.empty_like(torch.from_numpy(out)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(out))
        times = torch.tensor([1.0 + rank, 5.0 - rank], dtype=torch.float64)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        if rank == 0:
            full = generate(b, device="cpu")
            want = A.csr_attention(full["q"].float().numpy(), full["k"].float().numpy(),
                                   full["v"].float().numpy(), full["indptr"].numpy(),
                                   full["pages"].numpy(), b.lengths)
            got = assemble(parts).numpy()
            np.save(result_path, np.array([float(np.abs(got - want).max()), *times.tolist()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_ranks_reassemble_the_unsharded_oracle(world, tmp_path):
    result = tmp_path / "result.npy"
    mp.start_processes(_rank_main, args=(world, _free_port(), str(result)), nprocs=world, join=True,
                       start_method="spawn")
    err, t0, t1 = np.load(result)
    assert err < 1e-5
    assert (t0, t1) == (float(world), 5.0)        # max over ranks, elementwise
