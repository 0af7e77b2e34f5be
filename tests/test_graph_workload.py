"""The C5 graph workload's replay steps: lengths grow by one token per step, every
request's slots are distinct and inside the pool, and appended tokens take the
pool's spare slots in request order (CPU only)."""
import torch

from sglang_decode.workloads import baseline, graph_step


def test_c5_steps_grow_by_one_token_and_use_distinct_pool_slots():
    b = baseline("C5")
    total0 = sum(b.lengths)
    cap = b.config.batch_capacity
    assert b.pool_tokens >= total0 + (len(b.replay_batches) - 1) * cap
    for step, batch in enumerate(b.replay_batches):
        lengths, pos = graph_step(b, step, batch)
        assert lengths == [n + step for n in b.lengths[:batch]]
        assert pos.numel() == sum(lengths)
        assert int(pos.min()) >= 0 and int(pos.max()) < b.pool_tokens
        assert torch.unique(pos).numel() == pos.numel()
        # request 0: its original slots, then the spare slots total0, total0 + cap, ...
        first = pos[:lengths[0]].tolist()
        assert first[:b.lengths[0]] == list(range(b.lengths[0]))
        assert first[b.lengths[0]:] == [total0 + j * cap for j in range(step)]


def test_c5_rejects_steps_beyond_the_spare_slots():
    b = baseline("C5")
    spare = (b.pool_tokens - sum(b.lengths)) // b.config.batch_capacity
    try:
        graph_step(b, spare + 1, 1)
    except ValueError:
        return
    raise AssertionError("expected a ValueError")
