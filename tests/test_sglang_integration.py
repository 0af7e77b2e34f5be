"""SGLang integration of the B200 decode: the import patch (CPU) and ScheduledTritonBackend
driven by a stand-in SGLang (GPU).

SGLang is not installed here, so ``tests/fake_sglang.py`` provides the base class and the
model-runner / forward-batch objects with the attributes the adapter reads.  The GPU tests
run the adapter's decode through this library and compare it with the FP32 oracle (max-abs
2e-2, mean-abs 2e-3), and check every fallback to the original decode, the KV-cache write,
the once-per-step plan build and the CUDA-graph hook signatures.
"""
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import attention as A
from sglang_decode.integrations import patch_sglang as P
from tests import fake_sglang as F

# ---------------------------------------------------------------------------- import patch (CPU)


def _checkout(tmp_path, text):
    path = tmp_path / P.RUNNER
    path.parent.mkdir(parents=True)
    path.write_text(text)
    return path


def test_patch_swaps_the_import_and_reverts_it(tmp_path):
    original = f"import os\n{P.UPSTREAM_IMPORT}\n\nclass ModelRunner:\n    pass\n"
    path = _checkout(tmp_path, original)
    assert P.apply(tmp_path, expected_commit=None) == path
    patched = path.read_text()
    assert P.PATCHED_IMPORT in patched and P.UPSTREAM_IMPORT not in patched
    P.apply(tmp_path, revert=True, expected_commit=None)
    assert path.read_text() == original


@pytest.mark.parametrize("sites", [0, 2])
def test_patch_needs_exactly_one_import_site(tmp_path, sites):
    text = "import os\n" + f"{P.UPSTREAM_IMPORT}\n" * sites
    path = _checkout(tmp_path, text)
    with pytest.raises(P.PatchError):
        P.apply(tmp_path, expected_commit=None)
    assert path.read_text() == text


def test_patch_refuses_other_commits_and_non_checkouts(tmp_path):
    text = f"{P.UPSTREAM_IMPORT}\n"
    path = _checkout(tmp_path, text)
    with pytest.raises(P.PatchError, match="not a git checkout"):
        P.apply(tmp_path)
    env = dict(os.environ, GIT_AUTHOR_NAME="t", GIT_AUTHOR_EMAIL="t@t", GIT_COMMITTER_NAME="t",
               GIT_COMMITTER_EMAIL="t@t")
    for cmd in (["git", "init", "-q"], ["git", "add", "-A"], ["git", "commit", "-q", "-m", "x"]):
        subprocess.run(cmd, cwd=tmp_path, check=True, env=env)
    with pytest.raises(P.PatchError, match="expected SGLang commit"):
        P.apply(tmp_path)
    assert path.read_text() == text
    with pytest.raises(SystemExit):
        P.main([str(tmp_path)])


# ---------------------------------------------------------------------------- adapter (GPU)


@pytest.fixture
def adapter():
    saved = F.install()
    try:
        from sglang_decode.integrations import sglang_backend
        yield sglang_backend
    finally:
        F.uninstall(saved)


def _runner(query_heads, kv_heads, layers=3, slots=8192, dtype=torch.bfloat16):
    return F.FakeModelRunner(layers=layers, query_heads=query_heads, kv_heads=kv_heads, head_dim=128,
                             dtype=dtype, slots=slots)


def _batch(runner, lengths, seed=3, decode=True):
    """Requests with distinct random slots; the newest token's slot is out_cache_loc."""
    g = torch.Generator().manual_seed(seed)
    slots = torch.randperm(runner.token_to_kv_pool.k[0].shape[0], generator=g)[:sum(lengths)]
    req = torch.randperm(runner.req_to_token_pool.req_to_token.shape[0], generator=g)[:len(lengths)]
    table = runner.req_to_token_pool.req_to_token
    loc, cursor = [], 0
    for r, n in zip(req.tolist(), lengths):
        table[r, :n] = slots[cursor:cursor + n].to(table.dtype).to(table.device)
        loc.append(int(slots[cursor + n - 1]))
        cursor += n
    dev = runner.device
    return F.FakeForwardBatch(batch_size=len(lengths), forward_mode=F.FakeMode(decode), spec_info=None,
                              req_pool_indices=req.to(dev), seq_lens=torch.tensor(lengths, device=dev),
                              out_cache_loc=torch.tensor(loc, device=dev),
                              token_to_kv_pool=runner.token_to_kv_pool)


def _count_prepares(engine):
    calls = {"n": 0}
    original = engine.prepare

    def counted():
        calls["n"] += 1
        original()
    engine.prepare = counted
    return calls


def _oracle(backend, runner, fb, layer, q):
    meta = backend.forward_metadata
    pool = runner.token_to_kv_pool
    bs = fb.batch_size
    lengths = fb.seq_lens.tolist()
    return A.csr_attention(q.view(bs, layer.tp_q_head_num, 128).float().cpu().numpy(),
                           pool.k[layer.layer_id].float().cpu().numpy(),
                           pool.v[layer.layer_id].float().cpu().numpy(),
                           meta.kv_indptr.cpu().numpy(), meta.kv_indices.cpu().numpy(), lengths,
                           layer.scaling, logit_cap=layer.logit_cap)


def _check(got, want):
    diff = np.abs(got.float().cpu().numpy().reshape(want.shape) - want)
    assert diff.max() <= 2e-2 and diff.mean() <= 2e-3, (diff.max(), diff.mean())


@pytest.mark.gpu
@pytest.mark.parametrize("query_heads,kv_heads", [(28, 4), (32, 4), (32, 8)])
def test_adapter_decode_matches_oracle_and_builds_one_plan_per_step(adapter, query_heads, kv_heads,
                                                                     cuda_device):
    runner = _runner(query_heads, kv_heads)
    backend = adapter.ScheduledTritonBackend(runner)
    assert backend.scheduled is not None, "this geometry must run on the B200 engine"
    prepares = _count_prepares(backend.scheduled)
    lengths = [1, 37, 129, 600, 2048, 4096 - 1, 300]
    fb = _batch(runner, lengths)
    backend.init_forward_metadata(fb)
    g = torch.Generator(device="cuda").manual_seed(11)
    for layer_id in range(3):
        layer = F.FakeLayer.make(layer_id, query_heads, kv_heads, 128)
        q = torch.randn(len(lengths), query_heads * 128, generator=g, device="cuda", dtype=torch.bfloat16)
        k = torch.randn(len(lengths), kv_heads, 128, generator=g, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(len(lengths), kv_heads, 128, generator=g, device="cuda", dtype=torch.bfloat16)
        out = backend.forward_decode(q, k, v, layer, fb)
        torch.cuda.synchronize()
        assert out.shape == (len(lengths), query_heads * 128)
        # the launch itself stored the new token's K/V (no set_kv_buffer call) and the
        # decode saw them: the oracle reads the updated pool
        pool = runner.token_to_kv_pool
        assert torch.equal(pool.k[layer_id][fb.out_cache_loc.long()], k)
        assert torch.equal(pool.v[layer_id][fb.out_cache_loc.long()], v)
        _check(out, _oracle(backend, runner, fb, layer, q))
    assert backend.fallback_calls == 0
    assert runner.token_to_kv_pool.writes == 0, "the KV write is fused into the decode launch"
    assert prepares["n"] == 1, "the plan is built once per step and reused by every layer"
    assert backend.scheduled.layers[0].status.item() == 0


@pytest.mark.gpu
def test_adapter_reads_q_k_v_in_place_from_the_projection_output(adapter, cuda_device):
    """q, k, v as SGLang passes them: views of one QKV projection output (q flat
    [bs, Hq*D], k/v [bs, Hkv, D]); no per-layer Q copy, the pool written by the launch."""
    runner = _runner(28, 4)
    backend = adapter.ScheduledTritonBackend(runner)
    lengths = [5, 700, 64, 1500]
    fb = _batch(runner, lengths, seed=8)
    backend.init_forward_metadata(fb)
    g = torch.Generator(device="cuda").manual_seed(12)
    bs, hq, hkv, d = len(lengths), 28, 4, 128
    for layer_id in range(2):
        layer = F.FakeLayer.make(layer_id, hq, hkv, d)
        qkv = torch.randn(bs, (hq + 2 * hkv) * d, generator=g, device="cuda", dtype=torch.bfloat16)
        q = qkv[:, :hq * d]
        k = qkv[:, hq * d:(hq + hkv) * d].view(bs, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(bs, hkv, d)
        out = backend.forward_decode(q, k, v, layer, fb)
        torch.cuda.synchronize()
        pool = runner.token_to_kv_pool
        assert torch.equal(pool.k[layer_id][fb.out_cache_loc.long()], k)
        _check(out, _oracle(backend, runner, fb, layer, q))
    assert backend.fallback_calls == 0 and runner.token_to_kv_pool.writes == 0
    assert backend.scheduled.layers[0].status.item() == 0


@pytest.mark.gpu
def test_adapter_rebuilds_the_plan_per_layer_when_reuse_is_off(adapter, monkeypatch, cuda_device):
    monkeypatch.setenv("DECODE_REUSE_PLAN", "0")
    runner = _runner(28, 4)
    backend = adapter.ScheduledTritonBackend(runner)
    prepares = _count_prepares(backend.scheduled)
    fb = _batch(runner, [100, 200])
    backend.init_forward_metadata(fb)
    for layer_id in range(3):
        layer = F.FakeLayer.make(layer_id, 28, 4, 128)
        q = torch.randn(2, 28 * 128, device="cuda", dtype=torch.bfloat16)
        kv = torch.randn(2, 4, 128, device="cuda", dtype=torch.bfloat16)
        backend.forward_decode(q, kv, kv, layer, fb)
    assert prepares["n"] == 3 and backend.fallback_calls == 0


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["sliding_window", "prefill", "over_capacity", "disabled", "spec_info"])
def test_adapter_falls_back_to_the_original_decode(adapter, monkeypatch, case, cuda_device):
    if case == "over_capacity":
        monkeypatch.setenv("DECODE_BATCH_CAPACITY", "2")
    if case == "disabled":
        monkeypatch.setenv("DECODE_DISABLE", "1")
    runner = _runner(28, 4)
    backend = adapter.ScheduledTritonBackend(runner)
    assert (backend.scheduled is None) == (case == "disabled")
    fb = _batch(runner, [50, 60, 70], decode=case != "prefill")
    if case == "spec_info":
        fb.spec_info = object()
    backend.init_forward_metadata(fb)
    layer = F.FakeLayer.make(0, 28, 4, 128, sliding_window_size=512 if case == "sliding_window" else -1)
    q = torch.randn(3, 28 * 128, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(3, 4, 128, device="cuda", dtype=torch.bfloat16)
    out = backend.forward_decode(q, kv, kv, layer, fb)
    assert backend.fallback_calls == 1
    assert out.shape == (3, 28 * 128)


@pytest.mark.gpu
def test_adapter_leaves_groups_above_16_and_other_head_dims_upstream(adapter, cuda_device):
    assert adapter.ScheduledTritonBackend(_runner(68, 4)).scheduled is None     # group 17
    odd = F.FakeModelRunner(layers=1, query_heads=8, kv_heads=8, head_dim=96, dtype=torch.bfloat16, slots=64)
    assert adapter.ScheduledTritonBackend(odd).scheduled is None


@pytest.mark.gpu
def test_adapter_cuda_graph_hooks_take_upstream_positional_arguments(adapter, cuda_device):
    runner = _runner(28, 4)
    backend = adapter.ScheduledTritonBackend(runner)
    fb = _batch(runner, [10, 20, 30])
    bs = fb.batch_size
    backend.init_forward_metadata_capture_cuda_graph(bs, bs, fb.req_pool_indices, fb.seq_lens, None,
                                                     F.FakeMode(True), None)
    assert backend._eligible_step and int(backend.scheduled.plan.active.item()) == bs
    backend.init_forward_metadata_replay_cuda_graph(bs, fb.req_pool_indices, fb.seq_lens,
                                                    int(fb.seq_lens.sum()), None, F.FakeMode(True), None,
                                                    fb.seq_lens.cpu())
    assert backend._eligible_step
    layer = F.FakeLayer.make(0, 28, 4, 128)
    q = torch.randn(bs, 28 * 128, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(bs, 4, 128, device="cuda", dtype=torch.bfloat16)
    out = backend.forward_decode(q, kv, kv, layer, fb)
    _check(out, _oracle(backend, runner, fb, layer, q))
    backend.init_forward_metadata_replay_cuda_graph(bs, fb.req_pool_indices, fb.seq_lens,
                                                    int(fb.seq_lens.sum()), None, F.FakeMode(True), object(),
                                                    fb.seq_lens.cpu())
    assert not backend._eligible_step


@pytest.mark.gpu
@pytest.mark.parametrize("cap", [5.0, 30.0, 50.0])
def test_adapter_runs_soft_capped_layers_on_the_engine(adapter, cap, cuda_device):
    """Gemma-2-style soft cap: the reference's adapter falls back; this one decodes with the cap."""
    runner = _runner(32, 4, layers=1)
    backend = adapter.ScheduledTritonBackend(runner)
    fb = _batch(runner, [17, 300, 1500, 4000])
    backend.init_forward_metadata(fb)
    layer = F.FakeLayer.make(0, 32, 4, 128, logit_cap=cap)
    g = torch.Generator(device="cuda").manual_seed(int(cap))
    q = 3.0 * torch.randn(4, 32 * 128, generator=g, device="cuda", dtype=torch.bfloat16)   # large scores
    kv = torch.randn(4, 4, 128, generator=g, device="cuda", dtype=torch.bfloat16)
    out = backend.forward_decode(q, kv, kv, layer, fb)
    torch.cuda.synchronize()
    assert backend.fallback_calls == 0
    _check(out, _oracle(backend, runner, fb, layer, q))
    uncapped = _oracle(backend, runner, fb, F.FakeLayer.make(0, 32, 4, 128), q)
    assert np.abs(_oracle(backend, runner, fb, layer, q) - uncapped).max() > 1e-3   # the cap matters here
