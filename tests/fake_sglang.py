"""A stand-in for the parts of SGLang v0.4.6.post5 that ScheduledTritonBackend touches.

SGLang is not installed here.  ``install()`` puts a minimal ``sglang`` module tree into
``sys.modules`` whose ``TritonAttnBackend`` does what the upstream base class does for
the adapter: it reads the model runner's geometry in ``__init__``, builds the CSR decode
metadata (``kv_indptr``, ``kv_indices``, ``num_kv_splits``) from ``req_to_token`` in its
``init_forward_metadata*`` hooks (same positional signatures), and has a
``forward_decode`` of its own, here an FP32 torch decode that counts its calls so tests
can see when the adapter falls back.  ``FakeModelRunner`` / ``FakeForwardBatch`` /
``FakeLayer`` carry the attributes the adapter reads.
"""
from __future__ import annotations

import math
import sys
import types

import torch


class FakeMode:
    def __init__(self, decode=True):
        self.decode = decode

    def is_decode_or_idle(self):
        return self.decode


class FakeMetadata(types.SimpleNamespace):
    pass


class FakeTritonAttnBackend:
    """Upstream-like base: geometry from the model runner, CSR metadata per step."""

    def __init__(self, model_runner, skip_prefill=False, kv_indptr_buf=None):
        c = model_runner.model_config
        self.model_runner = model_runner
        self.num_head = c.num_attention_heads
        self.num_kv_head = c.num_key_value_heads
        self.max_kv_splits = model_runner.server_args.triton_attention_num_kv_splits
        self.max_context_len = c.context_len
        self.device = model_runner.device
        self.device_core_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.forward_metadata = None
        self.fallback_calls = 0

    # -- metadata: kv_indptr / kv_indices over req_to_token, upstream-style split counts
    def _metadata(self, bs, req_pool_indices, seq_lens):
        pool = self.model_runner.req_to_token_pool.req_to_token
        lens = seq_lens[:bs].to(torch.int64)
        indptr = torch.zeros(bs + 1, dtype=torch.int32, device=self.device)
        indptr[1:] = torch.cumsum(lens, 0).to(torch.int32)
        rows = [pool[int(req_pool_indices[i]), :int(lens[i])] for i in range(bs)]
        indices = torch.cat(rows).to(torch.int32) if rows else torch.zeros(0, dtype=torch.int32, device=self.device)
        longest = int(lens.max()) if bs else 1
        chunk = max(1, math.ceil(longest / self.max_kv_splits))
        splits = torch.clamp((lens + chunk - 1) // chunk, 1, self.max_kv_splits).to(torch.int32)
        self.forward_metadata = FakeMetadata(kv_indptr=indptr, kv_indices=indices, num_kv_splits=splits)

    def init_forward_metadata(self, forward_batch):
        self._metadata(forward_batch.batch_size, forward_batch.req_pool_indices, forward_batch.seq_lens)

    def init_forward_metadata_capture_cuda_graph(self, bs, num_tokens, req_pool_indices, seq_lens,
                                                 encoder_lens, forward_mode, spec_info):
        self._metadata(bs, req_pool_indices, seq_lens)

    def init_forward_metadata_replay_cuda_graph(self, bs, req_pool_indices, seq_lens, seq_lens_sum,
                                                encoder_lens, forward_mode, spec_info, seq_lens_cpu):
        self._metadata(bs, req_pool_indices, seq_lens)

    def forward_decode(self, q, k, v, layer, forward_batch, save_kv_cache=True):
        """The original decode the adapter falls back to (FP32 torch, no logit cap)."""
        self.fallback_calls += 1
        pool = forward_batch.token_to_kv_pool
        if save_kv_cache:
            pool.set_kv_buffer(layer, forward_batch.out_cache_loc, k, v)
        meta = self.forward_metadata
        kb, vb = pool.get_key_buffer(layer.layer_id), pool.get_value_buffer(layer.layer_id)
        bs = q.shape[0]
        hq, hkv, d = layer.tp_q_head_num, layer.tp_k_head_num, layer.qk_head_dim
        out = torch.zeros(bs, hq, d, dtype=torch.float32, device=q.device)
        qf = q.view(bs, hq, d).float()
        for r in range(bs):
            rows = meta.kv_indices[meta.kv_indptr[r]:meta.kv_indptr[r + 1]].long()
            key = kb[rows].float().repeat_interleave(hq // hkv, dim=1)      # [L, Hq, D]
            val = vb[rows].float().repeat_interleave(hq // hkv, dim=1)
            s = torch.einsum("hd,lhd->hl", qf[r], key) * layer.scaling
            out[r] = torch.einsum("hl,lhd->hd", torch.softmax(s, dim=-1), val)
        return out.to(q.dtype).view(bs, -1)


class FakeKVPool:
    def __init__(self, layers, slots, kv_heads, head_dim, dtype, device, seed=5):
        g = torch.Generator(device=device).manual_seed(seed)
        self.k = [torch.randn(slots, kv_heads, head_dim, generator=g, device=device, dtype=dtype) for _ in range(layers)]
        self.v = [torch.randn(slots, kv_heads, head_dim, generator=g, device=device, dtype=dtype) for _ in range(layers)]
        self.writes = 0

    def get_key_buffer(self, layer_id):
        return self.k[layer_id]

    def get_value_buffer(self, layer_id):
        return self.v[layer_id]

    def set_kv_buffer(self, layer, loc, cache_k, cache_v):
        self.k[layer.layer_id][loc.long()] = cache_k.view(loc.numel(), *self.k[layer.layer_id].shape[1:])
        self.v[layer.layer_id][loc.long()] = cache_v.view(loc.numel(), *self.v[layer.layer_id].shape[1:])
        self.writes += 1


class FakeModelRunner:
    def __init__(self, *, layers, query_heads, kv_heads, head_dim, dtype, slots, max_requests=256,
                 context_len=4096, kv_splits=8, device="cuda"):
        self.device = torch.device(device)
        hf = types.SimpleNamespace(num_hidden_layers=layers)
        self.model_config = types.SimpleNamespace(
            num_attention_heads=query_heads, num_key_value_heads=kv_heads, context_len=context_len,
            hf_config=hf, is_multimodal=False, is_encoder_decoder=False, is_deepseek_mla=False)
        self.server_args = types.SimpleNamespace(pp_size=1, speculative_algorithm=None,
                                                 triton_attention_num_kv_splits=kv_splits)
        self.token_to_kv_pool = FakeKVPool(layers, slots, kv_heads, head_dim, dtype, self.device)
        self.req_to_token_pool = types.SimpleNamespace(
            req_to_token=torch.zeros(max_requests, context_len, dtype=torch.int32, device=self.device))


class FakeLayer(types.SimpleNamespace):
    @classmethod
    def make(cls, layer_id, query_heads, kv_heads, head_dim, logit_cap=0.0, sliding_window_size=-1):
        return cls(layer_id=layer_id, tp_q_head_num=query_heads, tp_k_head_num=kv_heads,
                   qk_head_dim=head_dim, v_head_dim=head_dim, scaling=head_dim ** -0.5,
                   logit_cap=logit_cap, sliding_window_size=sliding_window_size)


class FakeForwardBatch(types.SimpleNamespace):
    pass


_MODULES = ("sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.attention",
            "sglang.srt.layers.attention.triton_backend")


def install():
    """Register the fake module tree; returns the previous entries for ``uninstall``."""
    saved = {name: sys.modules.get(name) for name in _MODULES}
    for name in _MODULES:
        sys.modules[name] = types.ModuleType(name)
    sys.modules["sglang.srt.layers.attention.triton_backend"].TritonAttnBackend = FakeTritonAttnBackend
    sys.modules.pop("sglang_decode.integrations.sglang_backend", None)
    return saved


def uninstall(saved):
    for name, module in saved.items():
        if module is None:
            sys.modules.pop(name, None)
        else:
            sys.modules[name] = module
    sys.modules.pop("sglang_decode.integrations.sglang_backend", None)
