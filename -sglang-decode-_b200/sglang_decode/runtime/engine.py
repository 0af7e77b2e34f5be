"""Plan/execute API shared by the standalone harness and the SGLang adapter.

Same API and checks as the reference's ``runtime/engine.py:1-74``:
``DecodeEngine(config, device, dtype, layers, rules, force_mode)`` with
``prepare()`` (GPU plan build, once per compatible group per step) and
``execute(q, k, v, pages, layer=0, *, indptr=None, scale=None, logit_cap=0.0)`` (paged
``[page, token, head, dim]`` or CSR ``[token, head, dim]`` KV, arbitrary strides).
``execute`` enqueues the sm_100a persistent decode kernel and the split merge (a
programmatic dependent launch that overlaps the decode's tail) through the torch operator
``torch.ops.sglang_decode.decode``, which calls the C ABI; the claim counter is reset by
the plan build and left at zero by the call itself (the merge clears it once the decode has
completed; the reference's per-layer memset is not needed).
"""
from dataclasses import dataclass

import torch

from .. import _native
from ..config import DecodeConfig
from ..planning.builder import build_plan
from .workspace import LayerBuffers, PlanBuffers

_DTYPES = {torch.float16: _native.DTYPE_F16, torch.bfloat16: _native.DTYPE_BF16}
_FP8 = getattr(torch, "float8_e4m3fn", None)


@dataclass(frozen=True)
class PlanKey:
    """Caller-supplied sequence identity; pointer equality alone is insufficient."""
    sequence_layout: str
    split_layout: str
    head_layout: tuple
    attention_window: str = "full"


class DecodeEngine:
    def __init__(self, config: DecodeConfig, device="cuda", dtype=torch.bfloat16,
                 layers=1, rules=(), force_mode=-1):
        self.config, self.force_mode = config, force_mode
        self.dtype = dtype
        self.plan = PlanBuffers(config, device, rules)
        self.plan.has_static_rule = any(r.mode == 2 for r in rules)
        # One contiguous array of per-layer claim counters, reset by every plan build.
        self.counters = torch.zeros((layers, 2), dtype=torch.int32, device=self.plan.device)
        self.plan.register_counters(self.counters)
        self.layers = [LayerBuffers.allocate(config, self.plan.device, dtype, counter=self.counters[i])
                       for i in range(layers)]
        self._calls = {}       # layer -> arguments of its last execute (for c_args)
        self._default_scale = config.head_dim ** -0.5
        self._decode = _native.ops().decode

    def prepare(self):
        """Call once per compatible group per step, including on every graph replay."""
        build_plan(self.plan, self.force_mode)

    def execute(self, q, k, v, pages, layer=0, *, indptr=None, scale=None, logit_cap=0.0,
                k_scale=1.0, v_scale=1.0, k_new=None, v_new=None, new_loc=None):
        """KV layout: [pages,page_size,kv_heads,D], or CSR [tokens,kv_heads,D].

        Metadata and Q/KV must be ready on the current CUDA stream. Fixed buffers
        are reused; consumers must finish before reusing this execution instance.
        ``logit_cap`` > 0 soft-caps the scaled scores, s -> cap * tanh(s / cap), as SGLang
        does for models such as Gemma-2 (an addition: the reference has no capped path).
        K/V may be fp8 (``torch.float8_e4m3fn``, head_dim 128) with a fp16/bf16 Q: scores
        then use ``k_scale * k`` and the output ``v_scale * v`` (also an addition).

        Additions for the SGLang step around the decode (the reference copies Q into a
        capacity-sized buffer and calls ``set_kv_buffer`` first):

        * Q may have fewer rows than the capacity (any strides); the plan's active count
          must not exceed ``q.shape[0]`` (a task past it reads zeros and sets status 64).
        * ``k_new``/``v_new`` ([q rows, kv_heads, D], Q's dtype, any strides) with
          ``new_loc`` ([q rows] int64 or int32 token slots) add the KV-cache write to the
          call: row r is stored at slot ``new_loc[r]`` (an fp8 pool stores
          ``e4m3(x / k_scale)``, saturating) by a kernel chained right before the decode,
          so the result equals ``set_kv_buffer`` followed by the decode.
        """
        out = self.layers[layer]
        # Argument checks run in the operator (C++): wrong dtypes, shapes, devices or
        # scales raise ValueError there, before anything is enqueued.
        call = (q, k, v, pages, indptr, out.output, out.partial, out.lse, out.counter, out.status,
                self.plan.storage, self.plan.geometry, self.config.page_size,
                self._default_scale if scale is None else float(scale), float(logit_cap or 0.0),
                float(k_scale), float(v_scale), k_new, v_new, new_loc)
        self._calls[layer] = call
        self._decode(*call)          # torch.ops.sglang_decode.decode -> sgld_decode_persistent
        return out.output

    def c_args(self, layer=0):
        """The ``sgld_decode_args`` (ctypes) of this layer's last ``execute`` call, for callers
        that use the C ABI directly (e.g. ``sgld_decode_kernel_kind`` or the allocation-free
        entry point).  The struct points at the same tensors as that call."""
        (q, k, v, pages, indptr, output, partial, lse, counter, status, _, _, page_size, scale, cap, k_scale, v_scale,
         k_new, v_new, new_loc) = self._calls[layer]
        hq, hkv, d = self.config.query_heads, self.config.kv_heads, self.config.head_dim
        a = _native.DecodeArgs()
        a.q, a.k, a.v, a.out, a.pages = q.data_ptr(), k.data_ptr(), v.data_ptr(), output.data_ptr(), pages.data_ptr()
        if indptr is None:
            a.k_stride[:], a.v_stride[:], a.pt_stride[:] = k.stride(), v.stride(), pages.stride()
            a.indptr = None
        else:
            ks, vs = k.stride(), v.stride()
            a.k_stride[:] = (ks[0], 0, ks[1], ks[2])
            a.v_stride[:] = (vs[0], 0, vs[1], vs[2])
            a.pt_stride[:] = (0, 0)
            a.indptr = indptr.data_ptr()
        a.page_size = page_size
        a.kv_extent = k.shape[0] if k.shape[0] == v.shape[0] else 0
        a.q_stride[:] = q.stride()
        a.dtype = _DTYPES[q.dtype]
        a.kv_dtype = _native.DTYPE_E4M3 if k.dtype == _FP8 else a.dtype
        a.query_heads, a.kv_heads, a.head_dim = hq, hkv, d
        a.scale, a.logit_cap, a.k_scale, a.v_scale = scale, cap, k_scale, v_scale
        a.q_rows = q.shape[0]
        if new_loc is not None:
            a.k_new, a.v_new, a.new_loc = k_new.data_ptr(), v_new.data_ptr(), new_loc.data_ptr()
            a.knew_stride[:] = k_new.stride()
            a.vnew_stride[:] = v_new.stride()
            a.new_loc_int32 = 1 if new_loc.dtype == torch.int32 else 0
        a.counter, a.partial, a.lse, a.status = counter.data_ptr(), partial.data_ptr(), lse.data_ptr(), status.data_ptr()
        return a

    def kernel_kind(self, layer=0):
        """Name of the decode kernel this layer's last ``execute`` launched ("tcgen05", ...)."""
        return _native.decode_kernel_kind(self.c_args(layer), self.plan.c_buffers, self.plan.c_geometry)


def merge_splits(partial, lse, counts, error, out):
    """Stand-alone split merge (reference kernels/merge.py:7-30) into ``out`` [B, Hq, D]."""
    if partial.dtype != torch.float32 or lse.dtype != torch.float32:
        raise ValueError("partial and lse must be fp32")
    if out.dtype not in _DTYPES or not out.is_contiguous() or not partial.is_contiguous():
        raise ValueError("out must be contiguous fp16/bf16 and partial contiguous")
    b, hq, smax, d = partial.shape
    if tuple(lse.shape) != (b, hq, smax) or tuple(out.shape) != (b, hq, d) or counts.numel() < b:
        raise ValueError("merge shapes disagree")
    _native.ops().merge(partial, lse, counts, error, out)
    return out
