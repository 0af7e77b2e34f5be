"""Long-lived, instance-private device buffers. Allocate before graph capture.

Same buffers and attribute names as the reference's ``runtime/workspace.py:1-40``:
``PlanBuffers`` holds the int32 SoA plan arrays and ``LayerBuffers`` the per-layer
claim counter, fp32 partial/LSE split slots and the output.  Additions of the B200
kernel: ``LayerBuffers.status`` (bounded-wait error word); ``counter`` has two words
(claim counter + a spare word; the merge zeroes both).
"""
from dataclasses import dataclass

import torch

from .. import _native
from ..config import DecodeConfig


class PlanBuffers:
    """Plan arrays, sized Bcap / E = Bcap*Smax / T = E*Hkv / W (workspace.py:7-23).  The same
    attribute names as the reference; here they are views of one storage tensor."""

    def __init__(self, config: DecodeConfig, device, rules=()):
        self.config = config
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())

        # Every plan buffer is a view of one int32 storage, in sgld_plan_buffers order
        # (sgld_plan_buffers_in_storage): the operators take the plan as that single tensor.
        sizes = _native.plan_field_words(config.batch_capacity, config.max_splits, config.kv_heads, config.workers)
        self.storage = torch.zeros(sum(sizes), dtype=torch.int32, device=self.device)
        offset = 0
        for name, n in zip(_native.PLAN_FIELDS, sizes):
            setattr(self, name, self.storage[offset:offset + n])
            offset += n
        rows = [[r.min_tasks, r.max_tasks, r.min_ratio, r.max_ratio, r.mode] for r in rules]
        self.rules = torch.tensor(rows or [[0, 0, 100, 100, 1]], dtype=torch.int32, device=self.device)
        self.rule_count = len(rows)
        self.has_static_rule = any(row[4] == 2 for row in rows)
        self.counters = None
        # Operator geometry (batch_capacity, max_splits, max_context, groups, workers).
        self.geometry = [config.batch_capacity, config.max_splits, config.max_context, config.kv_heads,
                         config.workers]
        # C views: pointers are stable for the lifetime of this object.
        self.c_buffers = _native.PlanBuffersC(
            **{name: getattr(self, name).data_ptr() for name in _native.PLAN_FIELDS})
        self.c_geometry = _native.PlanGeometry(config.batch_capacity, config.max_splits,
                                               config.max_context, config.kv_heads, config.workers)

    @property
    def rules_ptr(self):
        return self.rules.data_ptr() if self.rule_count else None

    def register_counters(self, counters: torch.Tensor):
        """Claim counters (int32) that every plan build resets to zero."""
        if counters.dtype != torch.int32 or not counters.is_contiguous():
            raise ValueError("counters must be a contiguous int32 tensor")
        self.counters = counters

    @property
    def counters_ptr(self):
        return self.counters.data_ptr() if self.counters is not None else None

    @property
    def counter_words(self):
        return self.counters.numel() if self.counters is not None else 0


@dataclass
class LayerBuffers:
    counter: torch.Tensor
    partial: torch.Tensor
    lse: torch.Tensor
    output: torch.Tensor
    status: torch.Tensor = None

    @classmethod
    def allocate(cls, config, device, dtype=torch.bfloat16, counter=None):
        shape = (config.batch_capacity, config.query_heads, config.max_splits)
        if counter is None:
            counter = torch.zeros(2, dtype=torch.int32, device=device)
        return cls(counter,
                   torch.empty((*shape, config.head_dim), dtype=torch.float32, device=device),
                   torch.empty(shape, dtype=torch.float32, device=device),
                   torch.empty((config.batch_capacity, config.query_heads, config.head_dim),
                               dtype=dtype, device=device),
                   torch.zeros(1, dtype=torch.int32, device=device))
