"""GPU plan launch: one sm_100a kernel builds the whole step's task table.

Replaces the reference's ``planning/builder.py:6-33`` (four Triton launches) with a
single C-ABI call, ``sgld_plan_build``.  The call also zeroes the claim counters of
every layer buffer registered with the plan (the reference's per-layer memset,
``runtime/engine.py:62``).  No allocation, host readback or tensor rebinding.
"""
import torch

from .. import _native


def build_plan(plan, force_mode=-1):
    """Enqueue the plan build for ``plan`` (a PlanBuffers) on the current stream."""
    stream = torch.cuda.current_stream(plan.device).cuda_stream
    _native.plan_build(plan.c_buffers, plan.c_geometry, int(force_mode), plan.rules_ptr,
                       plan.rule_count, plan.counters_ptr, plan.counter_words, stream)


def any_static_rule(plan):
    # Capture-time metadata set by the runtime, never inspect a device scalar here.
    return getattr(plan, "has_static_rule", False)
