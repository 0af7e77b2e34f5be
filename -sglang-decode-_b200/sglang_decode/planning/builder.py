"""GPU plan launch: one sm_100a kernel builds the whole step's task table.

Replaces the reference's ``planning/builder.py:6-33`` (four Triton launches) with a
single call of ``torch.ops.sglang_decode.plan_build``, which calls ``sgld_plan_build``.  The call also zeroes the claim counters of
every layer buffer registered with the plan (the reference's per-layer memset,
``runtime/engine.py:62``).  No allocation, host readback or tensor rebinding.
"""
from .. import _native


def build_plan(plan, force_mode=-1):
    """Enqueue the plan build for ``plan`` (a PlanBuffers) on the current stream."""
    _native.ops().plan_build(plan.storage, plan.geometry, int(force_mode),
                             plan.rules if plan.rule_count else None, plan.rule_count, plan.counters)


def any_static_rule(plan):
    # Capture-time metadata set by the runtime, never inspect a device scalar here.
    return getattr(plan, "has_static_rule", False)
