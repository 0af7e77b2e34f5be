"""CPU oracle for the paged GQA decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference computes for the decode
path (StrongObserver/-SGLang-Decode-, ``src/sglang_decode``):

* ``oracle.planning`` -- the task-table specification
  (``planning/reference.py:15-76``) and the exact device-table semantics of the
  Triton plan kernels (``kernels/plan.py:7-135``, ``planning/builder.py:6-33``).
* ``oracle.attention`` -- the FP32 numerical oracle
  (``reference/attention.py:5-18``), the per-split partial/LSE slots
  (``kernels/attention.py:12-84``) and the split merge (``kernels/merge.py:7-30``).

Pinning: both modules are checked against golden vectors produced by the
reference itself (its CPU spec, and its Triton kernels run by the Triton CPU
interpreter) -- see ``tests/golden/make_golden.py`` and ``tests/test_oracle_*.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker or the timed
CPU baseline.  The product package never imports it.
"""
