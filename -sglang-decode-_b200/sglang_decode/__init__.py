"""B200-native paged GQA decode for SGLang (drop-in for ``sglang_decode``).

Same public surface as the reference package: ``config`` (DecodeConfig, Mode),
``planning`` (build_plan, load_policy), ``runtime`` (DecodeEngine, PlanKey,
DecodeGraph, PlanBuffers, LayerBuffers) and ``integrations.sglang_backend``.
All GPU work runs in ``libsgld_sm100.so`` (hand-written sm_100a CUDA behind a C
ABI).  Importing this package does not initialise CUDA.
"""
__version__ = "0.2.0"
