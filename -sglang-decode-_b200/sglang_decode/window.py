"""Sliding-window decode over CSR KV (page size 1), with no kernel change.

The reference has no sliding-window path: its SGLang adapter falls back for such layers
(``integrations/sglang_backend.py:84-90``) and ``PlanKey`` only names the window
(``runtime/engine.py:17``).  Here a window uses SGLang / FlashInfer's ``window_left``
convention: the decode query of a request of length L attends to its last
W = min(L, window_left + 1) tokens (window_left < 0 means no window).

A CSR request's tokens are one contiguous run of ``kv_indices`` starting at ``indptr[r]``, and
the decode kernel reads ``kv_indices[base_r + t]`` for t < length_r, using ``indptr`` only for
the bases.  The window is therefore the same kernel with bases ``indptr[r] + L - W`` and lengths
W: write the windowed lengths into the plan (one plan per window size, as ``PlanKey``'s
``attention_window`` field says) and pass the shifted bases as ``indptr``.
"""
from __future__ import annotations

import torch


def window_lengths(lengths, window_left: int):
    """W_r = min(L_r, window_left + 1); unchanged when window_left < 0.  Works on Python lists
    and on int32 tensors (on any device)."""
    if window_left < 0:
        return lengths
    if isinstance(lengths, torch.Tensor):
        return torch.clamp(lengths, max=window_left + 1)
    return [min(n, window_left + 1) for n in lengths]


def window_bases(indptr: torch.Tensor, lengths: torch.Tensor, window_left: int) -> torch.Tensor:
    """Per-request CSR bases of the window: indptr[r] + L_r - W_r (int32, on indptr's device).

    ``indptr`` holds at least len(lengths) entries; ``lengths`` are the full lengths.  Entries
    past len(lengths) are copied unchanged (the plan never reads them)."""
    if indptr.dtype != torch.int32 or lengths.dtype != torch.int32:
        raise ValueError("indptr and lengths must be int32")
    out = indptr.clone()
    if window_left < 0:
        return out
    n = lengths.numel()
    w = window_lengths(lengths, window_left)
    out[:n] = indptr[:n] + (lengths - w)
    return out
