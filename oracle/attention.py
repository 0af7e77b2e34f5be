"""FP32 numerical oracle for paged / CSR GQA decode (test infrastructure only).

Restates the reference's ``paged_attention`` (``reference/attention.py:5-18``):
per request, gather the request's K/V rows, take an FP32 softmax over all of its
tokens for every query head (query head h reads KV head h // group), and return
``[Bcap, Hq, D]`` FP32 with zero rows for empty / inactive requests.

Also restated, for slot-level checks of the split-KV path:

* ``split_partials`` -- the per-record normalised partial output and natural-log
  LSE written to slot ``(request*Hq + head)*Smax + split``
  (``kernels/attention.py:53-84``);
* ``merge_splits`` -- the LSE-weighted merge over ``counts[r]`` splits in original
  split order with the 1e-30 denominator floor and NaN rows on error
  (``kernels/merge.py:7-30``).

Inputs are numpy arrays of any float dtype (fp16 K/V rows are upcast to FP32 after
the gather, as the reference does with ``.float()``); bf16 callers upcast with torch.
"""
from __future__ import annotations

import numpy as np


def _group(q: np.ndarray, k: np.ndarray) -> int:
    hq, hkv = q.shape[1], k.shape[-2]
    if hq % hkv:
        raise ValueError("query heads must be a multiple of KV heads")
    return hq // hkv


def _attend(qr: np.ndarray, key: np.ndarray, value: np.ndarray, group: int, scale: float,
            logit_cap: float = 0.0):
    """One request: qr [Hq, D], key/value [T, Hkv, D] (any float dtype, upcast here)
    -> [Hq, D] FP32 softmax attention, one KV head at a time (strided BLAS views).

    ``logit_cap > 0`` soft-caps the scaled scores, s -> cap * tanh(s / cap), before the
    softmax (SGLang's decode, vendored in the reference at
    ``third_party/sglang/decode_attention.py:124-128``)."""
    hkv, d = key.shape[1], qr.shape[-1]
    q3 = qr.reshape(hkv, group, d).astype(np.float32)
    key = key.astype(np.float32, copy=False)
    value = value.astype(np.float32, copy=False)
    out = np.empty((hkv, group, d), dtype=np.float32)
    for h in range(hkv):
        score = (q3[h] @ key[:, h, :].T) * np.float32(scale)                 # [G, T]
        if logit_cap > 0:
            score = np.float32(logit_cap) * np.tanh(score / np.float32(logit_cap))
        score -= score.max(axis=-1, keepdims=True)
        prob = np.exp(score)
        prob /= prob.sum(axis=-1, keepdims=True)
        out[h] = prob @ value[:, h, :]                                       # [G, D]
    return out.reshape(qr.shape)


def request_attention(qr, key, value, scale=None, logit_cap=0.0):
    """One request's FP32 decode (reference/attention.py:10-17 for a single row):
    qr [Hq, D], key/value [T, Hkv, D] already gathered in token order -> [Hq, D] FP32.

    For callers that gather a request's rows themselves (e.g. on the device, to upcast
    only those rows): ``paged_attention`` / ``csr_attention`` are this plus the gather."""
    scale = qr.shape[-1] ** -0.5 if scale is None else scale
    group = qr.shape[0] // key.shape[1]
    if group * key.shape[1] != qr.shape[0]:
        raise ValueError("query heads must be a multiple of KV heads")
    if key.shape[0] == 0:
        return np.zeros(qr.shape, dtype=np.float32)
    return _attend(qr, key, value, group, scale, logit_cap)


def paged_attention(q, k, v, pages, lengths, page_size, scale=None, logit_cap=0.0):
    """FP32 paged decode oracle (reference/attention.py:5-18).

    q [Bcap, Hq, D]; k, v [P, page_size, Hkv, D]; pages [Bcap, max_pages] int.
    """
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    group = _group(q, k)
    out = np.zeros(q.shape, dtype=np.float32)
    for r, length in enumerate(lengths):
        if length == 0:
            continue
        token = np.arange(length)
        physical = np.asarray(pages[r])[token // page_size].astype(np.int64)
        inner = token % page_size
        out[r] = _attend(q[r], k[physical, inner], v[physical, inner], group, scale, logit_cap)
    return out


def csr_attention(q, k, v, indptr, indices, lengths=None, scale=None, logit_cap=0.0):
    """FP32 CSR decode oracle: token t of request r lives at row indices[indptr[r] + t].

    k, v [N, Hkv, D].  This is the page_size=1 path the reference's engine takes when
    ``indptr`` is given (runtime/engine.py:54-61, kernels/attention.py:60-63).
    """
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    group = _group(q, k)
    out = np.zeros(q.shape, dtype=np.float32)
    if lengths is None:
        lengths = [int(indptr[r + 1] - indptr[r]) for r in range(len(indptr) - 1)]
    for r, length in enumerate(lengths):
        if length == 0:
            continue
        rows = np.asarray(indices[int(indptr[r]):int(indptr[r]) + length]).astype(np.int64)
        out[r] = _attend(q[r], k[rows], v[rows], group, scale, logit_cap)
    return out


def _rows_for(r, begin, end, *, pages=None, page_size=1, indptr=None, indices=None):
    token = np.arange(begin, end)
    if indptr is not None:
        return np.asarray(indices)[int(indptr[r]) + token].astype(np.int64), np.zeros_like(token)
    return np.asarray(pages[r])[token // page_size].astype(np.int64), token % page_size


def split_partials(q, k, v, records, max_splits, scale=None, *, pages=None, page_size=1,
                   indptr=None, indices=None):
    """Normalised partial output and natural-log LSE per (request, q_head, split) slot.

    ``records`` is a list of (request, split, begin, end).  Returns dense arrays
    partial [Bcap, Hq, Smax, D] and lse [Bcap, Hq, Smax] (NaN where no record wrote),
    following kernels/attention.py:53-84 in FP32.
    """
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    bcap, hq, d = q.shape
    csr = indptr is not None
    hkv = k.shape[1] if csr else k.shape[2]
    group = hq // hkv
    partial = np.full((bcap, hq, max_splits, d), np.nan, dtype=np.float32)
    lse = np.full((bcap, hq, max_splits), np.nan, dtype=np.float32)
    for request, split, begin, end in records:
        phys, inner = _rows_for(request, begin, end, pages=pages, page_size=page_size,
                                indptr=indptr, indices=indices)
        key = (k[phys] if csr else k[phys, inner]).astype(np.float32)        # [T, Hkv, D]
        value = (v[phys] if csr else v[phys, inner]).astype(np.float32)
        q3 = q[request].reshape(hkv, group, d).astype(np.float32)
        score = np.matmul(q3, key.transpose(1, 2, 0)) * np.float32(scale)    # [Hkv, G, T]
        m = score.max(axis=-1, keepdims=True)
        prob = np.exp(score - m)
        den = prob.sum(axis=-1, keepdims=True)
        acc = np.matmul(prob, value.transpose(1, 0, 2))                      # [Hkv, G, D]
        partial[request, :, split] = (acc / den).reshape(hq, d)
        lse[request, :, split] = (m + np.log(den)).reshape(hq)
    return partial, lse


def merge_splits(partial, lse, counts, error=0):
    """LSE merge over the first counts[r] splits, in split order (kernels/merge.py:7-30)."""
    bcap, hq, _, d = partial.shape
    out = np.zeros((bcap, hq, d), dtype=np.float32)
    for r in range(bcap):
        for h in range(hq):
            m = np.float32(-np.inf)
            den = np.float32(0.0)
            acc = np.zeros(d, dtype=np.float32)
            for s in range(int(counts[r])):
                new_m = max(m, lse[r, h, s])
                old_w = np.exp(np.float32(m - new_m))
                w = np.exp(np.float32(lse[r, h, s] - new_m))
                acc = acc * old_w + partial[r, h, s] * w
                den = den * old_w + w
                m = new_m
            out[r, h] = acc / max(den, np.float32(1e-30))
    if error:
        out[:] = np.nan
    return out


def tolerance_report(actual, expected):
    """(max_abs, mean_abs) error -- the north-star bar is 2e-2 / 2e-3."""
    diff = np.abs(np.asarray(actual, dtype=np.float64) - np.asarray(expected, dtype=np.float64))
    return float(diff.max()) if diff.size else 0.0, float(diff.mean()) if diff.size else 0.0
