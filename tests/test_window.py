"""Sliding-window CSR views (sglang_decode.window): the windowed bases and lengths select each
request's last min(L, window_left + 1) tokens; the oracle restricted to those tokens equals
the oracle on the windowed view (CPU)."""
import numpy as np
import torch

from oracle import attention as A
from sglang_decode.window import window_bases, window_lengths


def test_window_lengths_and_bases():
    lengths = torch.tensor([0, 1, 5, 100, 7], dtype=torch.int32)
    indptr = torch.tensor([0, 0, 1, 6, 106, 113, 113], dtype=torch.int32)
    assert window_lengths([0, 1, 5, 100, 7], -1) == [0, 1, 5, 100, 7]
    assert window_lengths([0, 1, 5, 100, 7], 4) == [0, 1, 5, 5, 5]
    w = window_lengths(lengths, 4)
    assert w.tolist() == [0, 1, 5, 5, 5]
    b = window_bases(indptr, lengths, 4)
    assert b.tolist() == [0, 0, 1, 101, 108, 113, 113]
    assert window_bases(indptr, lengths, -1).tolist() == indptr.tolist()
    assert window_lengths(lengths, 0).tolist() == [0, 1, 1, 1, 1]


def test_windowed_view_matches_attention_over_the_last_tokens():
    rng = np.random.default_rng(0)
    lengths = [1, 9, 40, 3]
    hq, hkv, d = 4, 2, 16
    indptr = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    idx = rng.permutation(60)[:sum(lengths)].astype(np.int32)
    k = rng.standard_normal((60, hkv, d)).astype(np.float32)
    v = rng.standard_normal((60, hkv, d)).astype(np.float32)
    q = rng.standard_normal((4, hq, d)).astype(np.float32)
    for window_left in (0, 2, 8, 100):
        wl = window_lengths(lengths, window_left)
        bases = window_bases(torch.from_numpy(indptr), torch.tensor(lengths, dtype=torch.int32), window_left).numpy()
        got = np.stack([A.request_attention(q[r], k[idx[bases[r]:bases[r] + wl[r]]], v[idx[bases[r]:bases[r] + wl[r]]])
                        for r in range(len(lengths))])
        want = np.stack([A.request_attention(q[r], k[idx[indptr[r] + lengths[r] - wl[r]:indptr[r] + lengths[r]]],
                                             v[idx[indptr[r] + lengths[r] - wl[r]:indptr[r] + lengths[r]]])
                         for r in range(len(lengths))])
        assert np.allclose(got, want)
