"""The split-KV combine oracle (``oracle.combine``) against unsplit attention, fp64, on CPU.

Splitting the keys of a sequence into equal chunks and merging the per-chunk (O, LSE) partials
must reproduce attention over all keys exactly (to fp64 rounding): non-causal for any query chunk,
and causal (ring attention: chunk c attends to chunks 0..c, the diagonal one top-left causal).
These properties pin the combine restatement the GPU tests check the kernel against.
"""

from __future__ import annotations

import numpy as np
import torch

import oracle
from fused_attn.workloads import make_qkv


def _chunks(x, s):
    return [c.contiguous() for c in torch.chunk(x, s, dim=2)]


def test_combine_of_key_chunks_equals_full_attention():
    q, k, v = make_qkv(1, 2, 256, 64, dtype=torch.float32, seed=61)
    qs, ks, vs = _chunks(q, 4), _chunks(k, 4), _chunks(v, 4)
    for causal in (False, True):
        o_full, lse_full = oracle.numpy_attention(q, k, v, causal=causal)
        for c in range(4):
            js = range(c + 1) if causal else range(4)
            parts = [oracle.numpy_attention(qs[c], ks[j], vs[j], causal=causal and j == c)
                     for j in js]
            o, lse = oracle.combine([p[0] for p in parts], [p[1] for p in parts])
            rows = slice(64 * c, 64 * (c + 1))
            assert np.abs(o - o_full[:, :, rows]).max() < 1e-12
            assert np.abs(lse - lse_full[:, :, rows]).max() < 1e-12


def test_combine_sentinels():
    """+inf / -inf partial rows weigh nothing; a row with no keys anywhere is o = 0, lse = +inf."""
    rng = np.random.default_rng(62)
    o1 = rng.standard_normal((1, 1, 3, 64))
    o2 = rng.standard_normal((1, 1, 3, 64))
    l1 = np.array([[[0.5, np.inf, np.inf]]])
    l2 = np.array([[[-np.inf, 1.5, np.inf]]])
    o, lse = oracle.combine([o1, o2], [l1, l2])
    assert np.allclose(o[0, 0, 0], o1[0, 0, 0]) and lse[0, 0, 0] == 0.5
    assert np.allclose(o[0, 0, 1], o2[0, 0, 1]) and lse[0, 0, 1] == 1.5
    assert np.all(o[0, 0, 2] == 0.0) and lse[0, 0, 2] == np.inf
    # Single partial: identity.
    o, lse = oracle.combine([o1], [np.full((1, 1, 3), 2.0)])
    assert np.allclose(o, o1) and np.all(lse == 2.0)
