"""Sparse MLA prefill in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

out[t, h, :] = sum_j softmax_j(scale * q[t, h, :] . kv[s_j, :]) * kv[s_j, :512] over the row's selected tokens
(absorbed-latent MLA attention as DeepSeek-V3.2 sparse attention defines it; the reference calls the TRTLLM sparse
MLA kernel, ssengine/kernels.py config 25, absent here: parity unpinned). slot(p) = pages[p // 128] * 128 + p % 128.
"""

from __future__ import annotations

import numpy as np

DV = 512


def slot_of(pages, pos):
    pos = np.asarray(pos, np.int64)
    return np.asarray(pages, np.int64)[pos // 128] * 128 + pos % 128


def sparse_mla(q, kv, indices, pages, scale):
    """q [n, 64, 576] rows of one request, kv [slots, 576], indices [n, m] positions (-1 = none) -> [n, 64, 512]."""
    q = np.asarray(q, np.float64)
    kv = np.asarray(kv, np.float64)
    out = np.zeros((q.shape[0], q.shape[1], DV))
    for i in range(q.shape[0]):
        sel = np.asarray(indices[i])
        sel = sel[sel >= 0]
        sel = sel[(sel // 128 < len(pages))]
        sel = sel[np.asarray(pages, np.int64)[sel // 128] >= 0]          # a token on a missing page is not read
        if sel.size == 0:
            continue
        k = kv[slot_of(pages, sel)]                       # [m, 576]
        s = scale * (q[i] @ k.T)                          # [64, m]
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[i] = p @ k[:, :DV]
    return out
