"""DSA lightning indexer in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

- Logits over pooled keys (kpool = 4 tokens): logit[t, p] = sum_h w[t, h] * relu(q[t, h, :] . k_pool[p, :]) for the
  pools p < (pos_t + 1) // 4 that row t may see (the fork's kpool indexer calling DeepGEMM `fp8_mqa_logits`,
  ssengine/kernels.py config 19; the score is the DeepSeek-V3.2 lightning-indexer formula). Parity: the fork and
  DeepGEMM are absent; the score and the pool visibility are cross-checked against DeepGEMM's own reference of the
  score as vLLM 0.22.0 vendors it (`fp8_mqa_logits_torch`, fixture tests/golden/indexer_vllm.npz: same masked
  columns, values within 3.2e-3 of each row's largest logit, its bf16 score rounding); this build keeps q / k in bf16.
- Pool -> token expansion: restated from ssengine/model/kpool_fast.py:23-41 (`_expand_rows_kernel`; pure index
  arithmetic, the fork's `expand_pools_and_append_tail`).
- Pool keys paged like the KV: pool p of a request sits in its KV page p // 32 at row page * 32 + p % 32.
"""

from __future__ import annotations

import numpy as np

POOL = 4
POOLS_PER_PAGE = 32


def pool_rows(pages, n_pools):
    """Row of each pool 0..n_pools-1 in the paged pool-key cache."""
    p = np.arange(n_pools)
    return np.asarray(pages, np.int64)[p // POOLS_PER_PAGE] * POOLS_PER_PAGE + p % POOLS_PER_PAGE


def logits(q, w, k_cache, pages, positions):
    """q [n, 32, 128], w [n, 32], k_cache [rows, 128], pages of the request, positions [n] -> list of float64 rows
    (row i has (pos_i + 1) // 4 entries)."""
    out = []
    for i in range(q.shape[0]):
        n = (int(positions[i]) + 1) // POOL
        k = np.asarray(k_cache)[pool_rows(pages, n)].astype(np.float64)        # [n, 128]
        s = np.asarray(q[i], np.float64) @ k.T                                    # [32, n]
        out.append((np.maximum(s, 0.0) * np.asarray(w[i], np.float64)[:, None]).sum(axis=0))
    return out


def expand(pool_ids, positions, k):
    """pool_ids int [rows, k] (-1 fill), positions [rows] -> int32 [rows, 4k + 3]."""
    pool_ids = np.asarray(pool_ids)
    rows = pool_ids.shape[0]
    out = np.full((rows, 4 * k + 3), -1, np.int32)
    for r in range(rows):
        seq_len = int(positions[r]) + 1
        for c in range(4 * k):
            pid = int(pool_ids[r, c // POOL])
            out[r, c] = pid * POOL + c % POOL if pid >= 0 else -1
        tail_start = (seq_len // POOL) * POOL
        for off in range(seq_len - tail_start):
            out[r, 4 * k + off] = tail_start + off
    return out
