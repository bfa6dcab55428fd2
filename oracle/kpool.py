"""Indexer key pools in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

pool[p, c] = sum_j softmax_j(gate[4p+j, c] + ape[j, c]) * k[4p+j, c], the reference's `ref_compress`
(tests/test_kpool_cpu.py:20-25); tokens of a pool before a chunk's start come from the request's tail ring, seeded
with the previous chunk's trailing tokens (pp_patch.py:415-534, `ref_seed` tests/test_kpool_cpu.py:28-38). The
reference's property: any chunking of a prompt writes the pools of the unsplit prefill.

Parity: pinned to the reference's own insert path run here (pp_patch `kpool_heads` / `kpool_compress_insert` /
`kpool_seed_tail_cache` with its torch reference ops; tests/golden/kpool_ref.npz): pools within 2.2e-7 and the tail
ring identical, over chunked prefills of three requests that start inside pools and share microbatches.
"""

from __future__ import annotations

import numpy as np

POOL = 4


def compress(k4, g4, ape):
    """k4, g4 [4, D] (float), ape [4, D] -> [D] float64."""
    lg = np.asarray(g4, np.float64) + np.asarray(ape, np.float64)
    p = np.exp(lg - lg.max(axis=0, keepdims=True))
    p /= p.sum(axis=0, keepdims=True)
    return (p * np.asarray(k4, np.float64)).sum(axis=0)


def prefill_chunk(k_rows, g_rows, start, ape, pools, ring):
    """One request's chunk: rows at positions start.. ; pools dict p -> [D] (updated); ring [2, 4, D] (updated)."""
    n = len(k_rows)
    end = start + n
    for p in range(start // POOL, (end - POOL) // POOL + 1 if end >= POOL else 0):
        k4, g4 = [], []
        for j in range(POOL):
            pos = POOL * p + j
            if pos < start:
                k4.append(ring[0, pos % POOL]); g4.append(ring[1, pos % POOL])
            else:
                k4.append(k_rows[pos - start]); g4.append(g_rows[pos - start])
        pools[p] = compress(np.stack(k4), np.stack(g4), ape)
    for pos in range(max((end // POOL) * POOL, start), end):
        ring[0, pos % POOL] = k_rows[pos - start]
        ring[1, pos % POOL] = g_rows[pos - start]
    return pools, ring


def unsplit(k_all, g_all, ape):
    """All complete pools of a whole prompt."""
    n = len(k_all) // POOL
    return {p: compress(k_all[POOL * p:POOL * p + POOL], g_all[POOL * p:POOL * p + POOL], ape) for p in range(n)}
