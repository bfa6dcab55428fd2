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
- The FP8 form (the reference's indexer cache, 132-byte entries: DeepSeek-V3.2's indexer as vLLM 0.22.0 runs it,
  models/deepseek_v2.py `Indexer.forward` and `ops.indexer_k_quant_and_cache`): a pool key row is stored as e4m3
  codes of x / s with s = 2^ceil(log2(max(1e-4, amax) / 448)) (ue8m0), a page of B entries holding B x 128 codes then
  B fp32 scales; a query is quantized per (token, head) the same way (floor 1e-10, the raw scale amax * fl(1 / 448)),
  its scale folded into the head weight with softmax scale D^-0.5 and n_heads^-0.5; logit = sum_h w'_h *
  relu(q8_h . k8) * s_k. Pinned to vLLM's Triton kernels run on the CPU (`_indexer_k_quant_and_cache_kernel`,
  `_per_token_group_quant_fp8`) and to `fp8_mqa_logits_torch` (tests/golden/indexer_fp8_vllm.npz).
"""

from __future__ import annotations

import numpy as np

POOL = 4
POOLS_PER_PAGE = 32
FP8_MAX = 448.0
ENTRY_BYTES = 128 + 4                  # e4m3 row + fp32 scale


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


def ue8m0(raw) -> np.ndarray:
    """2^ceil(log2(raw)) for positive float32 raw scales, from the exponent bits (exact)."""
    m, e = np.frexp(np.asarray(raw, np.float32))
    return np.ldexp(np.float32(1.0), np.where(m == 0.5, e - 1, e)).astype(np.float32)


def quant_pool_rows(x):
    """Key rows float [n, 128] -> (e4m3 codes uint8 [n, 128], ue8m0 scales float32 [n])."""
    from .mla import e4m3_encode

    x = np.asarray(x, np.float32)
    s = ue8m0(np.maximum(np.float32(1e-4), np.abs(x).max(axis=-1)) / np.float32(FP8_MAX))
    return e4m3_encode(x / s[:, None]), s


def quant_query_heads(q):
    """Queries float [n, heads, 128] -> (codes uint8 [n, heads, 128], ue8m0 scales float32 [n, heads])."""
    from .mla import e4m3_encode

    q = np.asarray(q, np.float32)
    raw = np.maximum(np.abs(q).max(axis=-1), np.float32(1e-10)) * (np.float32(1.0) / np.float32(FP8_MAX))
    s = ue8m0(raw)
    return e4m3_encode(q / s[..., None]), s


def write_pool_pages(cache, rows, codes, scales, per_page: int = POOLS_PER_PAGE):
    """Store pool entries at cache rows `rows` (row r = entry r % per_page of page r // per_page) in pages of
    `per_page` entries: uint8 cache [pages, per_page * 132], codes first, then the fp32 scales."""
    cache = np.asarray(cache)
    for r, c, s in zip(np.asarray(rows, np.int64), codes, np.asarray(scales, np.float32)):
        if r < 0:
            continue
        p, e = divmod(int(r), per_page)
        cache[p, e * 128:(e + 1) * 128] = c
        cache[p, per_page * 128 + 4 * e:per_page * 128 + 4 * e + 4] = np.frombuffer(s.tobytes(), np.uint8)
    return cache


def read_pool_pages(cache, rows, per_page: int = POOLS_PER_PAGE):
    """(codes uint8 [n, 128], scales float32 [n]) of the entries at cache rows `rows`."""
    cache = np.asarray(cache)
    p, e = np.divmod(np.asarray(rows, np.int64), per_page)
    codes = np.stack([cache[pp, ee * 128:(ee + 1) * 128] for pp, ee in zip(p, e)]) if len(p) else \
        np.zeros((0, 128), np.uint8)
    sc = np.array([np.frombuffer(cache[pp, per_page * 128 + 4 * ee:per_page * 128 + 4 * ee + 4].tobytes(),
                                 np.float32)[0] for pp, ee in zip(p, e)], np.float32)
    return codes, sc


def logits_fp8(q_codes, q_scale, w, cache, pages, positions, per_page: int = POOLS_PER_PAGE):
    """FP8 logits over the pools each row may see, from e4m3 query codes [n, heads, 128] with their scales
    [n, heads], head weights w [n, heads] (before the scale fold) and the paged FP8 pool cache."""
    from .mla import e4m3_decode

    heads, dim = q_codes.shape[1], q_codes.shape[2]
    out = []
    for i in range(q_codes.shape[0]):
        n = (int(positions[i]) + 1) // POOL
        kc, ks = read_pool_pages(cache, pool_rows(pages, n), per_page)
        wf = np.asarray(w[i], np.float64) * np.asarray(q_scale[i], np.float64) * dim ** -0.5 * heads ** -0.5
        sc = e4m3_decode(q_codes[i]) @ e4m3_decode(kc).T                         # [heads, n]
        out.append((np.maximum(sc, 0.0) * wf[:, None]).sum(axis=0) * ks.astype(np.float64))
    return out
