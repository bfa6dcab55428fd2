"""DSA lightning indexer of one layer through the C ABI: pool logits (`ssb_indexer_logits`), the canonical per-row
top-k over the visible pools (`ssb_topk_canonical`) and the pool -> token expansion (`ssb_indexer_expand`).

Mirrors the reference's prefill indexer path: the fork's kpool `sparse_attn_indexer_kpool` (DeepGEMM
`fp8_mqa_logits` over each prefill chunk, `split_indexer_prefill_chunks` ssengine/model/pp_patch.py:587-634), the
routed top-k with canonicalisation (`_routed_top_k_per_row_prefill`, pp_patch.py:286-338, topk_canon.py) and
`kpool_fast.expand_into` (kpool_fast.py:48-59). No fallback: without the CUDA library these calls raise.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import lib

HEADS, DIM, POOL, POOLS_PER_PAGE, TILE = 32, 128, 4, 32, 128


def work_groups(q_starts, q_lens, starts) -> np.ndarray:
    """Per request (first query row, query rows, position of its first row): int32 [G, 4] groups of <= 8 rows
    {request, first row, rows, pool tiles}, longest first (host side, like the reference's metadata)."""
    g = []
    for r, (qs, n, st) in enumerate(zip(q_starts, q_lens, starts)):
        for q0 in range(int(qs), int(qs) + int(n), 8):
            nq = min(8, int(qs) + int(n) - q0)
            last_pos = int(st) + (q0 + nq - 1 - int(qs))
            tiles = -(-((last_pos + 1) // POOL) // TILE)
            if tiles > 0:
                g.append((r, q0, nq, tiles))
    g.sort(key=lambda e: -e[3])
    return np.asarray(g, np.int32).reshape(-1, 4)


def key_ranges(positions: torch.Tensor):
    """Per row: the visible pools [0, (pos + 1) // 4) as int32 (ks, ke) on the device."""
    ke = ((positions + 1) // POOL).to(torch.int32)
    return torch.zeros_like(ke), ke


def logits(q: torch.Tensor, w: torch.Tensor, k_cache: torch.Tensor, page_table: torch.Tensor, groups: torch.Tensor,
           out: torch.Tensor, status: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """q bf16 [T, 32, 128], w bf16 [T, >= 32] head weights (a column view of the projection output: unit column
    stride, row stride a multiple of 8), k_cache bf16 [pages * 32, 128], page_table int32 [R, width], groups int32
    [G, 4] (device), out fp32 [T, ldl]."""
    so = lib.load()
    assert q.dtype == torch.bfloat16 and q.is_contiguous() and q.shape[1:] == (HEADS, DIM)
    assert w.dtype == torch.bfloat16 and w.stride(1) == 1 and w.shape[1] >= HEADS and k_cache.dtype == torch.bfloat16
    assert page_table.dtype == torch.int32 and groups.dtype == torch.int32 and out.dtype == torch.float32
    rc = so.ssb_indexer_logits(q.data_ptr(), w.data_ptr(), w.stride(0), q.shape[0], k_cache.data_ptr(),
                               k_cache.shape[0],
                               page_table.data_ptr(), page_table.shape[1], groups.data_ptr(), groups.shape[0],
                               out.data_ptr(), out.stride(0), None if status is None else status.data_ptr(),
                               lib.stream_ptr(stream))
    lib.check("ssb_indexer_logits", rc)
    return out


def topk(logit_rows: torch.Tensor, positions: torch.Tensor, k: int, out: torch.Tensor, stream=None,
         ranges: tuple | None = None) -> torch.Tensor:
    """Canonical top-k pool ids per row over [0, (pos + 1) // 4) (-1 fill), int32 [rows, k]. `ranges`: the rows' (ks,
    ke) from `key_ranges`, computed beforehand on a stream ordered before `stream` (when the call runs on a stream
    other than the current one, whose torch ops would not be ordered with it)."""
    so = lib.load()
    ks, ke = ranges if ranges is not None else key_ranges(positions)
    rc = so.ssb_topk_canonical(logit_rows.data_ptr(), logit_rows.shape[0], logit_rows.stride(0), ks.data_ptr(),
                               ke.data_ptr(), k, out.data_ptr(), logit_rows.shape[1], lib.stream_ptr(stream))
    lib.check("ssb_topk_canonical", rc)
    return out


def kpool_insert(k: torch.Tensor, gate: torch.Tensor, ape: torch.Tensor, reqs: torch.Tensor, max_rows: int,
                 page_table: torch.Tensor, pool_cache: torch.Tensor, tail_ring: torch.Tensor, stream=None) -> None:
    """Compress the pools the chunk completes into the pool-key cache and keep its trailing incomplete pool in the
    tail ring (reqs int32 [R, 4] on the device: first row, rows, start position, tail block)."""
    so = lib.load()
    assert k.dtype == torch.bfloat16 and gate.dtype == torch.bfloat16 and k.stride(0) == gate.stride(0)
    assert ape.dtype == torch.float32 and reqs.dtype == torch.int32 and pool_cache.dtype == torch.bfloat16
    rc = so.ssb_kpool_insert(k.data_ptr(), gate.data_ptr(), k.stride(0), ape.data_ptr(), reqs.data_ptr(),
                             reqs.shape[0], max_rows, page_table.data_ptr(), page_table.shape[1], pool_cache.data_ptr(),
                             tail_ring.data_ptr(), lib.stream_ptr(stream))
    lib.check("ssb_kpool_insert", rc)


def expand(pool_ids: torch.Tensor, positions: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """Token indices int32 [rows, 4k + 3] of the selected pools plus the row's incomplete last pool."""
    so = lib.load()
    k = pool_ids.shape[1]
    rc = so.ssb_indexer_expand(pool_ids.data_ptr(), pool_ids.stride(0), k, positions.data_ptr(), pool_ids.shape[0],
                               out.data_ptr(), out.stride(0), lib.stream_ptr(stream))
    lib.check("ssb_indexer_expand", rc)
    return out[:, :4 * k + 3]
