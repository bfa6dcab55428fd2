"""DSA lightning indexer of one layer through the C ABI: pool logits (`ssb_indexer_logits`), the canonical per-row
top-k over the visible pools (`ssb_topk_canonical`) and the pool -> token expansion (`ssb_indexer_expand`).

Mirrors the reference's prefill indexer path: the fork's kpool `sparse_attn_indexer_kpool` (DeepGEMM
`fp8_mqa_logits` over each prefill chunk, `split_indexer_prefill_chunks` ssengine/model/pp_patch.py:587-634), the
routed top-k with canonicalisation (`_routed_top_k_per_row_prefill`, pp_patch.py:286-338, topk_canon.py) and
`kpool_fast.expand_into` (kpool_fast.py:48-59). No fallback: without the CUDA library these calls raise.

The FP8 forms (`q_quant`, `logits_fp8`, `kpool_insert_fp8`) keep the pool keys in the reference's 132-byte entries
(32 pools a 128-token page: 33 rows of 128 bytes, the codes then the scales) and quantize the queries per (token,
head), as vLLM's DeepSeek-V3.2 indexer does; they are not wired into the stage yet.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import lib

HEADS, DIM, POOL, POOLS_PER_PAGE, TILE = 32, 128, 4, 32, 128
FP8_PAGE_ROWS = 33                 # an FP8 pool page: 32 rows of 128 e4m3 codes, then a row of 32 fp32 scales


def work_groups(q_starts, q_lens, starts) -> np.ndarray:
    """Per request (first query row, query rows, position of its first row): int32 [G, 4] groups of <= 8 rows
    {request, first row, rows, pool tiles}, longest first (host side, like the reference's metadata); groups of equal
    tiles keep request and row order. A request's groups start at its first row every 8 rows; a group's tiles cover
    the pools visible to its last row ((position + 1) // 4 of them, 128 a tile); groups with no visible pool are
    left out."""
    qs, n, st = (np.asarray(a, np.int64).reshape(-1) for a in (q_starts, q_lens, starts))
    cnt = -(-np.maximum(n, 0) // 8)                                   # groups per request
    r = np.repeat(np.arange(len(n), dtype=np.int64), cnt)
    q0 = qs[r] + 8 * (np.arange(int(cnt.sum()), dtype=np.int64) - np.repeat(np.cumsum(cnt) - cnt, cnt))
    nq = np.minimum(8, qs[r] + n[r] - q0)
    tiles = -(-((st[r] + (q0 + nq - 1 - qs[r]) + 1) // POOL) // TILE)
    g = np.stack([r, q0, nq, tiles], axis=1)[tiles > 0]
    return g[np.argsort(-g[:, 3], kind="stable")].astype(np.int32).reshape(-1, 4)


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


def q_quant(q: torch.Tensor, q8: torch.Tensor, q_scale: torch.Tensor, stream=None) -> None:
    """FP8 indexer queries: bf16 [T, 32, 128] -> e4m3 codes uint8 [T, 32, 128] and fp32 ue8m0 scales [T, 32]."""
    so = lib.load()
    assert q.dtype == torch.bfloat16 and q.is_contiguous() and q.shape[1:] == (HEADS, DIM)
    assert q8.dtype == torch.uint8 and q8.is_contiguous() and q8.numel() == q.numel()
    assert q_scale.dtype == torch.float32 and q_scale.is_contiguous() and q_scale.numel() == q.shape[0] * HEADS
    lib.check("ssb_indexer_q_quant", so.ssb_indexer_q_quant(q.data_ptr(), q.shape[0] * HEADS, q8.data_ptr(),
                                                            q_scale.data_ptr(), lib.stream_ptr(stream)))


def logits_fp8(q8: torch.Tensor, q_scale: torch.Tensor, w: torch.Tensor, k_pages: torch.Tensor,
               page_table: torch.Tensor, groups: torch.Tensor, out: torch.Tensor, status: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
    """The FP8 form of `logits`: q8 uint8 [T, 32, 128] with q_scale fp32 [T, 32] (from `q_quant`), w bf16 [T, >= 32]
    head weights read in place, k_pages uint8 [pages * 33, 128] (the 132-byte-entry pool pages)."""
    so = lib.load()
    T = q8.shape[0]
    assert q8.dtype == torch.uint8 and q8.is_contiguous() and q8.shape[1:] == (HEADS, DIM)
    assert q_scale.dtype == torch.float32 and q_scale.is_contiguous() and q_scale.shape == (T, HEADS)
    assert w.dtype == torch.bfloat16 and w.stride(1) == 1 and w.shape[1] >= HEADS
    assert k_pages.dtype == torch.uint8 and k_pages.is_contiguous() and k_pages.shape[1] == DIM
    assert k_pages.shape[0] % FP8_PAGE_ROWS == 0 and out.dtype == torch.float32
    rc = so.ssb_indexer_logits_fp8(q8.data_ptr(), q_scale.data_ptr(), w.data_ptr(), w.stride(0), T, k_pages.data_ptr(),
                                   k_pages.shape[0] // FP8_PAGE_ROWS, page_table.data_ptr(), page_table.shape[1],
                                   groups.data_ptr(), groups.shape[0], out.data_ptr(), out.stride(0),
                                   None if status is None else status.data_ptr(), lib.stream_ptr(stream))
    lib.check("ssb_indexer_logits_fp8", rc)
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


def kpool_insert_fp8(k: torch.Tensor, gate: torch.Tensor, ape: torch.Tensor, reqs: torch.Tensor, max_rows: int,
                     page_table: torch.Tensor, pool_pages: torch.Tensor, tail_ring: torch.Tensor, stream=None) -> None:
    """`kpool_insert` into the FP8 pool pages (uint8 [pages * 33, 128]): codes and ue8m0 scales per pool row."""
    so = lib.load()
    assert k.dtype == torch.bfloat16 and gate.dtype == torch.bfloat16 and k.stride(0) == gate.stride(0)
    assert ape.dtype == torch.float32 and reqs.dtype == torch.int32 and pool_pages.dtype == torch.uint8
    assert pool_pages.shape[1] == DIM and pool_pages.shape[0] % FP8_PAGE_ROWS == 0
    rc = so.ssb_kpool_insert_fp8(k.data_ptr(), gate.data_ptr(), k.stride(0), ape.data_ptr(), reqs.data_ptr(),
                                 reqs.shape[0], max_rows, page_table.data_ptr(), page_table.shape[1],
                                 pool_pages.data_ptr(), tail_ring.data_ptr(), lib.stream_ptr(stream))
    lib.check("ssb_kpool_insert_fp8", rc)


def expand(pool_ids: torch.Tensor, positions: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """Token indices int32 [rows, 4k + 3] of the selected pools plus the row's incomplete last pool."""
    so = lib.load()
    k = pool_ids.shape[1]
    rc = so.ssb_indexer_expand(pool_ids.data_ptr(), pool_ids.stride(0), k, positions.data_ptr(), pool_ids.shape[0],
                               out.data_ptr(), out.stride(0), lib.stream_ptr(stream))
    lib.check("ssb_indexer_expand", rc)
    return out[:, :4 * k + 3]
