"""Sparse MLA prefill and the latent-cache append of one DSA layer through the C ABI (`ssb_sparse_mla`,
`ssb_mla_cache_append`).

Mirrors the reference's calls: the TRTLLM sparse MLA (`trtllm_batch_decode_with_kv_cache_mla` with the indexer's
top-k token lists, split at 32,768 rows: ssengine/model/pp_patch.py:643-672; ssengine/kernels.py config 25) and the
fork's MLA cache write at the g0 slot mapping (config 23). The latent cache here is bf16 rows of 576 (latent 512 +
rope 64). No fallback: without the CUDA library these calls raise.
"""

from __future__ import annotations

import torch

from . import lib

HEADS, DQ, DV = 64, 576, 512


def sparse_mla(q: torch.Tensor, kv_cache: torch.Tensor, indices: torch.Tensor, qsl: torch.Tensor,
               page_table: torch.Tensor, scale: float, out: torch.Tensor, n_idx: int | None = None,
               stream=None, status: torch.Tensor | None = None) -> torch.Tensor:
    """q bf16 [T, 64, 576], kv_cache bf16 [slots, 576], indices int32 [T, >= n_idx], qsl int32 [R + 1],
    page_table int32 [R, width] -> out bf16 [T, 64, 512]."""
    so = lib.load()
    assert q.dtype == torch.bfloat16 and q.is_contiguous() and q.shape[1:] == (HEADS, DQ)
    assert kv_cache.dtype == torch.bfloat16 and kv_cache.is_contiguous() and kv_cache.shape[1] == DQ
    assert indices.dtype == torch.int32 and indices.stride(1) == 1 and out.is_contiguous()
    n = indices.shape[1] if n_idx is None else n_idx
    rc = so.ssb_sparse_mla(q.data_ptr(), q.shape[0], kv_cache.data_ptr(), indices.data_ptr(), indices.stride(0), n,
                           qsl.data_ptr(), qsl.shape[0] - 1, page_table.data_ptr(), page_table.shape[1], scale,
                           out.data_ptr(), None if status is None else status.data_ptr(), lib.stream_ptr(stream))
    lib.check("ssb_sparse_mla", rc)
    return out


def cache_append(src: torch.Tensor, slots: torch.Tensor, kv_cache: torch.Tensor, stream=None) -> None:
    """Rows of src bf16 [T, 576] into kv_cache at slots int64 [T] (< 0: skipped)."""
    so = lib.load()
    assert src.dtype == torch.bfloat16 and src.stride(1) == 1 and slots.dtype == torch.int64
    rc = so.ssb_mla_cache_append(src.data_ptr(), src.stride(0), slots.data_ptr(), src.shape[0], kv_cache.data_ptr(),
                                 lib.stream_ptr(stream))
    lib.check("ssb_mla_cache_append", rc)
