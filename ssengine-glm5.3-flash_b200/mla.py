"""Sparse MLA prefill, the FP8 latent-cache append and the FP8 query pack of one DSA layer through the C ABI
(`ssb_sparse_mla`, `ssb_mla_cache_append`, `ssb_mla_q_pack`).

Mirrors the reference's calls: the TRTLLM sparse MLA with FP8 query and cache (`trtllm_batch_decode_with_kv_cache_mla`
with the indexer's top-k token lists and bmm1 = scale * q_scale * k_scale, bmm2 = k_scale; split at 32,768 rows:
ssengine/model/pp_patch.py:643-672; ssengine/kernels.py config 25), the fork's FP8 MLA cache write
(`concat_and_cache_mla`, config 23) and the query's `scaled_fp8_quant`. The latent cache is e4m3 rows of 576 bytes
(latent 512 + rope 64). No fallback: without the CUDA library these calls raise.
"""

from __future__ import annotations

import torch

from . import lib

HEADS, DQ, DV = 64, 576, 512


def sparse_mla(q8: torch.Tensor, kv_cache: torch.Tensor, indices: torch.Tensor, qsl: torch.Tensor,
               page_table: torch.Tensor, bmm1: float, out: torch.Tensor, bmm2: float = 1.0, n_idx: int | None = None,
               stream=None, status: torch.Tensor | None = None) -> torch.Tensor:
    """q8 e4m3 bytes uint8 [T, 64, 576], kv_cache e4m3 bytes uint8 [slots, 576], indices int32 [T, >= n_idx], qsl int32
    [R + 1], page_table int32 [R, width] -> out bf16 [T, 64, 512]."""
    so = lib.load()
    assert q8.dtype == torch.uint8 and q8.is_contiguous() and q8.shape[1:] == (HEADS, DQ)
    assert kv_cache.dtype == torch.uint8 and kv_cache.is_contiguous() and kv_cache.shape[1] == DQ
    assert indices.dtype == torch.int32 and indices.stride(1) == 1
    assert out.dtype == torch.bfloat16 and out.is_contiguous()
    n = indices.shape[1] if n_idx is None else n_idx
    rc = so.ssb_sparse_mla(q8.data_ptr(), q8.shape[0], kv_cache.data_ptr(), indices.data_ptr(), indices.stride(0), n,
                           qsl.data_ptr(), qsl.shape[0] - 1, page_table.data_ptr(), page_table.shape[1], bmm1, bmm2,
                           out.data_ptr(), None if status is None else status.data_ptr(), lib.stream_ptr(stream))
    lib.check("ssb_sparse_mla", rc)
    return out


def cache_append(src: torch.Tensor, slots: torch.Tensor, kv_cache: torch.Tensor, k_scale: float = 1.0,
                 stream=None) -> None:
    """Rows of src bf16 [T, 576] into kv_cache uint8 [slots, 576] as e4m3(x / k_scale) at slots int64 [T] (< 0:
    skipped)."""
    so = lib.load()
    assert src.dtype == torch.bfloat16 and src.stride(1) == 1 and slots.dtype == torch.int64
    assert kv_cache.dtype == torch.uint8 and kv_cache.shape[1] == DQ
    rc = so.ssb_mla_cache_append(src.data_ptr(), src.stride(0), slots.data_ptr(), src.shape[0], kv_cache.data_ptr(),
                                 k_scale, lib.stream_ptr(stream))
    lib.check("ssb_mla_cache_append", rc)


def q_pack(lat: torch.Tensor, rows_pad: int, rope: torch.Tensor, rope_stride: int, T: int, q8: torch.Tensor,
           q_scale: float = 1.0, stream=None) -> torch.Tensor:
    """lat bf16 [64 * rows_pad, 512] (head-major absorbed queries), rope: bf16 rows whose head h slice starts at column
    h * rope_stride (64 values) -> q8 uint8 [T, 64, 576] = e4m3([lat | rope] / q_scale)."""
    so = lib.load()
    assert lat.dtype == torch.bfloat16 and lat.is_contiguous() and lat.shape == (HEADS * rows_pad, DV)
    assert rope.dtype == torch.bfloat16 and rope.stride(1) == 1
    assert q8.dtype == torch.uint8 and q8.is_contiguous() and q8.shape == (T, HEADS, DQ)
    rc = so.ssb_mla_q_pack(lat.data_ptr(), rows_pad, rope.data_ptr(), rope.stride(0), rope_stride, T, q8.data_ptr(),
                           q_scale, lib.stream_ptr(stream))
    lib.check("ssb_mla_q_pack", rc)
    return q8
