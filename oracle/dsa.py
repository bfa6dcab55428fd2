"""DSA attention block pieces in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

The block follows the reference's op order for a DSA layer (ssengine/kernels.py configs 12-27: fused q/kv
down-projection, q / kv latent RMSNorm, q_b, q absorb bmm, MLA cache append, indexer projections, kpool insert, logits,
top-k, expansion, sparse MLA, v_up bmm, o_proj); the per-op arithmetic is restated from the published DeepSeek-V3.2 /
MLA definitions (parity unpinned: the fork and its kernels are absent). Rotary embedding: interleaved pairs
(2i, 2i + 1) of each 64-dim rope slice, angle pos * theta^(-i / 32) -- the MLA rope as upstream vLLM 0.22.0 builds
GLM-5's DSA layers (vllm/model_executor/models/deepseek_v2.py: `GlmMoeDsaForCausalLM` is the DeepSeek-V2/V3.2 model,
whose MLA rotary embedding has is_neox_style=False).
"""

from __future__ import annotations

import numpy as np

from . import nvfp4
from .mhc import bf16


def rmsnorm(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * np.asarray(w, np.float64)


def rope(x, positions, theta):
    """x [..., T, 64] or [T, heads, 64] with positions [T] broadcast on the row axis -> rotated (float64)."""
    x = np.asarray(x, np.float64)
    i = np.arange(32)
    ang = np.asarray(positions, np.float64)[:, None] * theta ** (-i / 32.0)          # [T, 32]
    if x.ndim == 3:
        ang = ang[:, None, :]
    c, s = np.cos(ang), np.sin(ang)
    a, b = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = b * c + a * s
    return out


def grouped_linear(x_heads, codes, sf, gs_w, gs_in):
    """x_heads [heads, T, K] bf16 values; weights codes [heads, N, K], sf [heads, N, K / 16] -> [heads, T, N]."""
    out = []
    for h in range(x_heads.shape[0]):
        xc, xs = nvfp4.quantize(np.asarray(x_heads[h], np.float32), gs_in)
        xq = nvfp4.dequantize(xc, xs, gs_in).astype(np.float64)
        w = nvfp4.dequantize(codes[h], sf[h], gs_w).astype(np.float64)
        out.append(xq @ w.T)
    return np.stack(out)


def grouped_linear_bf16(x_heads, w):
    """x_heads [heads, T, K] bf16 values, w [heads, N, K] bf16 values -> [heads, T, N] float64 (the BF16 batched
    GEMM of the MLA absorb / v_up)."""
    return np.matmul(np.asarray(x_heads, np.float64), np.asarray(w, np.float64).transpose(0, 2, 1))


__all__ = ["rmsnorm", "rope", "grouped_linear", "grouped_linear_bf16", "bf16"]
