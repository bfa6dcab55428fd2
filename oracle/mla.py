"""Sparse MLA prefill over the FP8 latent cache in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

out[t, h, :] = bmm2 * sum_j softmax_j(bmm1 * q8[t, h, :] . kv8[s_j, :]) * kv8[s_j, :512] over the row's selected
tokens (absorbed-latent MLA attention as DeepSeek-V3.2 sparse attention defines it), with q8 = e4m3(q / q_scale),
kv8 = e4m3(kv / k_scale), bmm1 = softmax scale * q_scale * k_scale, bmm2 = k_scale: the reference's FP8 query and
cache (ssengine/model/stage.py:88 kv_cache_dtype "fp8_e4m3"; ssengine/kernels.py configs 23 `concat_and_cache_mla`
and 25, the TRTLLM sparse MLA "FP8 q and cache", scales as vLLM 0.22's FlashInfer sparse MLA backend passes them,
vllm/v1/attention/backends/mla/flashinfer_mla_sparse.py `forward_mqa`). slot(p) = pages[p // 128] * 128 + p % 128;
a token on a missing page (negative entry) is not read. The kernel itself is third-party and absent here; the
attention over e4m3 inputs is cross-checked against FlashMLA's reference of sparse MLA prefill as vLLM 0.22.0 vendors
it (`reference_mla_sparse_prefill`, tests/golden/mla_vllm.npz: 2e-7 relative, -1 fills, repeated tokens and short rows
included); the e4m3 codec is pinned to torch's float8_e4m3fn cast (tests/test_oracle_mla.py).

E4M3 (OCP FP8): 1 sign, 4 exponent bits (bias 7), 3 mantissa bits; normals (1 + m / 8) 2^(e - 7), subnormals
m 2^-9, largest finite 448; encoding rounds to nearest, ties to even, and saturates to +-448 (the device's
`cvt.rn.satfinite`).
"""

from __future__ import annotations

import numpy as np

DV = 512
E4M3_MAX = 448.0


def e4m3_encode(x) -> np.ndarray:
    """float values -> e4m3 bytes (round to nearest even, saturating)."""
    x = np.asarray(x, np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.minimum(np.abs(x), E4M3_MAX)
    e = np.clip(np.floor(np.log2(np.maximum(a, 2.0 ** -12))), -6, 8)       # binade (subnormals share -6)
    step = 2.0 ** (e - 3)
    r = np.minimum(np.round(a / step) * step, E4M3_MAX)                     # exact: a / step scales by a power of 2
    normal = r >= 2.0 ** -6
    er = np.floor(np.log2(np.maximum(r, 2.0 ** -12)))
    E = np.where(normal, er + 7, 0).astype(np.int64)
    M = np.where(normal, np.round(r / 2.0 ** er * 8 - 8), np.round(r / 2.0 ** -9)).astype(np.int64)
    return (sign | (E << 3).astype(np.uint8) | M.astype(np.uint8)).astype(np.uint8)


def e4m3_decode(b) -> np.ndarray:
    """e4m3 bytes -> float64 values (the NaN codes 0x7f / 0xff are not produced by the encoder)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    E, M = (b >> 3) & 15, b & 7
    return s * np.where(E == 0, M * 2.0 ** -9, (1.0 + M / 8.0) * 2.0 ** (E - 7))


def quantize(x, scale: float) -> np.ndarray:
    """bf16-valued x -> e4m3 bytes of x * (1 / scale), the product rounded to fp32 first (the device's arithmetic)."""
    inv = np.float32(1.0) / np.float32(scale)
    return e4m3_encode(np.asarray(x, np.float32) * inv)


def slot_of(pages, pos):
    pos = np.asarray(pos, np.int64)
    return np.asarray(pages, np.int64)[pos // 128] * 128 + pos % 128


def sparse_mla(q8, kv8, indices, pages, bmm1: float, bmm2: float):
    """q8 [n, 64, 576] e4m3 bytes of one request's rows, kv8 [slots, 576] e4m3 bytes, indices [n, m] positions
    (-1 = none) -> float64 [n, 64, 512]."""
    q = e4m3_decode(q8)
    kv = e4m3_decode(kv8)
    out = np.zeros((q.shape[0], q.shape[1], DV))
    for i in range(q.shape[0]):
        sel = np.asarray(indices[i])
        sel = sel[sel >= 0]
        sel = sel[(sel // 128 < len(pages))]
        sel = sel[np.asarray(pages, np.int64)[sel // 128] >= 0]          # a token on a missing page is not read
        if sel.size == 0:
            continue
        k = kv[slot_of(pages, sel)]                       # [m, 576]
        s = bmm1 * (q[i] @ k.T)                           # [64, m]
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[i] = bmm2 * (p @ k[:, :DV])
    return out
