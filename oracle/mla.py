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
CHUNK = 1 << 20        # values per piece of a large encode


def e4m3_encode(x) -> np.ndarray:
    """fp32 values -> e4m3 bytes (round to nearest even, saturating to +-448, the sign of zero kept), by integer
    arithmetic on the fp32 bits: normals (|x| >= 2^-6) round their 23-bit mantissa to 3 bits, smaller values are
    multiples of 2^-9 (rint of |x| * 512; 8 of them is the smallest normal, code 0x08). Same bytes as
    `e4m3_encode_reference` below (tested) at a fraction of its cost. Large inputs go through in pieces of 2^20
    values (each value's code depends on that value alone), so that the temporaries stay in cache."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size > CHUNK:
        flat, out = x.reshape(-1), np.empty(x.size, np.uint8)
        for i in range(0, x.size, CHUNK):
            out[i:i + CHUNK] = e4m3_encode(flat[i:i + CHUNK])
        return out.reshape(x.shape)
    u = x.view(np.uint32)
    sign = ((u >> np.uint32(31)).astype(np.uint8) << np.uint8(7))
    a = u & np.uint32(0x7FFFFFFF)
    r = (a + np.uint32(0x7FFFF) + ((a >> np.uint32(20)) & np.uint32(1))) & np.uint32(0xFFF00000)
    e4 = (r >> np.uint32(23)).astype(np.int32) - 120                  # biased e4m3 exponent (127 - 7)
    normal = ((e4 << 3) | ((r >> np.uint32(20)) & np.uint32(7)).astype(np.int32)).clip(0, 0x7E).astype(np.uint8)
    sub = np.rint(np.abs(x) * np.float32(512.0)).astype(np.uint8)     # 0..8
    code = np.where(a >= np.uint32(0x3C800000), normal, sub)           # 2^-6
    code = np.where(a >= np.uint32(0x43E00000), np.uint8(0x7E), code)  # >= 448: saturate
    return (code | sign).astype(np.uint8)


def e4m3_encode_reference(x) -> np.ndarray:
    """float values -> e4m3 bytes (round to nearest even, saturating) in float64 arithmetic: the slow restatement the
    fast encoder is checked against."""
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


def _e4m3_values(b) -> np.ndarray:
    b = np.asarray(b, np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    E, M = (b >> 3) & 15, b & 7
    return s * np.where(E == 0, M * 2.0 ** -9, (1.0 + M / 8.0) * 2.0 ** (E - 7))


_E4M3_TABLE = _e4m3_values(np.arange(256))


def e4m3_decode(b) -> np.ndarray:
    """e4m3 bytes -> float64 values, by a table of the 256 codes (sign x 2^(E - 7) x (1 + M / 8); E = 0: M x 2^-9);
    the NaN codes 0x7f / 0xff are not produced by the encoder."""
    return _E4M3_TABLE[np.asarray(b, np.uint8)]


def quantize(x, scale: float) -> np.ndarray:
    """bf16-valued x -> e4m3 bytes of x * (1 / scale), the product rounded to fp32 first (the device's arithmetic)."""
    inv = np.float32(1.0) / np.float32(scale)
    return e4m3_encode(np.asarray(x, np.float32) * inv)


def slot_of(pages, pos):
    pos = np.asarray(pos, np.int64)
    return np.asarray(pages, np.int64)[pos // 128] * 128 + pos % 128


BLOCK = 128            # index columns per block of the FP8 attention
LAZY = 3.0             # a block raising a row's (base-2) max by more than this rescales the accumulated output
P_SCALE = 32.0         # P enters the P.V product as e4m3(32 p)


def sparse_mla_fp8p(q, kv8, cols, pages, bmm1: float, bmm2: float, decoded=None) -> np.ndarray:
    """One query row with its softmax weights rounded to e4m3 where the FP8 attention rounds them (the activation
    quantization point of the P.V product, as the reference's FP8 sparse MLA kernel has one): the row's index
    columns in blocks of 128 (blocks without a selected token skipped); base-2 scores x = s * bmm1 * log2(e) (fp32);
    a running max m kept until a block raises it by more than 2^3 (then the accumulated output and sum are scaled by
    2^(m_old - m_new)); p = 2^(x - m) (fp32); the sum of p unrounded; the product with e4m3(32 p) / 32.
    q [64, 576] float64 (the decoded e4m3 query), cols [m] (-1 = none) -> float64 [64, 512]. `decoded`: (sorted
    slots, their decoded rows) covering every slot the row reads, to decode shared cache rows once per call."""
    H = q.shape[0]
    o = np.zeros((H, DV))
    l = np.zeros(H)
    m = np.full(H, -np.inf, np.float32)
    sc = np.float32(bmm1 * 1.4426950408889634)
    pg = np.asarray(pages, np.int64)
    for b0 in range(0, len(cols), BLOCK):
        c = np.asarray(cols[b0:b0 + BLOCK], np.int64)
        c = c[(c >= 0) & (c // 128 < len(pg))]
        c = c[pg[c // 128] >= 0] if c.size else c
        if c.size == 0:
            continue
        slots = slot_of(pg, c)
        k = e4m3_decode(kv8[slots]) if decoded is None else decoded[1][np.searchsorted(decoded[0], slots)]
        x = ((q @ k.T).astype(np.float32) * sc).astype(np.float32)         # [64, mb]
        mb = x.max(axis=1)
        fresh = m == -np.inf
        jump = ~fresh & (mb > m + np.float32(LAZY))
        alpha = np.where(jump, np.exp2(np.where(jump, m - mb, 0).astype(np.float32)), 1.0)
        o *= alpha[:, None]
        l *= alpha
        m = np.where(fresh | jump, mb, m).astype(np.float32)
        p = np.exp2((x - m[:, None]).astype(np.float32)).astype(np.float32)
        l += p.astype(np.float64).sum(axis=1)
        pq = e4m3_decode(e4m3_encode(p * np.float32(P_SCALE)))
        o += pq @ k[:, :DV]
    return np.where(l[:, None] > 0, o * (bmm2 / (np.maximum(l, 1e-300)[:, None] * P_SCALE)), 0.0)


def sparse_mla(q8, kv8, indices, pages, bmm1: float, bmm2: float, p_fp8: bool = False):
    """q8 [n, 64, 576] e4m3 bytes of one request's rows, kv8 [slots, 576] e4m3 bytes, indices [n, m] positions
    (-1 = none) -> float64 [n, 64, 512]. p_fp8: the softmax weights rounded to e4m3 as the FP8 attention rounds them
    (`sparse_mla_fp8p`); else the exact softmax."""
    q = e4m3_decode(q8)
    out = np.zeros((q.shape[0], q.shape[1], DV))
    if p_fp8:
        pg = np.asarray(pages, np.int64)
        c = np.asarray(indices, np.int64).ravel()
        c = c[(c >= 0) & (c // 128 < len(pg))]
        c = c[pg[c // 128] >= 0] if c.size else c
        used = np.unique(slot_of(pg, c))                                   # every cache row any query row reads
        decoded = (used, e4m3_decode(kv8[used]))
        for i in range(q.shape[0]):
            out[i] = sparse_mla_fp8p(q[i], kv8, indices[i], pages, bmm1, bmm2, decoded)
        return out
    for i in range(q.shape[0]):
        sel = np.asarray(indices[i])
        sel = sel[sel >= 0]
        sel = sel[(sel // 128 < len(pages))]
        sel = sel[np.asarray(pages, np.int64)[sel // 128] >= 0]          # a token on a missing page is not read
        if sel.size == 0:
            continue
        k = e4m3_decode(kv8[slot_of(pages, sel)])         # [m, 576] (only the selected rows are decoded)
        s = bmm1 * (q[i] @ k.T)                           # [64, m]
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[i] = bmm2 * (p @ k[:, :DV])
    return out
