"""NVFP4 codec in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Format (NVIDIA NVFP4, as the reference's checkpoint and its quantizers use it: vLLM `scaled_fp4_quant`, called at
ssengine/kernels.py:109-118,179-181 of the reference; FlashInfer `mm_fp4` / trtllm MoE consume it):
- element: e2m1 (1 sign, 2 exponent, 1 mantissa bit, bias 1): magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6; code bit 3 is
  the sign. Two codes per byte, the even-indexed element in the low nibble.
- block scale: one unsigned e4m3 (bias 7, 3 mantissa bits, max 448, subnormals to 2^-9) per 16 consecutive elements
  along K.
- tensor scale: one fp32 "global scale" gs per tensor; a value decodes as e2m1(code) * e4m3(sf) / gs.

The quantization rule below is this project's own definition (the reference's quantizer is a closed library kernel
and is not reproduced). Every step is a single IEEE-754 fp32 operation, so the CUDA quantizer, which issues the same
operations with `__fdiv_rn` / `__fmul_rn`, produces the same bytes:
    amax = max |x| over the 16-block
    sf   = e4m3_rne_satfinite((amax / 6) * gs)
    r    = gs / float(sf)                      (codes are 0 when sf decodes to 0)
    code = e2m1_rne_satfinite(x * r)           (ties to the even code; the sign bit is the sign of x * r, so a
                                                value that rounds to zero keeps its sign, as the hardware
                                                conversion cvt.rn.satfinite.e2m1x2 and vLLM's quantizer give it;
                                                with sf = 0, r = 0 and every code is a signed zero)

Scale-factor storage ("128x4 atoms", the operand layout of the tcgen05 block-scaled MMA): rows padded to a multiple
of 128, K padded to a multiple of 256 (one GEMM k-block: 4 atom columns of 64 elements); the 128-row x 4-scale atom
(row block rb, atom column cb) is 512 contiguous bytes at ((rb * n_cb) + cb) * 512, and inside it scale (r, c) sits at
byte (r % 32) * 16 + ((r // 32) % 4) * 4 + c % 4.

Parity: known-answer tests of the format (tests/test_oracle_nvfp4.py), and a cross-check against the quantizer the
reference calls, upstream vLLM 0.22.0 `scaled_fp4_quant`, run on a B200 (tests/golden/nvfp4_vllm.npz,
tests/test_oracle_vllm_golden.py): the swizzled scale layout is identical to the 128x4 atoms; scales and codes are
byte-identical except for blocks whose (amax / 6) * gs sits on an e4m3 rounding midpoint, where vLLM's
reciprocal-multiply (amax * (1/6)) can land on the other side and the whole block then differs by one scale step.
"""

from __future__ import annotations

import numpy as np

E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_VALUES = np.concatenate([E2M1_MAG, -E2M1_MAG]).astype(np.float32)   # code -> value (code 8 is -0)
E4M3_MAX = np.float32(448.0)
SF_VEC = 16          # elements per block scale
ATOM_ROWS = 128
ATOM_COLS = 4


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for c in range(256):
        s, e, m = c >> 7, (c >> 3) & 0xF, c & 0x7
        if e == 0xF and m == 0x7:
            v = np.nan
        elif e == 0:
            v = m * 2.0 ** -9
        else:
            v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[c] = -v if s else v
    return t


E4M3_VALUES = _e4m3_table()


def e4m3_encode(v) -> np.ndarray:
    """fp32 -> e4m3 byte, round to nearest even, saturating at +-448 (NaN -> 0x7F)."""
    v = np.asarray(v, dtype=np.float32)
    sign = np.signbit(v)
    a = np.abs(v)
    out = np.zeros(a.shape, dtype=np.uint8)
    nan = np.isnan(a)
    sat = ~nan & (a >= E4M3_MAX)
    rest = ~nan & ~sat & (a > 0)
    x = a[rest]
    _, ex = np.frexp(x)                       # x = m * 2**ex, m in [0.5, 1): floor(log2 x) = ex - 1
    e = np.maximum(ex.astype(np.int32) - 1, -6)
    quantum = np.ldexp(np.float32(1.0), e - 3).astype(np.float32)
    q = np.rint(x / quantum).astype(np.float32) * quantum      # exact: power-of-two scaling
    q = np.minimum(q, E4M3_MAX)
    codes = np.zeros(x.shape, dtype=np.uint8)
    nz = q > 0
    qn = q[nz]
    sub = qn < np.float32(2.0 ** -6)
    c = np.empty(qn.shape, dtype=np.int32)
    c[sub] = np.rint(qn[sub] / np.float32(2.0 ** -9)).astype(np.int32)
    _, ex2 = np.frexp(qn[~sub])
    e2 = ex2.astype(np.int32) - 1
    mant = np.rint((qn[~sub] / np.ldexp(np.float32(1.0), e2).astype(np.float32) - 1.0) * 8.0).astype(np.int32)
    c[~sub] = ((e2 + 7) << 3) | mant
    codes[nz] = c.astype(np.uint8)
    out[rest] = codes
    out[sat] = 0x7E
    out[nan] = 0x7F
    out[sign & ~nan] |= 0x80
    out[(out & 0x7F) == 0] = 0          # no negative zero
    return out


def e4m3_decode(c) -> np.ndarray:
    return E4M3_VALUES[np.asarray(c, dtype=np.uint8)]


def e2m1_encode(a) -> np.ndarray:
    """fp32 -> e2m1 code (0..15), round to nearest, ties to the even code, saturating at +-6, the sign bit the sign
    of the input (-0.1 and -0.0 give code 8, negative zero); NaN -> 0."""
    a = np.asarray(a, dtype=np.float32)
    m = np.abs(a)
    idx = ((m > 0.25).astype(np.uint8) + (m >= 0.75) + (m > 1.25) + (m >= 1.75) + (m > 2.5) + (m >= 3.5)
           + (m > 5.0)).astype(np.uint8)
    neg = np.signbit(a) & ~np.isnan(a)
    return (idx | (neg.astype(np.uint8) << 3)).astype(np.uint8)


def e2m1_decode(c) -> np.ndarray:
    return E2M1_VALUES[np.asarray(c, dtype=np.uint8)]


def quantize(x, gs: float) -> tuple[np.ndarray, np.ndarray]:
    """x [R, K] (K % 16 == 0) -> (codes uint8 [R, K], one per element; scales uint8 [R, K // 16])."""
    x = np.asarray(x, dtype=np.float32)
    R, K = x.shape
    assert K % SF_VEC == 0, K
    gs = np.float32(gs)
    blk = x.reshape(R, K // SF_VEC, SF_VEC)
    amax = np.abs(blk).max(axis=2)
    sf = e4m3_encode((amax / np.float32(6.0)).astype(np.float32) * gs)
    sfv = e4m3_decode(sf)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(sfv > 0, gs / np.where(sfv > 0, sfv, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    codes = e2m1_encode((blk * r[:, :, None]).astype(np.float32))      # r = 0: signed zeros
    return codes.reshape(R, K), sf


def dequantize(codes, sf, gs: float) -> np.ndarray:
    """(codes [R, K], scales [R, K // 16], gs) -> fp32 [R, K]."""
    codes = np.asarray(codes, dtype=np.uint8)
    R, K = codes.shape
    v = e2m1_decode(codes).reshape(R, K // SF_VEC, SF_VEC) * e4m3_decode(sf)[:, :, None]
    return (v / np.float32(gs)).astype(np.float32).reshape(R, K)


# Weight dequantization memo for timing runs (the CPU baseline dequantizes its weights once, in its warm-up, and then
# times the arithmetic): None = off (the default; tests never use it), else a dict keyed by the arrays' identities.
# The caller keeps the weight arrays alive while the memo is on and clears it afterwards.
WEIGHT_MEMO: dict | None = None


def dequantize_weight(codes, sf, gs: float, dtype=np.float32) -> np.ndarray:
    """`dequantize` of a weight tensor (as `dtype`), through WEIGHT_MEMO when it is on."""
    if WEIGHT_MEMO is None:
        return dequantize(codes, sf, gs).astype(dtype, copy=False)
    key = (id(codes), id(sf), float(gs), np.dtype(dtype).str)
    w = WEIGHT_MEMO.get(key)
    if w is None:
        w = WEIGHT_MEMO[key] = dequantize(codes, sf, gs).astype(dtype, copy=False)
    return w


def pack(codes) -> np.ndarray:
    """codes [R, K] -> bytes [R, K // 2], element 2i in the low nibble."""
    codes = np.asarray(codes, dtype=np.uint8)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def unpack(packed) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


def atom_cols(k: int) -> int:
    """Atom columns per row block: K padded to 256 (one GEMM k-block), 4 atoms (64 elements each) per 256."""
    return -(-k // 256) * 4


def sf_to_atoms(sf) -> np.ndarray:
    """scales [R, K // 16] -> flat uint8 in the 128x4-atom layout: rows padded to 128, K padded to 256, zeros."""
    sf = np.asarray(sf, dtype=np.uint8)
    R, C = sf.shape
    nrb, ncb = -(-R // ATOM_ROWS), atom_cols(C * SF_VEC)
    pad = np.zeros((nrb * ATOM_ROWS, ncb * ATOM_COLS), dtype=np.uint8)
    pad[:R, :C] = sf
    # [rb, r32 = r // 32 within the block, r % 32, cb, c] -> [rb, cb, r % 32, r32, c]
    a = pad.reshape(nrb, 4, 32, ncb, ATOM_COLS).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(a).reshape(-1)


def atoms_to_sf(flat, rows: int, cols: int) -> np.ndarray:
    """Inverse of `sf_to_atoms`: flat atoms -> scales [rows, cols]."""
    nrb, ncb = -(-rows // ATOM_ROWS), atom_cols(cols * SF_VEC)
    a = np.asarray(flat, dtype=np.uint8)[: nrb * ncb * 512].reshape(nrb, ncb, 32, 4, ATOM_COLS)
    return np.ascontiguousarray(a.transpose(0, 3, 2, 1, 4)).reshape(nrb * ATOM_ROWS, ncb * ATOM_COLS)[:rows, :cols]
