"""Stage-level pieces of the oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py): RMSNorm, the NVFP4 lm_head
and the greedy token, restating the reference's `head_logits` / argmax (ssengine/model/stage.py:746-762): the last
row of each finished request -> final RMSNorm -> lm_head -> argmax (the lowest index among equal maxima).
Parity: the lm_head runs in the absent vLLM fork; the RMSNorm is cross-checked against vLLM 0.22.0's `rms_norm`
(tests/golden/norms_vllm.npz: identical bytes with vLLM's rounding of the normalized row before the weight multiply
restated, within one bf16 step with this build's single rounding); the head and argmax by rule KATs."""

from __future__ import annotations

import numpy as np

from oracle import nvfp4


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    inv = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + eps)
    return (x * inv.astype(np.float32) * np.asarray(w, dtype=np.float32)).astype(np.float32)


def head_logits(normed, codes, sf, gs_head: float, gs_x: float) -> np.ndarray:
    """normed fp32 [n, H] (bf16 values) -> NVFP4 input quant -> fp32 logits against the dequantized lm_head."""
    q, s = nvfp4.quantize(normed, gs_x)
    return nvfp4.dequantize(q, s, gs_x) @ nvfp4.dequantize(codes, sf, gs_head).T


def argmax_lowest(logits) -> np.ndarray:
    return np.argmax(np.asarray(logits), axis=1).astype(np.int64)   # numpy returns the first maximum
