"""mHC (4-stream hyper-connections) in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

Interface followed: the reference's fused layer-boundary op `MegaMhcPostPre` (ssengine/model/pp_patch.py:125-153:
residual, post mix, comb mix, layer input; RMSNorm with the layer's norm weight) and the stage edge
(`edge_send` = the last layer's hc_post flattened to [T, 4 * H], `edge_recv` = a standalone hc_pre, :156-163). The
arithmetic inside those library calls (DeepGEMM `mega_mhc`, vLLM TileLang) is absent from the reference tree; this
follows the published algorithm as the upstream vLLM 0.22.0 CPU path states it
(vllm/model_executor/kernels/mhc/torch.py `mhc_pre_torch` / `mhc_post_torch`):

  post:  new_res[j] = post[j] * x + sum_i comb[i, j] * res[i]                 (bf16 out)
  pre:   z = new_res flattened [4H] (fp32 of the bf16 values); mixes = (z @ fn.T) * rsqrt(mean(z^2) + rms_eps)
         pre  = sigmoid(mixes[0:4] * scale[0] + base[0:4]) + pre_eps
         post = sigmoid(mixes[4:8] * scale[1] + base[4:8]) * post_mult
         comb = softmax_row(mixes[8:24].view(4, 4) * scale[2] + base[8:24]) + sinkhorn_eps
         comb = comb / (colsum + sinkhorn_eps); then (repeat - 1) x: row-normalise, column-normalise (+ eps)
         y    = RMSNorm(sum_i pre[i] * new_res[i]) * norm_weight                (bf16 out; the layer input)

Parity: pinned to the outputs of vLLM 0.22.0's `mhc_pre_torch` / `mhc_post_torch` on seeded inputs
(tests/golden/mhc_vllm.npz, tests/test_oracle_vllm_golden.py); the reference's own fused kernels are third-party
libraries absent here.
"""

from __future__ import annotations

import numpy as np

HC = 4


def bf16(x) -> np.ndarray:
    """Round fp32 to bf16 (nearest even) and back to fp32 (32-bit integer arithmetic; only NaN bit patterns wrap).
    Large inputs go through in pieces of 2^20 values, so that the temporaries stay in cache."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size > 1 << 20:
        flat, out = x.reshape(-1), np.empty(x.size, np.float32)
        for i in range(0, x.size, 1 << 20):
            out[i:i + (1 << 20)] = bf16(flat[i:i + (1 << 20)])
        return out.reshape(x.shape)
    u = x.view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def sigmoid(v):
    return (1.0 / (1.0 + np.exp(-np.asarray(v, dtype=np.float64)))).astype(np.float32)


def post(x, res, post_mix, comb):
    """x [T, H], res [T, 4, H], post_mix [T, 4], comb [T, 4, 4] -> bf16-valued fp32 [T, 4, H]."""
    x, res = np.asarray(x, np.float32), np.asarray(res, np.float32)
    mixed = np.einsum("tij,tih->tjh", np.asarray(comb, np.float64), res.astype(np.float64))
    return bf16((mixed + np.asarray(post_mix, np.float64)[:, :, None] * x[:, None, :].astype(np.float64)))


def pre_mixes(res, fn, scale, base, rms_eps, pre_eps, sinkhorn_eps, post_mult, repeat):
    """The pre step up to its layer input: res [T, 4, H] (bf16 values) -> (post_mix [T, 4], comb [T, 4, 4],
    layer input [T, H] bf16-valued, before the layer's RMSNorm) -- the outputs of vLLM's `mhc_pre_torch`."""
    res = np.asarray(res, np.float32)
    T, hc, H = res.shape
    z = res.reshape(T, hc * H).astype(np.float64)
    mixes = z @ np.asarray(fn, np.float64).T
    mixes = mixes / np.sqrt((z * z).sum(axis=1, keepdims=True) / (hc * H) + rms_eps)
    scale, base = np.asarray(scale, np.float64), np.asarray(base, np.float64)
    pre_mix = 1.0 / (1.0 + np.exp(-(mixes[:, :hc] * scale[0] + base[:hc]))) + pre_eps
    post_mix = 1.0 / (1.0 + np.exp(-(mixes[:, hc:2 * hc] * scale[1] + base[hc:2 * hc]))) * post_mult
    logits = mixes[:, 2 * hc:].reshape(T, hc, hc) * scale[2] + base[2 * hc:].reshape(1, hc, hc)
    e = np.exp(logits - logits.max(axis=2, keepdims=True))
    comb = e / e.sum(axis=2, keepdims=True) + sinkhorn_eps
    comb = comb / (comb.sum(axis=1, keepdims=True) + sinkhorn_eps)
    for _ in range(repeat - 1):
        comb = comb / (comb.sum(axis=2, keepdims=True) + sinkhorn_eps)
        comb = comb / (comb.sum(axis=1, keepdims=True) + sinkhorn_eps)
    li = (pre_mix[:, :, None] * res.astype(np.float64)).sum(axis=1)
    li = bf16(li)                                        # the op's layer input is bf16 before the norm
    return post_mix.astype(np.float32), comb.astype(np.float32), li


def pre(res, fn, scale, base, rms_eps, pre_eps, sinkhorn_eps, post_mult, repeat, norm_w, norm_eps):
    """res [T, 4, H] (bf16 values) -> (post_mix [T, 4], comb [T, 4, 4], y [T, H] bf16-valued)."""
    post_mix, comb, li = pre_mixes(res, fn, scale, base, rms_eps, pre_eps, sinkhorn_eps, post_mult, repeat)
    inv = 1.0 / np.sqrt((li.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + norm_eps)
    y = bf16(li * inv * np.asarray(norm_w, np.float64))
    return post_mix, comb, y


def post_pre(x, res, post_mix, comb, *args):
    """The fused layer boundary: post of the previous layer's output, then pre of the next layer."""
    new_res = post(x, res, post_mix, comb)
    return (new_res,) + pre(new_res, *args)
