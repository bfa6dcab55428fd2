"""KDA (Kimi delta attention) prefill in numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py).

Interface followed (the reference's `kda_prefill_forward`, ssengine/model/pp_patch.py:215-244, and its helpers):

- sequences are (first row, end row, state block, has initial state), the reference's `KdaPrefillMeta.seqs`
  (pp_patch.py:189-197; tables in kda_conv.py:135-143);
- short conv (kda_conv.py:56-64 `_x_row`, :66-102 `kda_conv_qkv_kernel`, :110-132 state kernels): channel-last,
  width 4, no bias, over the packed q|k|v columns [0, 3P) of the in_proj rows; the 3 rows before a sequence's first
  row come from its conv state block (rows 0..2 = x rows start-3..start-1), or are 0 for a fresh request;
  out = SiLU(sum_w W[c, w] * x[t - 3 + w, c]), accumulated in fp32 from 0 over w = 0..3, rounded to bf16; afterwards
  the block holds the sequence's last 3 x rows (old state rows where the sequence is shorter than 3);
- recurrent state: FP32 [H, D, D] per state block, zero for a fresh request (kda_state.py:19-36), read at the start
  and written back at the end of the sequence; index order [head][value][key] (vLLM's KDA state pages);
- scale D^-0.5; gate from the raw projection g with `A_log`, `dt_bias` and the lower bound, beta through a sigmoid,
  both inside the kernel (pp_patch.py:221-243).

The recurrence itself lives in a third-party kernel absent from the reference tree (FlashInfer persistent KDA). It is
restated from the published KDA/gated-delta-rule algorithm as the upstream vLLM 0.22.0 FLA port states it
(vllm/model_executor/layers/fla/ops/fused_recurrent.py `fused_recurrent_gated_delta_rule_fwd_kernel` with IS_KDA,
kda.py `chunk_kda` with `use_qk_l2norm_in_kernel=True` as vLLM's Kimi layer calls it):

  q, k <- q / sqrt(|q|^2 + 1e-6), k / sqrt(|k|^2 + 1e-6)          (per head row)
  gk   = lower_bound * sigmoid(exp(A_log[h]) * (g + dt_bias))    (per key channel; the bounded "safe" gate)
  b    = sigmoid(beta)
  S    <- diag(exp(gk)) S                                         (S: [key, value])
  u    = b * (v - S^T k);  S <- S + k u^T;  o = scale * S^T q

Parity: pinned to flash-linear-attention 0.5.1's fp32 references (`naive_kda_lowerbound_gate`,
`naive_recurrent_kda`; tests/golden/kda_fla.npz: gate within 6.5e-7, outputs and final states within 1.4e-7 relative
L2) and cross-checked against vLLM 0.22.0's `chunk_kda` run on a B200 (tests/golden/kda_vllm.npz: within 4e-3, its
operands in bf16); the reference's own KDA kernel is a third-party library absent here.
"""

from __future__ import annotations

import numpy as np

from .mhc import bf16

WIDTH = 4
L2_EPS = 1e-6


def silu(a):
    a = np.asarray(a, np.float64)
    return a / (1.0 + np.exp(-a))


def conv(x, weight, conv_state, seqs, P, bf16_products: bool = False):
    """x [T, >= 3P] bf16 values, weight [3P, 4] bf16 values, conv_state [blocks, 3, 3P] bf16 values (copied, not
    modified), seqs [(start, end, block, init)] -> (q, k, v [T, P] bf16-valued float32, new conv_state).
    Products of bf16 values are exact in fp32, as Dao's channel-last kernel forms them (the reference's conv is
    bitwise that kernel's per sequence); `bf16_products` rounds each product to bf16 first, as vLLM's Triton
    `causal_conv1d_fn` does (used only to cross-check against it)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(weight, np.float32)
    st = np.array(conv_state, dtype=np.float32, copy=True)
    T, C = x.shape[0], 3 * P
    out = np.zeros((T, C), np.float32)
    for s, e, blk, init in seqs:
        n = e - s
        prev = st[blk] if init else np.zeros((WIDTH - 1, C), np.float32)
        rows = np.concatenate([prev, x[s:e, :C]], axis=0)                  # [n + 3, C]
        acc = np.zeros((n, C), np.float32)
        for j in range(WIDTH):                                              # products of bf16 values are exact
            prod = (w[:, j][None, :] * rows[j:j + n]).astype(np.float32)
            acc = (acc + (bf16(prod) if bf16_products else prod)).astype(np.float32)
        out[s:e] = bf16(silu(acc))
        st[blk] = rows[n:n + WIDTH - 1]                                     # last 3 rows (old state if n < 3)
    return out[:, :P], out[:, P:2 * P], out[:, 2 * P:], st


def gate(g, a_log, dt_bias, lower_bound, H, D):
    """Raw gate rows [T, H*D] -> per-channel log decay [T, H, D] (float64)."""
    g = np.asarray(g, np.float64).reshape(-1, H, D)
    z = np.exp(np.asarray(a_log, np.float64))[None, :, None] * (g + np.asarray(dt_bias, np.float64).reshape(1, H, D))
    return lower_bound / (1.0 + np.exp(-z))


def l2norm(x):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).sum(axis=-1, keepdims=True) + L2_EPS)


def recurrent(q, k, v, g, beta, a_log, dt_bias, lower_bound, scale, rec_state, seqs, H, D, heads=None):
    """Token-by-token KDA over each sequence. q, k, v [T, H*D] (conv outputs), g [T, H*D] raw gate, beta [T, H] raw;
    rec_state [blocks, H, D(value), D(key)] (copied) -> (out [T, H*D] float64, new rec_state float32). `heads`: only
    these heads are computed (the others' outputs stay 0 and their states as given), for large cases."""
    T = q.shape[0]
    qn = l2norm(np.asarray(q, np.float64).reshape(T, H, D))
    kn = l2norm(np.asarray(k, np.float64).reshape(T, H, D))
    vv = np.asarray(v, np.float64).reshape(T, H, D)
    gk = np.exp(gate(g, a_log, dt_bias, lower_bound, H, D))
    bt = 1.0 / (1.0 + np.exp(-np.asarray(beta, np.float64).reshape(T, H)))
    st = np.array(rec_state, dtype=np.float32, copy=True)
    out = np.zeros((T, H, D), np.float64)
    for s, e, blk, init in seqs:
        for h in (range(H) if heads is None else heads):
            S = st[blk, h].astype(np.float64).T.copy() if init else np.zeros((D, D))   # [key, value]
            for t in range(s, e):
                S *= gk[t, h][:, None]
                u = bt[t, h] * (vv[t, h] - S.T @ kn[t, h])
                S += np.outer(kn[t, h], u)
                out[t, h] = scale * (S.T @ qn[t, h])
            st[blk, h] = S.T.astype(np.float32)
    return out.reshape(T, H * D), st


def prefill(x, weight, conv_state, g, beta, a_log, dt_bias, lower_bound, rec_state, seqs, H, D):
    """The whole layer call: conv, then the recurrence -> (out, new conv_state, new rec_state)."""
    P = H * D
    q, k, v, cst = conv(x, weight, conv_state, seqs, P)
    out, rst = recurrent(q, k, v, g, beta, a_log, dt_bias, lower_bound, D ** -0.5, rec_state, seqs, H, D)
    return out, cst, rst


def gated_rmsnorm(o, gate, w, eps, D=128):
    """Per D-channel head: o * rsqrt(mean(o^2) + eps) * w * sigmoid(gate) (the KDA output norm)."""
    o = np.asarray(o, np.float64)
    T, P = o.shape
    oh = o.reshape(T, P // D, D)
    inv = 1.0 / np.sqrt((oh * oh).mean(axis=2, keepdims=True) + eps)
    g = 1.0 / (1.0 + np.exp(-np.asarray(gate, np.float64).reshape(T, P // D, D)))
    return (oh * inv * np.asarray(w, np.float64)[None, None, :] * g).reshape(T, P)


def nvfp4_linear(x, codes, sf, gs_w, gs_in):
    """bf16-valued x [T, K] quantized to NVFP4 with gs_in, times the dequantized weights [N, K] -> float64 [T, N]."""
    from . import nvfp4

    xc, xs = nvfp4.quantize(np.asarray(x, np.float32), gs_in)
    xq = nvfp4.dequantize(xc, xs, gs_in).astype(np.float64)
    w = nvfp4.dequantize_weight(codes, sf, gs_w, np.float64)
    return xq @ w.T


def attention_block(y, p, conv_state, rec_state, seqs, heads, gs_in, eps, lower_bound=-5.0, D=128):
    """The KDA attention block: in_proj -> f_b / g_b -> conv + recurrence -> gated RMSNorm -> o_proj, each projection
    NVFP4 with its output rounded to bf16 (the device's rounding points). p: in_proj, f_b, g_b, o_proj as (codes, sf,
    gs), conv_w, a_log, dt_bias, norm_w. -> (out bf16-valued [T, H], conv_state, rec_state)."""
    P = heads * D
    proj = bf16(nvfp4_linear(y, *p["in_proj"], gs_in))
    f_a, g_a = proj[:, 3 * P:3 * P + 128], proj[:, 3 * P + 128:3 * P + 256]
    beta = proj[:, 3 * P + 256:3 * P + 256 + heads]
    gate = bf16(nvfp4_linear(f_a, *p["f_b"], gs_in))
    ogate = bf16(nvfp4_linear(g_a, *p["g_b"], gs_in))
    o, cst, rst = prefill(proj[:, :3 * P], p["conv_w"], conv_state, gate, beta, p["a_log"], p["dt_bias"], lower_bound,
                          rec_state, seqs, heads, D)
    o = bf16(gated_rmsnorm(bf16(o), ogate, p["norm_w"], eps, D))
    return bf16(nvfp4_linear(o, *p["o_proj"], gs_in)), cst, rst
