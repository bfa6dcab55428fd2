"""One NVFP4 MoE layer in fp32 numpy -- the oracle's restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

What it restates. The reference runs the MoE block of every GLM-5.3-Flash MoE layer as (ssengine/kernels.py:174-193):
router GEMM (config 28) -> activation NVFP4 quant (29) -> FlashInfer `trtllm_fp4_block_scale_moe` (30: routing,
permute, grouped NVFP4 GEMM gate_up, SwiGLU, grouped GEMM down, finalize = weighted combine) plus the shared expert
(31, 32). That library (FlashInfer 0.7.2.dev20261008 / trtllm-gen) is absent from the reference tree and the
container, so this file follows the published algorithm of an NVFP4 top-k MoE with the routing BASELINE config 2
names (softmax over the router logits, top-k, renormalised), with every quantization point stated:

  xq        = nvfp4(x, gs_x)                                   (x: the layer input, bf16 values)
  logits    = deq(xq) @ deq(Wr).T                              fp32 [T, E]
  ids, w    = top-k of logits (descending, ties -> lower expert index); w = softmax over the k selected logits
  for every (t, j) and for the shared expert (index E, weight 1, every token):
    g, u    = deq(xq[t]) @ deq(W1[e]).T                        (rows [0, F) gate, [F, 2F) up)
    h       = silu(g) * u                                      silu(g) = g / (1 + exp(-g))
    hq      = nvfp4(h, gs_h)
    y       = deq(hq) @ deq(W2[e]).T
  out[t]    = sum_j w[t, j] * y[t, j] + y_shared[t]            (fp32, j in rank order, shared last)

Permutation (bit-exact contract with the CUDA path): expert-major, tokens ascending inside an expert, the shared
expert last; expert e's rows start at offset[e] = sum over e' < e of ceil(n_e' / 128) * 128 (so every 128-row tile
belongs to one expert).

Parity: the reference's library is absent; the routing rule is pinned by known-answer tests of the rule
(tests/test_oracle_moe.py), and the expert path is cross-checked against vLLM 0.22.0's CUTLASS NVFP4 MoE run on a
B200 on the same codes, scales, global scales and routing (tests/golden/moe_vllm.npz, tests/test_oracle_vllm_golden.py):
with vLLM's bf16 intermediates restated (`intermediates="bf16"`) the outputs agree to about 1e-4 relative L2; with this
layer's fp32 intermediates they differ by 2.4e-2, the requant of the bf16-rounded SwiGLU product accounting for it.
"""

from __future__ import annotations

import numpy as np

from oracle import nvfp4

TILE_M = 128


def route_softmax_topk(logits, k: int) -> tuple[np.ndarray, np.ndarray]:
    """logits fp32 [T, E] -> (ids int32 [T, k], weights fp32 [T, k]). Selection: k largest logits, ties to the lower
    expert index, slots in that rank order. Weights: softmax over the k selected logits."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    # stable sort on the negated value: equal values keep ascending index order
    order = np.argsort(-logits, axis=1, kind="stable")[:, :k].astype(np.int32)
    sel = np.take_along_axis(logits, order, axis=1)
    m = sel[:, :1]
    p = np.exp((sel - m).astype(np.float64)).astype(np.float32)
    w = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    return order, w


def route_sigmoid_bias(logits, k: int, bias, n_group: int = 1, topk_group: int = 1, scale: float = 1.0):
    """The reference model's routing (ssengine/kernels.py:182-187 "DeepSeek-V3 routing, scale 5/2"; its CPU test
    selects (logits.sigmoid() + bias).topk(8), tests/test_moe_tuning_cpu.py:63), restated from the published
    DeepSeek-V3 rule: score = sigmoid(logit) (evaluated in float64, rounded to fp32 once), choice = score + bias (fp32);
    with n_group > 1, a group's rank is the sum of its two largest choices and only the topk_group best groups stay
    eligible (ties: lower group); ids = the k largest eligible choices (ties: lower expert), slots in rank order;
    weights = the selected unbiased scores / their sum (fp32, summed in rank order) * scale.
    logits fp32 [T, E], bias fp32 [E] -> (ids int32 [T, k], weights fp32 [T, k])."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    score = (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)
    score = np.where(np.isnan(logits), np.float32(0), score)
    choice = (score + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    choice = np.where(np.isnan(logits), np.float32(-np.inf), choice)
    if n_group > 1:
        gs = E // n_group
        grp = np.sort(choice.reshape(T, n_group, gs), axis=2)
        gscore = (grp[:, :, -1] + grp[:, :, -2]).astype(np.float32)
        keep = np.argsort(-gscore, axis=1, kind="stable")[:, :topk_group]
        mask = np.zeros((T, n_group), bool)
        np.put_along_axis(mask, keep, True, axis=1)
        choice = np.where(np.repeat(mask, gs, axis=1), choice, np.float32(-np.inf))
    ids = np.argsort(-choice, axis=1, kind="stable")[:, :k].astype(np.int32)
    sel = np.take_along_axis(score, ids, axis=1)
    tot = np.zeros(T, np.float32)
    for j in range(k):
        tot = (tot + sel[:, j]).astype(np.float32)
    w = ((sel / tot[:, None]).astype(np.float32) * np.float32(scale)).astype(np.float32)
    return ids, w


def route(logits, k: int, p: dict):
    """The layer's routing rule: p["route"] = {"bias", "n_group", "topk_group", "scale"} selects the sigmoid rule,
    otherwise softmax top-k."""
    r = p.get("route")
    if r is None:
        return route_softmax_topk(logits, k)
    return route_sigmoid_bias(logits, k, r["bias"], r["n_group"], r["topk_group"], r["scale"])


def permutation(ids, num_experts: int, shared: bool = True):
    """Expert-major permutation. ids int32 [T, k] (experts 0..E-1). Returns
    (counts int32 [E(+1)], offsets int64 [E(+1) + 1] padded to 128-row tiles, rows int64 [T, k], shared_rows int64 [T]
    or None). rows[t, j] is the permuted row of (t, j)."""
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    E = num_experts
    ne = E + (1 if shared else 0)
    counts = np.bincount(ids.reshape(-1), minlength=E).astype(np.int64)
    if shared:
        counts = np.concatenate([counts, [T]])
    padded = -(-counts // TILE_M) * TILE_M
    offsets = np.zeros(ne + 1, dtype=np.int64)
    np.cumsum(padded, out=offsets[1:])
    rows = np.empty((T, k), dtype=np.int64)
    # rank of token t inside expert e = number of earlier tokens routed to e (a token routes to an expert once)
    flat_e = ids.reshape(-1)
    flat_t = np.repeat(np.arange(T), k)
    order = np.lexsort((flat_t, flat_e))           # expert-major, token ascending
    rank = np.empty_like(order)
    starts = np.concatenate([[0], np.cumsum(counts[:E])[:-1]])
    sorted_e = flat_e[order]
    rank[order] = np.arange(order.size) - starts[sorted_e]
    rows.reshape(-1)[:] = offsets[flat_e] + rank
    shared_rows = offsets[E] + np.arange(T) if shared else None
    return counts.astype(np.int32), offsets, rows, shared_rows


def _bf16(a) -> np.ndarray:
    """Round fp32 to bf16 (nearest even), returned as fp32 values."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def silu(g):
    g = np.asarray(g, dtype=np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def expert_ffn(xd, w1d, w2d, gs_h: float, F: int, intermediates: str = "fp32") -> np.ndarray:
    """xd [n, H] fp32 (dequantized input rows), w1d [2F, H], w2d [H, F] -> y [n, H] fp32.
    intermediates "bf16": the gate_up output and the SwiGLU product are rounded to bf16 before the requant, as vLLM's
    CUTLASS NVFP4 MoE keeps them (used only to cross-check against it); "fp32" is this layer's own rule."""
    gu = xd @ w1d.T
    if intermediates == "bf16":
        gu = _bf16(gu)
    h = silu(gu[:, :F]) * gu[:, F:]
    if intermediates == "bf16":
        h = _bf16(h)
    hq, hs = nvfp4.quantize(h, gs_h)
    return nvfp4.dequantize(hq, hs, gs_h) @ w2d.T


def dequantize_params(p: dict) -> dict:
    """fp32 weights of every GEMM (the checker's dequantized copy; the CPU baseline builds it once, outside timing)."""
    rc, rs, rg = p["router"]
    experts = [(nvfp4.dequantize(c1, s1, g1), nvfp4.dequantize(c2, s2, g2)) for (c1, s1, g1, c2, s2, g2) in
               p["experts"]]
    return {"router": nvfp4.dequantize(rc, rs, rg), "experts": experts}


def moe_forward(x, p: dict, k: int, ids=None, weights=None, return_parts: bool = False, dense: dict | None = None,
                intermediates: str = "fp32"):
    """x fp32 [T, H] (bf16 values) and the layer's logical NVFP4 parameters `p` (see `ssengine_b200.weights`):
    p["gs_x"], p["gs_h"], p["router"] = (codes [E, H], sf [E, H/16], gs), p["experts"] = list of E + 1 tuples
    (w1 codes [2F, H], w1 sf, w1 gs, w2 codes [H, F], w2 sf, w2 gs), the shared expert last.
    `ids` / `weights` override the routing (to check the FFN path on the CUDA path's own routing); `dense` is
    `dequantize_params(p)` when the caller holds it already, or "lazy" to dequantize one expert at a time.
    `intermediates` "bf16" restates vLLM's CUTLASS NVFP4 MoE (bf16 gate_up output, bf16 SwiGLU product, bf16 expert
    rows, weights and products in the combine, a bf16 sum) to cross-check the algorithm against it; the layer's own
    rule keeps all of them in fp32."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    E = len(p["experts"]) - 1
    F = p["experts"][0][0].shape[0] // 2
    xq, xs = nvfp4.quantize(x, p["gs_x"])
    xd = nvfp4.dequantize(xq, xs, p["gs_x"])
    lazy = isinstance(dense, str) and dense == "lazy"
    if lazy:
        # one expert's fp32 weights at a time (full-size layers on a row sample: 129 experts of 12.6M elements would
        # take 6.5 GB at once)
        dense = {"router": nvfp4.dequantize_weight(*p["router"]), "experts": None}
    elif dense is None:
        dense = dequantize_params(p)
    logits = (xd @ dense["router"].T).astype(np.float32)
    if ids is None:
        ids, weights = route(logits, k, p)
    ids = np.asarray(ids, dtype=np.int64)
    weights = np.asarray(weights, dtype=np.float32)
    out = np.zeros((T, H), dtype=np.float32)
    y_routed = np.zeros((T, k, H), dtype=np.float32)
    y_shared = np.zeros((T, H), dtype=np.float32)
    for e in range(E + 1):
        if e < E:
            tok, slot = np.nonzero(ids == e)
            o = np.argsort(tok, kind="stable")
            tok, slot = tok[o], slot[o]
        else:
            tok = np.arange(T)
        if tok.size == 0:
            continue
        if lazy:
            c1, s1, g1, c2, s2, g2 = p["experts"][e]
            w1d, w2d = nvfp4.dequantize_weight(c1, s1, g1), nvfp4.dequantize_weight(c2, s2, g2)
        else:
            w1d, w2d = dense["experts"][e]
        y = expert_ffn(xd[tok], w1d, w2d, p["gs_h"], F, intermediates)
        if e < E:
            y_routed[tok, slot] = y
        else:
            y_shared = y
    # combine in a fixed order: the k routed slots in rank order, the shared expert last
    if intermediates == "bf16":
        ws = _bf16(weights)
        for j in range(k):
            out += _bf16(ws[:, j:j + 1] * _bf16(y_routed[:, j]))
        out = _bf16(out + _bf16(y_shared))
    else:
        for j in range(k):
            out += weights[:, j:j + 1] * y_routed[:, j]
        out += y_shared
    if return_parts:
        return out, {"logits": logits, "ids": ids.astype(np.int32), "weights": weights, "y_routed": y_routed,
                     "y_shared": y_shared}
    return out
