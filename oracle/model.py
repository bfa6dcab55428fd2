"""One Glm5Next pipeline stage composed from the oracle's pieces -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows the reference's stage forward (ssengine/model/stage.py:725-762 `run` / `run_layers` / `head_logits`, the
layer order of the kernel manifest ssengine/kernels.py:75-205 and the mHC edge of pp_patch.py:156-183):

  stage 0:      x = embed[token]; res = hc_expand(x) (4 copies)        later stages: res = the received [T, 4, H]
  per layer:    boundary A (pre only for the stage's first layer, else post of the previous FFN rows + pre)
                -> attention (KDA: oracle/kda.attention_block; DSA: `dsa_block` below)
                -> boundary B (post of the attention rows + pre) -> FFN (MoE: oracle/moe.moe_forward; dense: the
                   same SwiGLU expert FFN with one expert)
  stage end:    res = post of the last FFN rows (the edge send / final hc_post)
  last stage:   merged = mean of the 4 streams of each finished request's last row (bf16) -> RMSNorm -> BF16 lm_head
                (the reference's, config 35) -> fp32 logits -> argmax (lowest index among equal maxima)

Every intermediate is rounded to bf16 where the device path stores bf16 (the rounding points of the stage-wise
tests), and every activation quantization point is the device path's (NVFP4 inputs of the projections and experts,
e4m3 query and latent cache, the sparse MLA's softmax weights as e4m3(32 p): oracle/mla.sparse_mla_fp8p), so that the
composition and the device path take the same quantization decisions up to summation order.
Parameters come as numpy (the test reads them out of the device objects); states (KDA conv / recurrent, latent cache,
pool keys, tail ring) are numpy arrays updated in place.
"""

from __future__ import annotations

import numpy as np

from . import dsa as od
from . import indexer as oidx
from . import kda as ok
from . import kpool as okp
from . import mhc as omhc
from . import mla as omla
from . import moe as omoe
from . import nvfp4
from . import stage as ostage
from . import topk as otopk
from .mhc import bf16


def dense_ffn(y, w, gs_x: float, gs_h: float) -> np.ndarray:
    """The dense SwiGLU FFN: w = (w1 codes [2F, H], sf, gs, w2 codes [H, F], sf, gs) -> bf16-valued [T, H]."""
    c1, s1, g1, c2, s2, g2 = w
    xq, xs = nvfp4.quantize(np.asarray(y, np.float32), gs_x)
    xd = nvfp4.dequantize(xq, xs, gs_x)
    F = c1.shape[0] // 2
    return bf16(omoe.expert_ffn(xd, nvfp4.dequantize_weight(c1, s1, g1), nvfp4.dequantize_weight(c2, s2, g2), gs_h,
                                F))


def dsa_block(y, p, positions, reqs, kv_cache, pool_cache, tail, gs_in: float):
    """The DSA attention block on rows y [T, H] (bf16 values). p: a_proj, q_b, wq_idx, idx_proj, o_proj (codes, sf,
    gs), w_uk, w_uv (per-head bf16 weights [64, N, K]), q_norm, kv_norm, ape, q_lora, nope, v_dim, theta, eps, scale, q_scale,
    k_scale, and optionally indexer_fp8. reqs: per request (first row, rows, start position, pages, tail block). kv_cache
    uint8 [slots, 576] e4m3, pool_cache [rows, 128] (bf16 values; with indexer_fp8 uint8 [pages * 33, 128], the
    reference's 132-byte entries), tail [blocks, 2, 4, 128] -- all updated in place. -> bf16-valued [T, H]."""
    T = y.shape[0]
    QL, L, RP, NH = p["q_lora"], 512, 64, 64
    nope, v_dim = p["nope"], p["v_dim"]
    qh = nope + RP
    lin = lambda x, w: ok.nvfp4_linear(x, *w, gs_in)
    a = bf16(lin(y, p["a_proj"]))
    qa = bf16(od.rmsnorm(a[:, :QL], p["q_norm"], p["eps"]))
    kvn = bf16(od.rmsnorm(a[:, QL:QL + L], p["kv_norm"], p["eps"]))
    k_rope = bf16(od.rope(a[:, QL + L:QL + L + RP], positions, p["theta"]))
    kv_rows = np.concatenate([kvn, k_rope], axis=1)
    for first, n, start, pages, _ in reqs:
        slots = omla.slot_of(pages, np.arange(start, start + n))
        kv_cache[slots] = omla.quantize(kv_rows[first:first + n], p["k_scale"])
    q = bf16(lin(qa, p["q_b"])).reshape(T, NH, qh)
    q[:, :, nope:] = bf16(od.rope(q[:, :, nope:], positions, p["theta"]))
    q_lat = bf16(od.grouped_linear_bf16(q[:, :, :nope].transpose(1, 0, 2), *p["w_uk"]))       # [64, T, 512]
    q8 = omla.quantize(np.concatenate([q_lat.transpose(1, 0, 2), q[:, :, nope:]], axis=2), p["q_scale"])
    q_idx = bf16(lin(qa, p["wq_idx"])).reshape(T, 32, 128)
    idx = bf16(lin(y, p["idx_proj"]))
    k_idx, w, gate = idx[:, :128], idx[:, 128:160], idx[:, 160:288]
    out_lat = np.zeros((T, NH, L))
    fp8 = bool(p.get("indexer_fp8"))          # pool_cache: uint8 [pages * 33, 128], the 132-byte entries
    for first, n, start, pages, tblk in reqs:
        rows = slice(first, first + n)
        pools, ring = okp.prefill_chunk(k_idx[rows], gate[rows], start, p["ape"], {}, tail[tblk].copy())
        tail[tblk] = bf16(ring)
        if fp8:
            cache = pool_cache.reshape(-1, 33 * 128)
            for pid, v in pools.items():
                codes, sc = oidx.quant_pool_rows(np.asarray(v, np.float32)[None])
                oidx.write_pool_pages(cache, oidx.pool_rows(pages, pid + 1)[pid:pid + 1], codes, sc)
            qc, qs = oidx.quant_query_heads(q_idx[rows])
            lg = oidx.logits_fp8(qc, qs, w[rows], cache, pages, positions[rows])
        else:
            for pid, v in pools.items():
                pool_cache[oidx.pool_rows(pages, pid + 1)[pid]] = bf16(v)
            lg = oidx.logits(q_idx[rows], w[rows], pool_cache, pages, positions[rows])
        width = max((len(r) for r in lg), default=0)
        dense = np.full((n, max(width, 1)), -np.inf, np.float32)
        for i, r in enumerate(lg):
            dense[i, :len(r)] = r
        ke = (positions[rows] + 1) // 4
        ids = otopk.canonical_topk(dense, np.zeros(n, np.int64), ke, 512)
        tok = oidx.expand(ids, positions[rows], 512)
        out_lat[rows] = omla.sparse_mla(q8[rows], kv_cache, tok, pages, p["scale"] * p["q_scale"] * p["k_scale"],
                                        p["k_scale"], p_fp8=True)
    o_lat = bf16(out_lat)
    v = bf16(od.grouped_linear_bf16(o_lat.transpose(1, 0, 2), *p["w_uv"]))                      # [64, T, v_dim]
    o_in = v.transpose(1, 0, 2).reshape(T, NH * v_dim)
    return bf16(lin(o_in, p["o_proj"]))


def layer_forward(L: dict, st: list, chunks: list, res, x_prev, post, comb, gs_x: float, gs_h: float):
    """One decoder layer: boundary A (pre only when x_prev is None, else post of x_prev + pre) -> attention ->
    boundary B -> FFN. res [T, 4, H]; the layer's states `st` are updated in place. Returns (res after boundary B,
    the FFN rows, post, comb) -- the next layer's inputs, as the device layer returns them."""
    qsl = np.concatenate([[0], np.cumsum([c["n"] for c in chunks])]).astype(np.int64)
    positions = np.concatenate([np.arange(c["start"], c["start"] + c["n"]) for c in chunks]).astype(np.int64)
    if x_prev is None:
        post_a, comb_a, y = omhc.pre(res, *L["bound_a"])
    else:
        res, post_a, comb_a, y = omhc.post_pre(x_prev, res, post, comb, *L["bound_a"])
    a = L["attn"]
    if L["kind"] == "kda":
        g = L["group"]
        seqs = [(int(qsl[r]), int(qsl[r + 1]), int(c["state_blocks"][g]), int(c["start"] > 0))
                for r, c in enumerate(chunks)]
        x_a, cst, rst = ok.attention_block(y, a, st[0], st[1], seqs, a["heads"], gs_x, a["eps"])
        st[0][...] = cst
        st[1][...] = rst
    else:
        reqs = [(int(qsl[r]), c["n"], c["start"], np.asarray(c["pages"], np.int64), int(c["state_blocks"][5]))
                for r, c in enumerate(chunks)]
        x_a = dsa_block(y, a, positions, reqs, st[0], st[1], st[2], gs_x)
    res, post, comb, y = omhc.post_pre(x_a, res, post_a, comb_a, *L["bound_b"])
    f = L["ffn"]
    if f["kind"] == "moe":
        x_b = bf16(omoe.moe_forward(y, f["p"], f["k"], dense="lazy"))
    else:
        x_b = dense_ffn(y, f["w"], gs_x, gs_h)
    return res, x_b, post, comb


def head(params: dict, chunks: list, res):
    """The last stage's head on the final residual: (logits of the is_last chunks' last rows in row order, argmax)."""
    qsl = np.cumsum([c["n"] for c in chunks])
    rows = [int(qsl[r]) - 1 for r, c in enumerate(chunks) if c["is_last"]]
    h = params["head"]
    if not rows:
        return np.zeros((0, h["w"].shape[0]), np.float32), np.zeros(0, np.int64)
    merged = bf16(res[rows].astype(np.float32).sum(axis=1, dtype=np.float32) * np.float32(0.25))
    normed = bf16(ostage.rmsnorm(merged, h["norm_w"], h["eps"]))
    logits = (normed.astype(np.float64) @ np.asarray(h["w"], np.float64).T).astype(np.float32)
    return logits, ostage.argmax_lowest(logits)


def stage_forward(params: dict, chunks: list, hidden_in, states: list, gs_x: float, gs_h: float, *,
                  first: bool, last: bool):
    """One stage over chunks in ROW order (dicts: start, n, pages, state_blocks, token_ids (stage 0), is_last).

    params: "embed" [V, H] (stage 0), "layers": list of {"kind": "kda" | "dsa", "bound_a", "bound_b" (omhc.pre
    argument tuples after `res`), "attn" (KDA: oracle/kda.attention_block's p plus "heads", "eps"; DSA: dsa_block's
    p), "group" (KDA state group), "ffn": {"kind": "moe", "p", "k"} | {"kind": "dense", "w"}}, "head" (last stage:
    w [V, H] bf16 values, norm_w, eps).
    states: per layer, KDA (conv_state, rec_state) or DSA (kv_cache, pool_cache, tail); updated in place.
    Returns (out, residuals): out = the stage's [T, 4, H] rows (bf16 values) or, on the last stage, (logits of the
    is_last chunks' last rows in row order, their argmax); residuals = each layer's residual after its attention
    sub-block's post (the boundary B residual) and the stage's final residual."""
    T = sum(c["n"] for c in chunks)
    if first:
        tok = np.concatenate([np.asarray(c["token_ids"], np.int64) for c in chunks])
        x0 = np.asarray(params["embed"], np.float32)[tok]
        res = np.repeat(x0[:, None, :], 4, axis=1)
    else:
        res = np.asarray(hidden_in, np.float32).reshape(T, 4, -1)
    x_prev = post = comb = None
    residuals = []
    for L, st in zip(params["layers"], states):
        res, x_prev, post, comb = layer_forward(L, st, chunks, res, x_prev, post, comb, gs_x, gs_h)
        residuals.append(res.copy())
    if x_prev is not None:
        res = omhc.post(x_prev, res, post, comb)
    residuals.append(res.copy())
    if not last:
        return res, residuals
    return head(params, chunks, res), residuals
