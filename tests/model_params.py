"""Test helper (not a test module): a StageModel's parameters and states read out of its device objects into the
numpy form oracle/model.py takes."""

from __future__ import annotations

import numpy as np
import torch


def _n(t):
    return t.float().cpu().numpy() if torch.is_tensor(t) else t


def _lin(L):
    return tuple(_n(v) if torch.is_tensor(v) and v.is_floating_point() else v.cpu().numpy() if torch.is_tensor(v)
                 else v for v in L.logical())


def bound_args(b):
    e = b.eps
    return (_n(b.fn), _n(b.scale), _n(b.base), e["rms_eps"], e["pre_eps"], e["sinkhorn_eps"], e["post_mult"], b.repeat,
            _n(b.norm_w), e["norm_eps"])


def stage_params(stage) -> dict:
    from ssengine_b200.layers import DenseFfn

    out = {"layers": []}
    for layer, i, dsa in zip(stage.layers, stage.layer_range, stage.is_dsa):
        blk = layer.attn
        if dsa:
            attn = {name: _lin(getattr(blk, name)) for name in ("a_proj", "q_b", "wq_idx", "idx_proj", "o_proj",
                                                                 "w_uk", "w_uv")}
            attn.update(q_norm=_n(blk.q_norm), kv_norm=_n(blk.kv_norm), ape=blk.ape.cpu().numpy(),
                        q_lora=blk.q_lora, nope=blk.nope, v_dim=blk.v_dim, theta=blk.theta, eps=blk.eps,
                        scale=blk.scale, q_scale=blk.q_scale, k_scale=blk.k_scale,
                        indexer_fp8=getattr(blk, "indexer_fp8", False))
        else:
            attn = {name: _lin(getattr(blk, name)) for name in ("in_proj", "f_b", "g_b", "o_proj")}
            attn.update(conv_w=_n(blk.kda.conv_weight), a_log=_n(blk.kda.a_log), dt_bias=_n(blk.kda.dt_bias),
                        norm_w=_n(blk.norm_w), heads=blk.heads, eps=blk.norm_eps)
        f = layer.ffn
        if isinstance(f, DenseFfn):
            ffn = {"kind": "dense", "w": tuple(v.cpu().numpy() if torch.is_tensor(v) else v for v in f.logical())}
        else:
            ffn = {"kind": "moe", "p": f.logical(), "k": f.k}
        out["layers"].append({"kind": "dsa" if dsa else "kda", "bound_a": bound_args(layer.bound_a),
                              "bound_b": bound_args(layer.bound_b), "attn": attn, "ffn": ffn,
                              "group": None if dsa else stage.kv.group[i]})
    if stage.first:
        out["embed"] = _n(stage.embed)
    if stage.last:
        out["head"] = {"w": _n(stage.head_w), "norm_w": _n(stage.norm_weight), "eps": stage.cfg.norm_eps}
    return out


def stage_states(stage) -> list:
    """Host copies of each layer's states (KDA: conv, recurrent; DSA: latent cache bytes, pool keys, tail ring)."""
    out = []
    for st, dsa in zip(stage.kda_states, stage.is_dsa):
        if dsa:                                   # an FP8 pool cache (uint8 pages) is kept as its bytes
            pools = st[1].cpu().numpy().copy() if st[1].dtype == torch.uint8 else _n(st[1]).copy()
            out.append([st[0].cpu().numpy().copy(), pools, _n(st[2]).copy()])
        else:
            out.append([_n(st[0]).copy(), st[1].cpu().numpy().copy()])
    return out


def row_chunks(plan) -> list:
    """The plan's chunks in the stage's row order, as oracle/model.stage_forward takes them."""
    from ssengine_b200.stage import row_order

    order = row_order([c.num_tokens for c in plan.chunks])
    return [dict(start=c.start, n=c.num_tokens, pages=list(c.kv_pages), state_blocks=list(c.state_blocks),
                 token_ids=c.token_ids, is_last=c.is_last) for c in (plan.chunks[i] for i in order)], order
