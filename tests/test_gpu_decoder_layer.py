"""GPU parity of one KDA + MoE decoder layer on the 4-stream residual (`layers.KdaDecoderLayer`: mHC boundary ->
KDA attention block -> mHC boundary -> NVFP4 MoE) against the oracle's composition (oracle/mhc.py, oracle/kda.py,
oracle/moe.py), entered with a previous sub-block's rows (post + pre boundary) and as a stage's first layer (pre only).

Tolerances: the residual stream after each boundary within 3e-2 relative L2 (the per-layer hidden-state bar); the MoE
rows within 3e-2 of the oracle's MoE on the device's own layer input (NVFP4 requantization of the chain's inputs
makes whole-chain comparisons of sub-block outputs looser, see tests/test_gpu_kda_block.py)."""

import numpy as np
import pytest
import torch

from oracle import kda as ok
from oracle import mhc as omhc
from oracle import moe as omoe

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def pre_args(b):
    n = lambda t: t.float().cpu().numpy()
    e = b.eps
    return (n(b.fn), n(b.scale), n(b.base), e["rms_eps"], e["pre_eps"], e["sinkhorn_eps"], e["post_mult"], b.repeat,
            n(b.norm_w), e["norm_eps"])


@pytest.mark.parametrize("first", [False, True])
def test_decoder_layer(cuda, first):
    from ssengine_b200 import weights
    from ssengine_b200.kda import seq_table
    from ssengine_b200.layers import KdaDecoderLayer

    H, heads, F, E, k, T = 512, 2, 256, 16, 4, 130
    P = heads * 128
    layer = KdaDecoderLayer(21, H, heads, F, E, k, cuda)
    rng = np.random.default_rng(5)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).to(cuda)
    f32 = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(cuda)
    res = bf(rng.standard_normal((T, 4, H)))
    x_prev = None if first else bf(rng.standard_normal((T, H)))
    post_prev = None if first else f32(rng.uniform(0.2, 2.0, (T, 4)))
    comb = rng.uniform(0, 1, (T, 4, 4))
    comb_prev = None if first else f32(comb / comb.sum(1, keepdims=True))
    seqs = [(0, 70, 1, 1), (70, 130, 2, 0)]
    cst = bf(rng.standard_normal((3, 3, 3 * P)))
    rst = f32(rng.standard_normal((3, heads, 128, 128)) * 0.05)
    n = lambda t: t.float().cpu().numpy()
    res0, cst0, rst0 = n(res), n(cst), rst.cpu().numpy()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    res_b, x_b, post_b, comb_b = layer.forward(res, x_prev, post_prev, comb_prev, seq_table(seqs, cuda), cst, rst,
                                               status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0 and int(layer.moe.status[0]) == 0

    # oracle chain
    if first:
        res_a = res0
        post_a, comb_a, y_a = omhc.pre(res_a, *pre_args(layer.bound_a))
    else:
        res_a, post_a, comb_a, y_a = omhc.post_pre(n(x_prev), res0, n(post_prev), n(comb_prev), *pre_args(layer.bound_a))
    blk = layer.attn
    p = {name: tuple(v.cpu().numpy() if torch.is_tensor(v) else v for v in getattr(blk, name).logical())
         for name in ("in_proj", "f_b", "g_b", "o_proj")}
    p.update(conv_w=n(blk.kda.conv_weight), a_log=n(blk.kda.a_log), dt_bias=n(blk.kda.dt_bias), norm_w=n(blk.norm_w))
    x_a, _, _ = ok.attention_block(y_a, p, cst0, rst0, seqs, heads, weights.GS_X, blk.norm_eps)
    res_bw, post_bw, comb_bw, y_b = omhc.post_pre(x_a, res_a, post_a, comb_a, *pre_args(layer.bound_b))
    assert rel(n(res_b), res_bw) < 3e-2, rel(n(res_b), res_bw)
    # the MoE rows against the oracle's MoE on the device's own FFN input (the boundary's y, recomputed from res_b)
    _, _, y_dev = omhc.pre(n(res_b), *pre_args(layer.bound_b))
    want = omoe.moe_forward(y_dev, layer.moe.logical(), k)
    assert rel(n(x_b), want) < 3e-2, rel(n(x_b), want)
