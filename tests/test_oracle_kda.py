"""CPU checks of the KDA oracle (oracle/kda.py): a request split into two chunks with the states carried through the
state blocks gives the same outputs and states as one call (the continuation contract of `kda_prefill_forward`,
ssengine/model/pp_patch.py:215-244, and of the conv state, ssengine/model/kda_conv.py:110-132); short sequences take
their conv rows from the old state; a fresh request ignores whatever its blocks held."""

import numpy as np

from oracle import kda as ok
from oracle.mhc import bf16

H, D = 2, 128
P = H * D


def inputs(rng, T):
    x = bf16(rng.standard_normal((T, 3 * P)))
    w = bf16(rng.uniform(-0.6, 0.6, (3 * P, 4)))
    g = bf16(rng.standard_normal((T, P)))
    beta = bf16(rng.standard_normal((T, H)))
    a_log = rng.uniform(-1, 1, H).astype(np.float32)
    dtb = (rng.standard_normal(P) * 0.5).astype(np.float32)
    return x, w, g, beta, a_log, dtb


def test_split_equals_whole():
    rng = np.random.default_rng(1)
    T, cut = 70, 29
    x, w, g, beta, a_log, dtb = inputs(rng, T)
    cst = bf16(rng.standard_normal((3, 3, 3 * P)))
    rst = (rng.standard_normal((3, H, D, D)) * 0.05).astype(np.float32)
    whole, c1, r1 = ok.prefill(x, w, cst, g, beta, a_log, dtb, -5.0, rst, [(0, T, 2, 1)], H, D)
    o_a, c2, r2 = ok.prefill(x[:cut], w, cst, g[:cut], beta[:cut], a_log, dtb, -5.0, rst, [(0, cut, 2, 1)], H, D)
    o_b, c3, r3 = ok.prefill(x[cut:], w, c2, g[cut:], beta[cut:], a_log, dtb, -5.0, r2, [(0, T - cut, 2, 1)], H, D)
    np.testing.assert_allclose(np.concatenate([o_a, o_b]), whole, rtol=1e-5, atol=1e-8)   # fp32 state between calls
    np.testing.assert_array_equal(c3, c1)
    np.testing.assert_allclose(r3, r1, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(r1[0], rst[0])          # other blocks untouched
    np.testing.assert_array_equal(c1[1], cst[1])


def test_short_sequence_conv_state_and_fresh_request():
    rng = np.random.default_rng(2)
    x, w, g, beta, a_log, dtb = inputs(rng, 4)
    cst = bf16(rng.standard_normal((2, 3, 3 * P)))
    _, _, _, st = ok.conv(x, w, cst, [(0, 1, 1, 1), (1, 4, 0, 0)], P)
    np.testing.assert_array_equal(st[1], np.concatenate([cst[1][1:], x[0:1, :3 * P]]))
    np.testing.assert_array_equal(st[0], x[1:4, :3 * P])
    q0, _, _, _ = ok.conv(x, w, cst, [(1, 4, 0, 0)], P)
    q1, _, _, _ = ok.conv(x, w, np.zeros_like(cst), [(1, 4, 0, 0)], P)
    np.testing.assert_array_equal(q0, q1)                 # fresh: the block's old rows are not read
    out0, _, r0 = ok.prefill(x, w, cst, g, beta, a_log, dtb, -5.0, np.ones((2, H, D, D), np.float32), [(0, 4, 1, 0)],
                             H, D)
    out1, _, r1 = ok.prefill(x, w, cst, g, beta, a_log, dtb, -5.0, np.zeros((2, H, D, D), np.float32), [(0, 4, 1, 0)],
                             H, D)
    np.testing.assert_array_equal(out0, out1)
    np.testing.assert_array_equal(r0[1], r1[1])
