"""GPU parity of the fused mHC layer boundary (`ssb_mhc`) against the oracle (oracle/mhc.py): post + pre (the
reference's `MegaMhcPostPre`), pre only (stage-edge receive), post only (stage-edge send); ragged token counts.
Tolerances: new residual within one bf16 rounding step; post and Sinkhorn mixes rtol 1e-3 (a 4H-long fp32 dot
product against the float64 oracle, then 20 Sinkhorn sweeps); layer input relative L2 1e-2."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import mhc as omhc

pytestmark = pytest.mark.gpu

EPS = dict(rms_eps=1e-6, pre_eps=1e-2, sinkhorn_eps=1e-6, post_mult=2.0, norm_eps=1e-6)
REPEAT = 20


def make(rng, T, H):
    x = omhc.bf16(rng.standard_normal((T, H)))
    res = omhc.bf16(rng.standard_normal((T, 4, H)))
    post_in = rng.uniform(0.2, 2.0, size=(T, 4)).astype(np.float32)
    comb_in = rng.uniform(0.0, 1.0, size=(T, 4, 4)).astype(np.float32)
    comb_in /= comb_in.sum(axis=1, keepdims=True)
    fn = (rng.standard_normal((24, 4 * H)) / np.sqrt(4 * H)).astype(np.float32)
    scale = np.array([0.8, 0.6, 1.5], dtype=np.float32)
    base = (rng.standard_normal(24) * 0.3).astype(np.float32)
    w = omhc.bf16(rng.uniform(0.5, 1.5, size=H))
    return x, res, post_in, comb_in, fn, scale, base, w


def run(cuda, T, H, args, post=True, pre=True):
    from ssengine_b200 import lib

    so = lib.load()
    x, res, post_in, comb_in, fn, scale, base, w = args
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(cuda)
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(cuda)
    keep = dict(x=bf(x), res=bf(res), pin=f32(post_in), cin=f32(comb_in), fn=f32(fn), scale=f32(scale), base=f32(base),
                w=bf(w))
    out = dict(nr=torch.zeros(T, 4, H, dtype=torch.bfloat16, device=cuda),
               po=torch.zeros(T, 4, dtype=torch.float32, device=cuda),
               co=torch.zeros(T, 4, 4, dtype=torch.float32, device=cuda),
               y=torch.zeros(T, H, dtype=torch.bfloat16, device=cuda))
    p = lib.MhcParamsC(H, 4, keep["fn"].data_ptr(), keep["scale"].data_ptr(), keep["base"].data_ptr(),
                       keep["w"].data_ptr(), EPS["rms_eps"], EPS["pre_eps"], EPS["sinkhorn_eps"], EPS["post_mult"],
                       EPS["norm_eps"], REPEAT)
    rc = so.ssb_mhc(ctypes.byref(p), keep["x"].data_ptr() if post else None, keep["res"].data_ptr(),
                    keep["pin"].data_ptr(), keep["cin"].data_ptr(), out["nr"].data_ptr(), out["po"].data_ptr(),
                    out["co"].data_ptr(), out["y"].data_ptr() if pre else None, T,
                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    lib.check("ssb_mhc", rc)
    torch.cuda.synchronize()
    return {k: v.float().cpu().numpy() for k, v in out.items()}


def pre_args(args):
    _, _, _, _, fn, scale, base, w = args
    return (fn, scale, base, EPS["rms_eps"], EPS["pre_eps"], EPS["sinkhorn_eps"], EPS["post_mult"], REPEAT, w,
            EPS["norm_eps"])


def close_bf16(got, want):
    # within one bf16 rounding step of the larger magnitude
    tol = np.maximum(np.abs(want), np.abs(got)) * 2.0 ** -7 + 1e-6
    assert (np.abs(got - want) <= tol).mean() > 0.999 and np.abs(got - want).max() <= 4 * tol.max()


@pytest.mark.parametrize("T,H", [(77, 256), (64, 4096), (1, 512)])
def test_post_pre_matches_oracle(cuda, T, H):
    args = make(np.random.default_rng(T + H), T, H)
    got = run(cuda, T, H, args)
    nr, po, co, y = omhc.post_pre(*args[:4], *pre_args(args))
    close_bf16(got["nr"], nr)
    np.testing.assert_allclose(got["po"], po, rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(got["co"], co, rtol=1e-3, atol=1e-4)
    assert np.linalg.norm(got["y"] - y) / np.linalg.norm(y) < 1e-2


def test_pre_only_and_post_only(cuda):
    T, H = 50, 1024
    args = make(np.random.default_rng(5), T, H)
    got = run(cuda, T, H, args, post=False)
    po, co, y = omhc.pre(args[1], *pre_args(args))
    np.testing.assert_allclose(got["po"], po, rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(got["co"], co, rtol=1e-3, atol=1e-4)
    assert np.linalg.norm(got["y"] - y) / np.linalg.norm(y) < 1e-2
    got2 = run(cuda, T, H, args, pre=False)
    close_bf16(got2["nr"], omhc.post(*args[:4]))
    assert not got2["y"].any()
