"""The oracle's DSA block (oracle/model.py `dsa_block`) through its FP8 indexer branch against its bf16 branch, on
the CPU. Over at most 512 pools a row the canonical top-512 keeps every pool whatever the logits, so the two branches
must give the same attention output bit for bit, leave the same latent cache and tail ring, and store the same pool
keys up to each pool's e4m3 rounding (the reference's 132-byte entries against bf16 rows). This holds the FP8 branch's
plumbing (pool pages, query scales, the per-request loop) to the branch the GPU stage tests already pinned."""

import numpy as np
import pytest
import torch

from oracle import indexer as oidx
from oracle import model as omodel
from oracle.mhc import bf16
from oracle.mla import e4m3_decode

import __graft_entry__

__graft_entry__.import_package()
from ssengine_b200 import weights  # noqa: E402


def _params(fp8: bool):
    g = torch.Generator().manual_seed(4)
    rng = np.random.default_rng(4)

    def lin(N, K):
        c, s, gs = weights.nvfp4_tensor(g, N, K, "cpu")
        return c.numpy(), s.numpy(), gs

    ql, nope, vd, H = 256, 64, 256, 256
    return dict(a_proj=lin(ql + 576, H), q_b=lin(64 * (nope + 64), ql), wq_idx=lin(4096, ql), idx_proj=lin(288, H),
                o_proj=lin(H, 64 * vd), w_uk=(bf16(rng.standard_normal((64, 512, nope)) / nope ** 0.5),),
                w_uv=(bf16(rng.standard_normal((64, vd, 512)) / 512 ** 0.5),), q_norm=np.ones(ql),
                kv_norm=np.ones(512), ape=rng.standard_normal((4, 128)) * 0.5, q_lora=ql, nope=nope, v_dim=vd,
                theta=10000.0, eps=1e-6, scale=(nope + 64) ** -0.5, q_scale=1.0, k_scale=1.0, indexer_fp8=fp8)


@pytest.mark.parametrize("reqs", [[(0, 300, 0)], [(0, 70, 0), (70, 45, 130), (115, 1, 301)]])
def test_fp8_branch_equals_the_bf16_branch_when_every_pool_is_kept(reqs):
    """reqs: (first row, rows, start position); a request starting past 0 reads the pools and tail ring left by a
    first pass over its earlier tokens (the same on both branches)."""
    rng = np.random.default_rng(9)
    T = sum(n for _, n, _ in reqs)
    y = bf16(rng.standard_normal((T, 256)))
    positions = np.concatenate([np.arange(s, s + n) for _, n, s in reqs])
    pages = [np.arange(67 + 4 * r, 67 + 4 * r + 4) for r in range(len(reqs))]
    blocks = 4
    pre = [(r, s) for r, (_, _, s) in enumerate(reqs) if s > 0]
    y_pre = bf16(rng.standard_normal((sum(s for _, s in pre), 256)))
    out, caches = {}, {}
    for fp8 in (False, True):
        p = _params(fp8)
        kv = np.zeros((blocks * 67 * 128, 576), np.uint8)
        pool = (np.zeros((blocks * 67 * 33, 128), np.uint8) if fp8 else
                np.zeros((blocks * 67 * 32, 128), np.float32))
        tail = np.zeros((blocks, 2, 4, 128), np.float32)
        # earlier tokens of the requests that start past 0 (their own pass, so that the caches hold a prefix)
        if pre:
            at, preq = 0, []
            for r, s in pre:
                preq.append((at, s, 0, pages[r], 1 + r))
                at += s
            omodel.dsa_block(y_pre, p, np.concatenate([np.arange(s) for _, s in pre]), preq, kv, pool, tail,
                             weights.GS_X)
        rq = [(f, n, s, pages[r], 1 + r) for r, (f, n, s) in enumerate(reqs)]
        out[fp8] = omodel.dsa_block(y, p, positions, rq, kv, pool, tail, weights.GS_X)
        caches[fp8] = (kv, pool, tail)
    assert all(((positions + 1) // 4) <= 512)
    np.testing.assert_array_equal(out[True], out[False])
    np.testing.assert_array_equal(caches[True][0], caches[False][0])            # latent cache bytes
    np.testing.assert_array_equal(caches[True][2], caches[False][2])            # tail ring
    # every written bf16 pool row against its e4m3 codes x scale in the 132-byte entries
    p16 = caches[False][1]
    rows = np.flatnonzero(np.abs(p16).sum(axis=1) > 0)
    assert len(rows) >= 70
    codes, scales = oidx.read_pool_pages(caches[True][1].reshape(-1, 33 * 128), rows)
    vals = e4m3_decode(codes) * scales[:, None]
    ref = p16[rows].astype(np.float64)
    assert (np.abs(vals - ref) <= 2.0 ** -4 * np.abs(ref) + scales[:, None] * 2.0 ** -9 + 1e-12).all()
