"""GPU parity of the FP8 sparse MLA prefill (`ssb_sparse_mla`), the FP8 latent-cache append (`ssb_mla_cache_append`)
and the FP8 query pack (`ssb_mla_q_pack`) against the oracle (oracle/mla.py): several requests over paged caches in
shuffled page order, ragged selections (-1 padding, rows with one token, rows with none), selections over several
128-column blocks with empty blocks between them, the indexer's full-width expanded layout, non-unit q / k scales.

Tolerances: outputs within 3e-2 relative L2 per row of the float64 attention over the same e4m3 query and cache
bytes (the softmax weights enter the P.V product as e4m3, as in the reference's FP8 kernel: ~1.5e-2 measured on the
CPU model of that rounding), and within 8e-3 of the oracle that rounds them at the same point
(oracle/mla.sparse_mla_fp8p); rows with no token are zeros; the cache append and the query pack bit-exact."""

import numpy as np
import pytest
import torch

from oracle import mla as omla

pytestmark = pytest.mark.gpu

REQS = [(0, 40), (500, 17), (2000, 9)]          # (position of the first query row, rows)
NIDX = 600
SCALE = 192 ** -0.5
TOL = 3e-2
TOL_FP8P = 8e-3       # against the oracle that rounds the softmax weights where the kernel does (sparse_mla_fp8p)


def _paged(rng, reqs):
    n_pages = [-(-(s + n) // 128) for s, n in reqs]
    perm = rng.permutation(sum(n_pages) + 2) + 1
    table = np.full((len(reqs), max(n_pages)), -1, np.int32)
    at = 0
    for r, n in enumerate(n_pages):
        table[r, :n] = perm[at:at + n]
        at += n
    return table, (int(perm.max()) + 1) * 128


def _run(cuda, q8, kv8, idx, qsl, table, bmm1, bmm2, n_idx):
    from ssengine_b200 import mla

    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out = torch.full((q8.shape[0], 64, 512), float("nan"), dtype=torch.bfloat16, device=cuda)
    mla.sparse_mla(u8(q8), u8(kv8), u8(idx), u8(qsl), u8(table), bmm1, out, bmm2=bmm2, n_idx=n_idx)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("q_scale,k_scale", [(1.0, 1.0), (4.0, 0.5)])
def test_sparse_mla_matches_oracle(cuda, q_scale, k_scale):
    rng = np.random.default_rng(3)
    T = sum(n for _, n in REQS)
    qsl = np.cumsum([0] + [n for _, n in REQS]).astype(np.int32)
    table, slots = _paged(rng, REQS)
    kv8 = omla.quantize(rng.standard_normal((slots, 576)).astype(np.float32) * k_scale, k_scale)
    q8 = omla.quantize(rng.standard_normal((T, 64, 576)).astype(np.float32) * q_scale, q_scale)
    idx = np.full((T, NIDX + 24), -1, np.int32)
    row = 0
    for s, n in REQS:
        for i in range(n):
            pos = s + i
            m = [NIDX, 1, 0, 37][row % 4] if row % 5 else min(NIDX, pos + 1)
            m = min(m, pos + 1)
            sel = rng.choice(pos + 1, size=m, replace=False) if m else np.zeros(0, int)
            if row % 3 == 0 and m <= 128:
                cols = rng.permutation(128)[:m] + 384              # one block, the blocks before it empty
            else:
                cols = rng.permutation(NIDX)[:m]
            idx[row, cols] = sel
            row += 1
    bmm1, bmm2 = SCALE * q_scale * k_scale, k_scale
    got = _run(cuda, q8, kv8, idx, qsl, table, bmm1, bmm2, NIDX)
    for r, (s, n) in enumerate(REQS):
        sl = slice(qsl[r], qsl[r + 1])
        want = omla.sparse_mla(q8[sl], kv8, idx[sl, :NIDX], table[r], bmm1, bmm2)
        want8 = omla.sparse_mla(q8[sl], kv8, idx[sl, :NIDX], table[r], bmm1, bmm2, p_fp8=True)
        for i in range(n):
            g, w = got[qsl[r] + i], want[i]
            if not (idx[qsl[r] + i, :NIDX] >= 0).any():
                assert not g.any()
                continue
            err = np.linalg.norm(g - w) / np.linalg.norm(w)
            assert err < TOL, (r, i, err)
            err8 = np.linalg.norm(g - want8[i]) / np.linalg.norm(want8[i])
            assert err8 < TOL_FP8P, (r, i, err8)


def test_sparse_mla_expanded_layout(cuda):
    """The indexer's expanded layout at the full width (512 pools x 4 tokens + 3 tail columns): pool tokens first,
    -1 padding up to column 2048, the incomplete pool's tokens after it. Rows near a request's start select a few
    blocks of columns (one holding only tail tokens), long rows all 17; a page missing from the table drops its
    tokens."""
    rng = np.random.default_rng(5)
    K, n_idx = 512, 4 * 512 + 3
    positions = [0, 2, 3, 6, 70, 1000, 2046, 2100, 5000, 9001]
    T = len(positions)
    width = max(positions) // 128 + 1
    table = (rng.permutation(width + 3)[:width] + 1).astype(np.int32)[None, :]
    table[0, 3] = -1                                               # tokens 384-511 unreadable
    slots = (int(table.max()) + 1) * 128
    kv8 = omla.quantize(rng.standard_normal((slots, 576)).astype(np.float32), 1.0)
    q8 = omla.quantize(rng.standard_normal((T, 64, 576)).astype(np.float32), 1.0)
    idx = np.full((T, n_idx), -1, np.int32)
    for r, pos in enumerate(positions):
        n_pools = (pos + 1) // 4
        pools = np.sort(rng.choice(n_pools, size=min(K, n_pools), replace=False)) if n_pools else np.zeros(0, int)
        for i, p in enumerate(pools):
            idx[r, 4 * i:4 * i + 4] = 4 * p + np.arange(4)
        tail0 = ((pos + 1) // 4) * 4
        idx[r, 4 * K:4 * K + (pos + 1 - tail0)] = np.arange(tail0, pos + 1)
    qsl = np.array([0, T], np.int32)
    got = _run(cuda, q8, kv8, idx, qsl, table, SCALE, 1.0, n_idx)
    want = omla.sparse_mla(q8, kv8, idx, table[0], SCALE, 1.0)
    want8 = omla.sparse_mla(q8, kv8, idx, table[0], SCALE, 1.0, p_fp8=True)
    for r in range(T):
        err = np.linalg.norm(got[r] - want[r]) / np.linalg.norm(want[r])
        assert err < TOL, (positions[r], err)
        err8 = np.linalg.norm(got[r] - want8[r]) / np.linalg.norm(want8[r])
        assert err8 < TOL_FP8P, (positions[r], err8)


@pytest.mark.parametrize("k_scale", [1.0, 0.37])
def test_cache_append(cuda, k_scale):
    from ssengine_b200 import mla

    rng = np.random.default_rng(4)
    src_f = rng.standard_normal((50, 584)).astype(np.float32) * 60        # some values past 448 / k_scale saturate
    src = torch.from_numpy(src_f).to(torch.bfloat16).to(cuda)
    slots = torch.from_numpy(rng.permutation(300)[:50].astype(np.int64)).to(cuda)
    slots[7] = -1
    cache = torch.zeros(300, 576, dtype=torch.uint8, device=cuda)
    mla.cache_append(src, slots, cache, k_scale)
    torch.cuda.synchronize()
    c, s = cache.cpu().numpy(), slots.cpu().numpy()
    want = omla.quantize(src[:, :576].float().cpu().numpy(), k_scale)
    for t in range(50):
        if s[t] >= 0:
            np.testing.assert_array_equal(c[s[t]], want[t])
    assert int((c != 0).any(axis=1).sum()) == 49


def test_q_pack(cuda):
    from ssengine_b200 import mla

    rng = np.random.default_rng(6)
    T, Tp, qh = 37, 128, 256
    lat = torch.from_numpy(rng.standard_normal((64 * Tp, 512)).astype(np.float32) * 30).to(torch.bfloat16).to(cuda)
    q = torch.from_numpy(rng.standard_normal((T, 64 * qh)).astype(np.float32) * 30).to(torch.bfloat16).to(cuda)
    q8 = torch.zeros(T, 64, 576, dtype=torch.uint8, device=cuda)
    mla.q_pack(lat, Tp, q[:, 192:], qh, T, q8, 2.5)
    torch.cuda.synchronize()
    lat_h = lat.float().cpu().numpy().reshape(64, Tp, 512)[:, :T].transpose(1, 0, 2)
    rope = q.float().cpu().numpy().reshape(T, 64, qh)[:, :, 192:]
    want = omla.quantize(np.concatenate([lat_h, rope], axis=2), 2.5)
    np.testing.assert_array_equal(q8.cpu().numpy(), want)
