"""GPU parity of the sparse MLA prefill (`ssb_sparse_mla`) and the latent-cache append (`ssb_mla_cache_append`)
against the oracle (oracle/mla.py): several requests over paged caches in shuffled page order, ragged selections
(-1 padding, rows with one token, rows with none), selections longer than one 32-token block.

Tolerances: outputs within 1e-2 relative L2 per row (bf16 probabilities and values on the tensor cores, fp32
accumulation, vs float64); rows with no token are zeros; the cache append is bit-exact."""

import numpy as np
import pytest
import torch

from oracle import mla as omla

pytestmark = pytest.mark.gpu

REQS = [(0, 40), (500, 17), (2000, 9)]          # (position of the first query row, rows)
NIDX = 200
SCALE = 192 ** -0.5


def test_sparse_mla_matches_oracle(cuda):
    from ssengine_b200 import mla

    rng = np.random.default_rng(3)
    T = sum(n for _, n in REQS)
    qsl = np.cumsum([0] + [n for _, n in REQS]).astype(np.int32)
    n_pages = [-(-(s + n) // 128) for s, n in REQS]
    perm = rng.permutation(sum(n_pages) + 2) + 1
    width = max(n_pages)
    table = np.full((len(REQS), width), -1, np.int32)
    at = 0
    for r, n in enumerate(n_pages):
        table[r, :n] = perm[at:at + n]
        at += n
    slots = (perm.max() + 1) * 128
    kv = rng.standard_normal((slots, 576)).astype(np.float32)
    q = rng.standard_normal((T, 64, 576)).astype(np.float32)
    idx = np.full((T, NIDX + 24), -1, np.int32)
    row = 0
    for s, n in REQS:
        for i in range(n):
            pos = s + i
            m = [NIDX, 1, 0, 37][row % 4] if row % 5 else min(NIDX, pos + 1)
            m = min(m, pos + 1)
            sel = rng.choice(pos + 1, size=m, replace=False) if m else np.zeros(0, int)
            cols = rng.permutation(NIDX)[:m]
            idx[row, cols] = sel
            row += 1
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(cuda)
    qd, kvd = bf(q), bf(kv)
    out = torch.full((T, 64, 512), float("nan"), dtype=torch.bfloat16, device=cuda)
    mla.sparse_mla(qd, kvd, torch.from_numpy(idx).to(cuda), torch.from_numpy(qsl).to(cuda),
                   torch.from_numpy(table).to(cuda), SCALE, out, n_idx=NIDX)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    qh, kvh = qd.float().cpu().numpy(), kvd.float().cpu().numpy()
    for r, (s, n) in enumerate(REQS):
        sl = slice(qsl[r], qsl[r + 1])
        want = omla.sparse_mla(qh[sl], kvh, idx[sl, :NIDX], table[r], SCALE)
        for i in range(n):
            g, w = got[qsl[r] + i], want[i]
            if not (idx[qsl[r] + i, :NIDX] >= 0).any():
                assert not g.any()
                continue
            assert np.linalg.norm(g - w) / np.linalg.norm(w) < 1e-2, (r, i, np.linalg.norm(g - w) / np.linalg.norm(w))


def test_cache_append(cuda):
    from ssengine_b200 import mla

    rng = np.random.default_rng(4)
    src = torch.from_numpy(rng.standard_normal((50, 584)).astype(np.float32)).to(torch.bfloat16).to(cuda)
    slots = torch.from_numpy(rng.permutation(300)[:50].astype(np.int64)).to(cuda)
    slots[7] = -1
    cache = torch.zeros(300, 576, dtype=torch.bfloat16, device=cuda)
    mla.cache_append(src, slots, cache)
    torch.cuda.synchronize()
    c, s, x = cache.cpu(), slots.cpu(), src[:, :576].cpu()
    for t in range(50):
        if s[t] >= 0:
            assert torch.equal(c[s[t]], x[t])
    assert int((c.abs().sum(1) > 0).sum()) == 49


def test_sparse_mla_expanded_layout(cuda):
    """The indexer's expanded layout at the full width (512 pools x 4 tokens + 3 tail columns): pool tokens first,
    -1 padding up to column 2048, the incomplete pool's tokens after it. Rows near a request's start select a few
    blocks of columns (one holding only tail tokens), long rows all 33; a page missing from the table drops its
    tokens."""
    from ssengine_b200 import mla

    rng = np.random.default_rng(5)
    K, n_idx = 512, 4 * 512 + 3
    positions = [0, 2, 3, 6, 70, 1000, 2046, 2100, 5000, 9001]
    T = len(positions)
    width = max(positions) // 128 + 1
    table = (rng.permutation(width + 3)[:width] + 1).astype(np.int32)[None, :]
    table[0, 3] = -1                                               # tokens 384-511 unreadable
    slots = (int(table.max()) + 1) * 128
    kv = rng.standard_normal((slots, 576)).astype(np.float32)
    q = rng.standard_normal((T, 64, 576)).astype(np.float32)
    idx = np.full((T, n_idx), -1, np.int32)
    for r, pos in enumerate(positions):
        n_pools = (pos + 1) // 4
        pools = np.sort(rng.choice(n_pools, size=min(K, n_pools), replace=False)) if n_pools else np.zeros(0, int)
        for i, p in enumerate(pools):
            idx[r, 4 * i:4 * i + 4] = 4 * p + np.arange(4)
        tail0 = ((pos + 1) // 4) * 4
        idx[r, 4 * K:4 * K + (pos + 1 - tail0)] = np.arange(tail0, pos + 1)
    qsl = np.array([0, T], np.int32)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(cuda)
    qd, kvd = bf(q), bf(kv)
    out = torch.full((T, 64, 512), float("nan"), dtype=torch.bfloat16, device=cuda)
    mla.sparse_mla(qd, kvd, torch.from_numpy(idx).to(cuda), torch.from_numpy(qsl).to(cuda),
                   torch.from_numpy(table).to(cuda), SCALE, out, n_idx=n_idx)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    want = omla.sparse_mla(qd.float().cpu().numpy(), kvd.float().cpu().numpy(), idx, table[0], SCALE)
    for r in range(T):
        err = np.linalg.norm(got[r] - want[r]) / np.linalg.norm(want[r])
        assert err < 1e-2, (positions[r], err)
