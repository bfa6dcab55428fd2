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
