"""GPU parity of the DSA indexer path against the oracle (oracle/indexer.py, oracle/topk.py): pool logits over paged
pool keys (`ssb_indexer_logits`) for several requests with prefixes (one query group spans several 128-pool tiles and
pages in shuffled order), the canonical top-k of those logits over each row's visible pools, and the pool -> token
expansion (`ssb_indexer_expand`).

Tolerances: logits within 2e-3 of each row's largest magnitude (bf16 products summed in fp32 on the tensor cores vs
float64); top-k index sets and the expansion bit-exact (the top-k is compared on the GPU's own logits)."""

import numpy as np
import pytest
import torch

from oracle import indexer as oidx
from oracle import topk as otopk

pytestmark = pytest.mark.gpu

REQS = [(0, 50), (37, 13), (300, 70), (1400, 21), (3, 1)]       # (position of the first query row, query rows)


def setup(cuda, seed=0):
    rng = np.random.default_rng(seed)
    T = sum(n for _, n in REQS)
    q_starts = np.cumsum([0] + [n for _, n in REQS])[:-1]
    positions = np.concatenate([np.arange(s, s + n) for s, n in REQS]).astype(np.int64)
    n_pages = [-(-(s + n) // 128) for s, n in REQS]
    perm = rng.permutation(sum(n_pages) + 3) + 1              # shuffled page ids, page 0 unused
    width = max(n_pages) + 2
    table = np.full((len(REQS), width), -1, np.int32)
    at = 0
    for r, n in enumerate(n_pages):
        table[r, :n] = perm[at:at + n]
        at += n
    rows = (perm.max() + 1) * 32
    q = rng.standard_normal((T, 32, 128)).astype(np.float32)
    k = rng.standard_normal((rows, 128)).astype(np.float32)
    w = rng.uniform(-1, 1, (T, 32)).astype(np.float32)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(cuda)
    w = bf(w).float().cpu().numpy()                          # the head weights arrive as bf16
    dev = dict(q=bf(q), k=bf(k), w=bf(w), table=torch.from_numpy(table).to(cuda),
               pos=torch.from_numpy(positions).to(cuda))
    host = dict(q=dev["q"].float().cpu().numpy(), k=dev["k"].float().cpu().numpy(), w=w, table=table,
                pos=positions, q_starts=q_starts)
    return T, dev, host


def test_logits_topk_expand(cuda):
    from ssengine_b200 import indexer

    T, dev, host = setup(cuda)
    groups = indexer.work_groups(host["q_starts"], [n for _, n in REQS], [s for s, _ in REQS])
    assert groups[:, 3].max() >= 3                            # a group over several pool tiles
    ldl = 512
    out = torch.full((T, ldl), float("nan"), dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    indexer.logits(dev["q"], dev["w"], dev["k"], dev["table"], torch.from_numpy(groups).to(cuda), out, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    got = out.cpu().numpy()
    for r, ((s, n), qs) in enumerate(zip(REQS, host["q_starts"])):
        sl = slice(qs, qs + n)
        want = oidx.logits(host["q"][sl], host["w"][sl], host["k"], host["table"][r], host["pos"][sl])
        for i, wr in enumerate(want):
            if len(wr) == 0:
                continue
            g = got[qs + i, :len(wr)]
            assert np.isfinite(g).all()
            scale = max(np.abs(wr).max(), 1e-6)
            assert np.abs(g - wr).max() <= 2e-3 * scale, (r, i, np.abs(g - wr).max(), scale)

    k = 16
    ids = torch.full((T, k), -7, dtype=torch.int32, device=cuda)
    indexer.topk(out, dev["pos"], k, ids)
    torch.cuda.synchronize()
    ke = (host["pos"] + 1) // 4
    want_ids = otopk.canonical_topk(got, np.zeros(T, np.int64), ke, k)
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids)

    tok = torch.full((T, 4 * k + 3), -9, dtype=torch.int32, device=cuda)
    indexer.expand(ids, dev["pos"], tok)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), oidx.expand(want_ids, host["pos"], k))
