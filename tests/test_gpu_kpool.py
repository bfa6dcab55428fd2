"""GPU parity of the indexer key pools (`ssb_kpool_insert`): two requests prefilled in chunkings that start inside
pools, chunks shorter than a pool and two requests in one microbatch write bit-identical pools to the unsplit prefill
(the reference's property, tests/test_kpool_cpu.py:95-122) and match the oracle (oracle/kpool.py) within one bf16
rounding step (fp32 softmax and sum on the GPU vs float64)."""

import numpy as np
import pytest
import torch

from oracle import kpool as okp

pytestmark = pytest.mark.gpu

D = 128
LENS = [300, 130]
PAGES = [[7, 2, 9], [4, 11]]          # request r's KV pages = pool pages (32 pools each)


def run(cuda, schedule, k_all, g_all, ape):
    from ssengine_b200 import indexer

    pool = torch.zeros(12 * 32, D, dtype=torch.bfloat16, device=cuda)
    ring = torch.zeros(4, 2, 4, D, dtype=torch.bfloat16, device=cuda)
    table = torch.tensor([[7, 2, 9], [4, 11, -1]], dtype=torch.int32, device=cuda)
    apd = torch.from_numpy(ape.astype(np.float32)).to(cuda)
    for mb in schedule:                                     # [(request, start, rows)]
        ks, gs, reqs, at = [], [], [], 0
        for r, s, n in mb:
            ks.append(k_all[r][s:s + n]); gs.append(g_all[r][s:s + n])
            reqs.append((at, n, s, r + 1))
            at += n
        k = torch.from_numpy(np.concatenate(ks)).to(torch.bfloat16).to(cuda)
        g = torch.from_numpy(np.concatenate(gs)).to(torch.bfloat16).to(cuda)
        rq = torch.tensor(reqs, dtype=torch.int32, device=cuda)
        tab = table[[r for r, _, _ in mb]].contiguous()
        indexer.kpool_insert(k, g, apd, rq, max(n for _, _, n in mb), tab, pool, ring)
    torch.cuda.synchronize()
    return pool.float().cpu().numpy()


def pools_of(cache, r):
    n = LENS[r] // 4
    p = np.arange(n)
    return cache[np.asarray(PAGES[r])[p // 32] * 32 + p % 32]


def test_chunkings_write_the_unsplit_pools(cuda):
    rng = np.random.default_rng(0)
    k_all = [rng.standard_normal((L, D)).astype(np.float32) for L in LENS]
    g_all = [rng.standard_normal((L, D)).astype(np.float32) for L in LENS]
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    k_all, g_all = [bf(a) for a in k_all], [bf(a) for a in g_all]
    ape = rng.standard_normal((4, D)).astype(np.float32)
    whole = run(cuda, [[(0, 0, 300)], [(1, 0, 130)]], k_all, g_all, ape)
    sched = [[(1, 0, 13)], [(0, 0, 37), (1, 13, 2)], [(1, 15, 50), (0, 37, 1)], [(0, 38, 200), (1, 65, 65)],
             [(0, 238, 62)]]
    split = run(cuda, sched, k_all, g_all, ape)
    for r in range(2):
        np.testing.assert_array_equal(pools_of(split, r), pools_of(whole, r))
        want = okp.unsplit(k_all[r], g_all[r], ape)
        got = pools_of(whole, r)
        w = np.stack([want[p] for p in range(len(want))])
        assert (np.abs(got - w) <= np.abs(w) * 2.0 ** -7 + 1e-6).all()
