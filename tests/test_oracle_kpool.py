"""CPU check of the kpool oracle (oracle/kpool.py): the reference's property (tests/test_kpool_cpu.py:95-101,
`test_any_chunking_writes_the_unsplit_pools`) -- a prompt prefilled in any chunking, including chunks that start inside
a pool and chunks shorter than a pool, writes the pools of the unsplit prefill."""

import numpy as np
import pytest

from oracle import kpool as okp


@pytest.mark.parametrize("cuts", [[1], [2], [3], [5, 6, 7], [9, 10, 23], [1, 2, 3, 4, 5, 6, 7, 30]])
def test_any_chunking_writes_the_unsplit_pools(cuts):
    rng = np.random.default_rng(0)
    L, D = 40, 8
    k = rng.standard_normal((L, D))
    g = rng.standard_normal((L, D))
    ape = rng.standard_normal((4, D))
    want = okp.unsplit(k, g, ape)
    pools, ring = {}, np.zeros((2, 4, D))
    bounds = [0, *cuts, L]
    for a, b in zip(bounds, bounds[1:]):
        okp.prefill_chunk(k[a:b], g[a:b], a, ape, pools, ring)
    assert sorted(pools) == sorted(want)
    for p in want:
        np.testing.assert_allclose(pools[p], want[p], rtol=1e-12)
