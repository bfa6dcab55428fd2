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


def test_pools_match_the_reference_flow():
    """Pools and tail ring written by the reference's own insert path (pp_patch `kpool_heads` /
    `kpool_compress_insert` / `kpool_seed_tail_cache` with its torch reference ops, tests/golden/kpool_ref.npz made by
    tests/golden/make_golden.py) over chunked prefills of three requests that start inside pools and share
    microbatches, against the oracle's chunk-by-chunk restatement."""
    import sys
    from pathlib import Path

    golden = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(golden))
    import make_golden as mg

    f = np.load(golden / "kpool_ref.npz")
    k, g, ape = mg.kpool_inputs()
    pools = [dict() for _ in mg.KPOOL_LENS]
    rings = [np.zeros((2, 4, 8)) for _ in mg.KPOOL_LENS]
    for mb in mg.KPOOL_SCHEDULE:
        for r, s, n in mb:
            okp.prefill_chunk(k[r][s:s + n], g[r][s:s + n], s, ape, pools[r], rings[r])
    got = np.concatenate([np.stack([pools[r][p] for p in range(n // 4)]) for r, n in enumerate(mg.KPOOL_LENS)])
    # the reference sums in fp32, the oracle in float64: measured 2.2e-7 absolute on values up to 1.6
    np.testing.assert_allclose(got, f["pools"], rtol=0, atol=2e-6)
    # the trailing partial pool of each request sits in its tail ring
    for r, n in enumerate(mg.KPOOL_LENS):
        for pos in range(n - n % 4, n):
            np.testing.assert_array_equal(rings[r][:, pos % 4], f["tail"][r, :, pos % 4])
