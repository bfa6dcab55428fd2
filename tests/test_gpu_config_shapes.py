"""GPU parity at the shapes the bench times.

- BASELINE config 2 exactly as `bench.py` builds it (T = 8192, H = 4096, 128 experts top-8 + shared, F = 1024, the
  bench's seeds): router logits, routing, expert counts, offsets, permuted rows, GEMM tile table and CTA-pair table over
  the whole microbatch; the layer output on a 512-row sample through the oracle (one expert's fp32 weights at a time).
- BASELINE config 3's attention-pair kernels: KDA with 32 heads over 8,192 tokens of three requests continuing cached
  states (every row of 3 sampled heads against the token-by-token recurrence); the indexer at positions beyond 16k, so
  that the canonical top-512 drops pools (logits of sampled rows, top-k and expansion of every row); sparse MLA over
  2,051 selected tokens of 64k-token prefixes (sampled rows).

Tolerances are the ones of the smaller-shape tests (tests/test_gpu_moe.py, test_gpu_kda.py, test_gpu_indexer.py,
test_gpu_mla.py): bit-exact for integer outputs, 3e-2 relative L2 for the MoE output (the per-layer bar), 2e-2 for KDA
outputs and states, 2e-3 of each row's largest logit, 3e-2 per sparse-MLA row."""

import numpy as np
import pytest
import torch

from oracle import indexer as oidx
from oracle import kda as ok
from oracle import mla as omla
from oracle import moe as omoe
from oracle import topk as otopk
from oracle.mhc import bf16

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


# ---------------------------------------------------------------------------------------------- config 2
def test_moe_layer_at_config2(cuda):
    import bench
    from ssengine_b200 import moe, weights

    T, H, F, E, k = 8192, bench.H, bench.F, bench.E, bench.K_TOP
    assert (H, F, E, k) == (4096, 1024, 128, 8)
    layer = moe.MoELayer.from_logical(weights.moe_logical(bench.SEED, H, F, E, device=cuda), k, cuda)
    x = weights.hidden_states(bench.SEED + 1, T, H, device=cuda)
    out = layer(x)
    torch.cuda.synchronize()
    layer.check_status()
    p = layer.logical()
    xf = x.float().cpu().numpy()
    o = out.float().cpu().numpy()

    logits = layer.ws_view("LOGITS", T, torch.float32, (T, E)).cpu().numpy()
    ids = layer.ws_view("IDS", T, torch.int32, (T, k)).cpu().numpy()
    wts = layer.ws_view("WEIGHTS", T, torch.float32, (T, k)).cpu().numpy()
    rid, rw = omoe.route_softmax_topk(logits, k)
    np.testing.assert_array_equal(ids, rid)
    np.testing.assert_allclose(wts, rw, rtol=2e-6, atol=1e-7)
    counts, offsets, rows, _ = omoe.permutation(ids, E)
    np.testing.assert_array_equal(layer.ws_view("COUNTS", T, torch.int32, (E + 1,)).cpu().numpy(), counts)
    np.testing.assert_array_equal(layer.ws_view("OFFSETS", T, torch.int32, (E + 2,)).cpu().numpy(), offsets)
    np.testing.assert_array_equal(layer.ws_view("ROWS", T, torch.int32, (T, k)).cpu().numpy(), rows)
    nt = layer.ws_view("NUM_MTILES", T, torch.int32, (2,)).cpu().numpy()
    assert nt[0] == offsets[-1] // 128
    cap = -(-(T * (k + 1) + (E + 1) * 127) // 128)
    both = layer.ws_view("MTILES", T, torch.int32, (cap + int(nt[1]), 4)).cpu().numpy()
    tiles = [(e, offsets[e] + 128 * i, min(128, counts[e] - 128 * i), 0)
             for e in range(E + 1) for i in range(-(-int(counts[e]) // 128))]
    assert [tuple(r) for r in both[:nt[0]].tolist()] == tiles
    pairs = [(e, offsets[e] + 256 * j, min(128, counts[e] - 256 * j), max(0, min(128, counts[e] - 256 * j - 128)))
             for e in range(E + 1) for j in range(-(-int(counts[e]) // 256))]
    assert [tuple(r) for r in both[cap:].tolist()] == pairs
    # odd tile counts per expert exist at this shape (CTA pairs with an empty second half)
    assert any((-(-int(c) // 128)) % 2 for c in counts)

    sample = np.sort(np.random.default_rng(2).choice(T, 512, replace=False))
    want, parts = omoe.moe_forward(xf[sample], p, k, ids=ids[sample], weights=wts[sample], dense="lazy",
                                   return_parts=True)
    np.testing.assert_allclose(logits[sample], parts["logits"], rtol=1e-4,
                               atol=1e-4 * np.abs(parts["logits"]).max())
    assert rel(o[sample], want) < 3e-2, rel(o[sample], want)


# ---------------------------------------------------------------------------------------------- config 3: KDA
def test_kda_at_config3_heads(cuda):
    from ssengine_b200.kda import KdaLayer, seq_table

    H, D = 32, 128
    P = H * D
    lens = [4100, 2900, 1192]
    st = np.concatenate([[0], np.cumsum(lens)])
    T = int(st[-1])
    seqs = [(int(st[i]), int(st[i + 1]), i + 1, 1) for i in range(3)]
    rng = np.random.default_rng(33)
    x = bf16(rng.standard_normal((T, 3 * P)).astype(np.float32))
    w = bf16(rng.uniform(-0.6, 0.6, (3 * P, 4)))
    g = bf16(rng.standard_normal((T, P)).astype(np.float32))
    beta = bf16(rng.standard_normal((T, H)))
    a_log = rng.uniform(-1, 1, H).astype(np.float32)
    dtb = (rng.standard_normal(P) * 0.5).astype(np.float32)
    cst = bf16(rng.standard_normal((4, 3, 3 * P)))
    rst = (rng.standard_normal((4, H, D, D)) * 0.05).astype(np.float32)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(cuda)
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)
    L = KdaLayer(bf(w), f32(a_log), f32(dtb), -5.0)
    dcst, drst = bf(cst), f32(rst)
    out = torch.zeros(T, P, dtype=torch.bfloat16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    L.prefill(bf(x), bf(g), bf(beta), out, seq_table(seqs, cuda), dcst, drst, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o = out.float().cpu().numpy().reshape(T, H, D)
    got_st = drst.cpu().numpy()
    q, kk, v, wcst = ok.conv(x, w, cst, seqs, P)
    np.testing.assert_array_equal(dcst.float().cpu().numpy(), wcst)
    heads = [0, 13, 31]
    want, wrst = ok.recurrent(q, kk, v, g, beta, a_log, dtb, -5.0, D ** -0.5, rst, seqs, H, D, heads=heads)
    want = want.reshape(T, H, D)
    for s, e, blk, _ in seqs:
        for h in heads:
            assert rel(o[s:e, h], want[s:e, h]) < 2e-2, (s, h, rel(o[s:e, h], want[s:e, h]))
            assert rel(got_st[blk, h], wrst[blk, h]) < 2e-2, (blk, h)


# ---------------------------------------------------------------------------------------------- config 3: DSA
def _pages(reqs, rng):
    """KV pages of each request (start position, rows) in a shuffled order -> int32 table [R, width], pages used."""
    n_pages = [-(-(s + n) // 128) for s, n in reqs]
    perm = rng.permutation(sum(n_pages)) + 1
    table = np.full((len(reqs), max(n_pages)), -1, np.int32)
    at = 0
    for r, n in enumerate(n_pages):
        table[r, :n] = perm[at:at + n]
        at += n
    return table, int(perm.max()) + 1


def test_indexer_selection_beyond_16k(cuda):
    from ssengine_b200 import indexer

    reqs = [(20000, 512), (40000, 512)]
    rng = np.random.default_rng(44)
    table, n_pages = _pages(reqs, rng)
    T = sum(n for _, n in reqs)
    qsl = np.cumsum([0] + [n for _, n in reqs]).astype(np.int32)
    positions = np.concatenate([np.arange(s, s + n) for s, n in reqs]).astype(np.int64)
    assert ((positions + 1) // 4).min() > 4 * 512          # every row sees more pools than it selects
    q = bf16(rng.standard_normal((T, 32, 128)))
    w = bf16(rng.uniform(0, 1, (T, 32)))                  # the head weights arrive as bf16
    kc = bf16(rng.standard_normal((n_pages * 32, 128)))
    d = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(cuda)
    groups = indexer.work_groups(qsl[:-1], [n for _, n in reqs], [s for s, _ in reqs])
    ldl = -(-int((positions.max() + 1) // 4) // 128) * 128
    logits = torch.full((T, ldl), float("nan"), dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    pos = d(positions, torch.int64)
    indexer.logits(d(q, torch.bfloat16), d(w, torch.bfloat16), d(kc, torch.bfloat16), d(table, torch.int32),
                   d(groups, torch.int32), logits, status)
    ids = torch.empty(T, 512, dtype=torch.int32, device=cuda)
    indexer.topk(logits, pos, 512, ids)
    tok = torch.empty(T, 4 * 512 + 3 + 5, dtype=torch.int32, device=cuda)
    indexer.expand(ids, pos, tok)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    lg = logits.cpu().numpy()
    for r, (s, n) in enumerate(reqs):
        sample = np.sort(rng.choice(n, 16, replace=False))
        want = oidx.logits(q[qsl[r] + sample], w[qsl[r] + sample], kc, table[r][table[r] >= 0], positions[qsl[r] + sample])
        for i, wr in zip(sample, want):
            got = lg[qsl[r] + i, :len(wr)]
            assert np.abs(got - wr).max() <= 2e-3 * np.abs(wr).max(), (r, i)
    ke = (positions + 1) // 4
    ids_ref = otopk.canonical_topk(lg, np.zeros(T, np.int64), ke, 512)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)
    assert (ids_ref >= 0).all()                             # full selections (every row has > 512 pools)
    np.testing.assert_array_equal(tok.cpu().numpy()[:, :2051], oidx.expand(ids_ref, positions, 512))


def test_sparse_mla_over_64k_prefixes(cuda):
    from ssengine_b200 import mla

    reqs = [(65536, 160), (61000, 96)]
    rng = np.random.default_rng(55)
    table, n_pages = _pages(reqs, rng)
    T = sum(n for _, n in reqs)
    qsl = np.cumsum([0] + [n for _, n in reqs]).astype(np.int32)
    positions = np.concatenate([np.arange(s, s + n) for s, n in reqs]).astype(np.int64)
    g = torch.Generator(device=cuda).manual_seed(5)
    kv = torch.randn(n_pages * 128, 576, device=cuda, generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
    q8 = (torch.randn(T, 64, 576, device=cuda, generator=g) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    # 512 selected pools per row among the visible ones, expanded with the row's tail: 2,051 columns
    pools = np.stack([np.sort(rng.choice((int(p) + 1) // 4, 512, replace=False)) for p in positions])
    idx = np.full((T, 2056), -1, np.int32)
    idx[:, :2051] = oidx.expand(pools, positions, 512)
    assert (idx[:, :2048] >= 0).all()
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out = torch.full((T, 64, 512), float("nan"), dtype=torch.bfloat16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    scale = 192 ** -0.5
    mla.sparse_mla(q8, kv, d(idx), d(qsl), d(table), scale, out, n_idx=2051, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o = out.float().cpu().numpy()
    kvh, qh = kv.cpu().numpy(), q8.cpu().numpy()
    for r, (s, n) in enumerate(reqs):
        sample = np.sort(rng.choice(n, 6, replace=False))
        rows = qsl[r] + sample
        want = omla.sparse_mla(qh[rows], kvh, idx[rows, :2051], table[r][table[r] >= 0], scale, 1.0)
        for i, row in enumerate(rows):
            assert rel(o[row], want[i]) < 3e-2, (r, int(row), rel(o[row], want[i]))
