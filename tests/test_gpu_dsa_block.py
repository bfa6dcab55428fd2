"""GPU parity of the DSA attention block (`layers.DsaAttention`), stage by stage on the device's own intermediates
against the oracle (oracle/dsa.py, oracle/kda.py `nvfp4_linear`, oracle/kpool.py, oracle/indexer.py, oracle/topk.py,
oracle/mla.py): two requests, one continuing a cached prefix whose chunk starts inside a pool (the tail ring), the
latent and pool-key caches paged.

Tolerances: projections and per-head GEMMs 1e-3 relative L2 (same NVFP4 codes, fp32 vs float64 sums, bf16 rounding);
norms and rope within a few bf16 steps; cache rows, transposes, index sets bit-exact; pool keys within one bf16 step;
logits 2e-3 of each row's largest magnitude; the FP8 cache rows and query bit-exact against the oracle's e4m3
quantizer; sparse MLA 3e-2 per row (its softmax weights enter P.V as e4m3)."""

import numpy as np
import pytest
import torch

from oracle import dsa as od
from oracle import indexer as oidx
from oracle import kda as ok
from oracle import kpool as okp
from oracle import mla as omla
from oracle import topk as otopk

pytestmark = pytest.mark.gpu

REQS = [(0, 48), (122, 40)]          # (start position, rows)


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def test_dsa_block_stagewise(cuda):
    from ssengine_b200 import indexer, weights
    from ssengine_b200.layers import DsaAttention

    H, QL = 512, 256
    blk = DsaAttention(31, H, cuda, q_lora=QL, nope=64, v_dim=256)
    rng = np.random.default_rng(8)
    T = sum(n for _, n in REQS)
    qsl = np.cumsum([0] + [n for _, n in REQS]).astype(np.int32)
    positions = np.concatenate([np.arange(s, s + n) for s, n in REQS]).astype(np.int64)
    pages = [[5], [2, 7]]
    width = 2
    table = np.full((2, width), -1, np.int32)
    for r, p in enumerate(pages):
        table[r, :len(p)] = p
    slots = np.array([table[r][p // 128] * 128 + p % 128 for r, (s, n) in enumerate(REQS)
                      for p in range(s, s + n)], np.int64)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).to(cuda)
    kv_cache = torch.from_numpy(omla.quantize(rng.standard_normal((8 * 128, 576)), 1.0)).to(cuda)   # cached prefix
    pool = bf(rng.standard_normal((8 * 32, 128)))
    ring = bf(rng.standard_normal((4, 2, 4, 128)))
    pool0, ring0 = (t.float().cpu().numpy() for t in (pool, ring))
    y = bf(rng.standard_normal((T, H)))
    reqs = np.array([(qsl[r], n, s, r + 1) for r, (s, n) in enumerate(REQS)], np.int32)
    groups = indexer.work_groups(qsl[:-1], [n for _, n in REQS], [s for s, _ in REQS])
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    d = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(cuda)
    out = blk.forward(y, d(positions, torch.int64), d(slots, torch.int64), d(qsl, torch.int32),
                      d(table, torch.int32), d(reqs, torch.int32), 48, d(groups, torch.int32), kv_cache, pool, ring,
                      status, keep=True)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    n = lambda t: t.float().cpu().numpy()
    P = {k: n(v) if v.dtype not in (torch.int32, torch.uint8) else v.cpu().numpy() for k, v in blk.parts.items()}
    gs = weights.GS_X
    lin = lambda x, L: ok.nvfp4_linear(x, *tuple(v.cpu().numpy() if torch.is_tensor(v) else v for v in L.logical()),
                                       gs)
    a_ref = od.bf16(lin(n(y), blk.a_proj))
    cols = QL + 576
    assert rel(P["a"][:, :QL + 512], a_ref[:, :QL + 512]) < 1e-3                      # the k rope slice is roped in place
    assert rel(P["qa"], od.bf16(od.rmsnorm(P["a"][:, :QL], n(blk.q_norm), blk.eps))) < 1e-2
    assert rel(P["kvn"], od.bf16(od.rmsnorm(P["a"][:, QL:QL + 512], n(blk.kv_norm), blk.eps))) < 1e-2
    k_rope = od.bf16(od.rope(a_ref[:, QL + 512:cols], positions, blk.theta))
    assert rel(P["kv_rows"][:, 512:], k_rope) < 2e-2
    np.testing.assert_array_equal(P["kv_rows"][:, :512], P["kvn"])
    kvc = kv_cache.cpu().numpy()
    np.testing.assert_array_equal(kvc[slots], omla.quantize(P["kv_rows"], blk.k_scale))
    q_ref = od.bf16(lin(P["qa"], blk.q_b)).reshape(T, 64, 128)
    q_ref[:, :, 64:] = od.bf16(od.rope(q_ref[:, :, 64:], positions, blk.theta))
    assert rel(P["q"].reshape(T, 64, 128), q_ref) < 2e-2
    qh = P["q"].reshape(T, 64, 128)[:, :, :64].transpose(1, 0, 2)
    lat = od.bf16(od.grouped_linear_bf16(qh, blk.w_uk.w.float().cpu().numpy()))     # [64, T, 512]
    Tp = P["q_lat"].shape[0] // 64
    assert rel(P["q_lat"].reshape(64, Tp, 512)[:, :T], lat) < 1e-3
    q_cat = np.concatenate([P["q_lat"].reshape(64, Tp, 512)[:, :T].transpose(1, 0, 2),
                            P["q"].reshape(T, 64, 128)[:, :, 64:]], axis=2)
    np.testing.assert_array_equal(P["q8"], omla.quantize(q_cat, blk.q_scale))
    assert rel(P["q_idx"], od.bf16(lin(P["qa"], blk.wq_idx))) < 1e-3
    assert rel(P["idx"][:, :288], od.bf16(lin(n(y), blk.idx_proj))) < 1e-3
    # pools: the oracle's kpool from the device's k / gate rows and the old ring
    pc = n(pool)
    ape = blk.ape.cpu().numpy()
    for r, (st, nr) in enumerate(REQS):
        rows = slice(qsl[r], qsl[r] + nr)
        k_rows, g_rows = P["idx"][rows, :128], P["idx"][rows, 160:288]
        pools, ring_r = okp.prefill_chunk(k_rows, g_rows, st, ape, {}, ring0[r + 1].copy())
        for p, v in pools.items():
            got = pc[table[r][p // 32] * 32 + p % 32]
            assert (np.abs(got - v) <= np.abs(v) * 2.0 ** -7 + 1e-6).all(), (r, p)
    # logits on the device's pool cache and its q_idx / weights
    for r, (st, nr) in enumerate(REQS):
        sl = slice(qsl[r], qsl[r] + nr)
        want = oidx.logits(P["q_idx"][sl].reshape(nr, 32, 128), P["w"][sl], pc, table[r][table[r] >= 0],
                           positions[sl])
        for i, wr in enumerate(want):
            if len(wr):
                assert np.abs(P["logits"][qsl[r] + i, :len(wr)] - wr).max() <= 2e-3 * np.abs(wr).max()
    ke = (positions + 1) // 4
    ids_ref = otopk.canonical_topk(P["logits"], np.zeros(T, np.int64), ke, 512)
    np.testing.assert_array_equal(blk.parts["ids"].cpu().numpy(), ids_ref)
    tok = blk.parts["tok"].cpu().numpy()
    np.testing.assert_array_equal(tok[:, :2051], oidx.expand(ids_ref, positions, 512))
    # sparse MLA on the device's q8, cache and token lists
    for r, (st, nr) in enumerate(REQS):
        sl = slice(qsl[r], qsl[r] + nr)
        want = omla.sparse_mla(P["q8"][sl], kvc, tok[sl, :2051], table[r][table[r] >= 0],
                               blk.scale * blk.q_scale * blk.k_scale, blk.k_scale)
        for i in range(nr):
            assert rel(P["o_lat"][qsl[r] + i], want[i]) < 3e-2, (r, i)
    v_ref = od.bf16(od.grouped_linear_bf16(P["o_lat"].transpose(1, 0, 2), blk.w_uv.w.float().cpu().numpy()))
    assert rel(P["v"].reshape(64, Tp, 256)[:, :T], v_ref) < 1e-3
    np.testing.assert_array_equal(P["o_in"].reshape(T, 64, 256), P["v"].reshape(64, Tp, 256)[:, :T].transpose(1, 0, 2))
    assert rel(n(out), od.bf16(lin(P["o_in"], blk.o_proj))) < 1e-3
