"""GPU parity of the FP8 indexer forms (`ssb_indexer_q_quant`, `ssb_kpool_insert_fp8`, `ssb_indexer_logits_fp8`)
against the oracle's FP8 restatement (oracle/indexer.py, pinned to vLLM's own quantizers and `fp8_mqa_logits_torch`):

- query codes and ue8m0 scales bit-exact;
- logits over pool pages of the reference's 132-byte entries, written by the oracle, within 1e-4 of each row's largest
  magnitude (exact e4m3 products summed in fp32 on the tensor cores vs float64);
- the FP8 pool insert against the validated bf16 insert on the same inputs: every code within one e4m3 step of the
  bf16 pool value over its scale, scales equal to the oracle's rule on the bf16 values except where a row's fp32 amax
  sits at a power-of-two boundary.

The three kernel tests passed on their first B200 run. The whole stage on these forms is checked in
tests/test_zy_indexer_fp8_stage.py, collected after the other GPU tests."""

import numpy as np
import pytest
import torch

from oracle import indexer as oidx
from oracle.mla import e4m3_decode

pytestmark = pytest.mark.gpu

REQS = [(0, 50), (37, 13), (300, 70), (1400, 21), (3, 1)]       # (position of the first query row, query rows)


def test_query_quantization_matches_the_oracle(cuda):
    from ssengine_b200 import indexer

    rng = np.random.default_rng(3)
    q = torch.from_numpy(rng.standard_normal((77, 32, 128)).astype(np.float32) * 3).to(torch.bfloat16).to(cuda)
    q[5, 7] = 0                                                  # an all-zero row takes the 1e-10 floor
    q8 = torch.empty(77, 32, 128, dtype=torch.uint8, device=cuda)
    qs = torch.empty(77, 32, dtype=torch.float32, device=cuda)
    indexer.q_quant(q, q8, qs)
    torch.cuda.synchronize()
    codes, scales = oidx.quant_query_heads(q.float().cpu().numpy())
    np.testing.assert_array_equal(q8.cpu().numpy(), codes)
    np.testing.assert_array_equal(qs.cpu().numpy(), scales)


def test_fp8_logits_over_reference_pages(cuda):
    from ssengine_b200 import indexer

    rng = np.random.default_rng(0)
    T = sum(n for _, n in REQS)
    q_starts = np.cumsum([0] + [n for _, n in REQS])[:-1]
    positions = np.concatenate([np.arange(s, s + n) for s, n in REQS]).astype(np.int64)
    n_pages = [-(-(s + n) // 128) for s, n in REQS]
    perm = rng.permutation(sum(n_pages) + 3) + 1
    width = max(n_pages) + 2
    table = np.full((len(REQS), width), -1, np.int32)
    at = 0
    for r, n in enumerate(n_pages):
        table[r, :n] = perm[at:at + n]
        at += n
    pages_total = int(perm.max()) + 1
    cache = np.zeros((pages_total, 33 * 128), np.uint8)
    for r, n in enumerate(n_pages):                              # every pool the request's pages hold
        pools = oidx.pool_rows(table[r, :n], n * 32)
        codes, sc = oidx.quant_pool_rows(rng.standard_normal((n * 32, 128)).astype(np.float32))
        oidx.write_pool_pages(cache, pools, codes, sc)
    q = torch.from_numpy(rng.standard_normal((T, 32, 128)).astype(np.float32)).to(torch.bfloat16).to(cuda)
    c = 128 ** -0.5 * 32 ** -0.5                                 # softmax scale x heads^-1/2, folded into w
    w = torch.from_numpy(rng.uniform(-1, 1, (T, 32)).astype(np.float32) * c).to(torch.bfloat16).to(cuda)
    q8 = torch.empty(T, 32, 128, dtype=torch.uint8, device=cuda)
    qs = torch.empty(T, 32, dtype=torch.float32, device=cuda)
    indexer.q_quant(q, q8, qs)
    groups = indexer.work_groups(q_starts, [n for _, n in REQS], [s for s, _ in REQS])
    out = torch.full((T, 512), float("nan"), dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    indexer.logits_fp8(q8, qs, w, torch.from_numpy(cache.reshape(-1, 128)).to(cuda), torch.from_numpy(table).to(cuda),
                       torch.from_numpy(groups).to(cuda), out, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    got = out.cpu().numpy()
    q8h, qsh, wh = q8.cpu().numpy(), qs.cpu().numpy(), w.float().cpu().numpy() / c
    for r, ((s, n), q0) in enumerate(zip(REQS, q_starts)):
        sl = slice(q0, q0 + n)
        want = oidx.logits_fp8(q8h[sl], qsh[sl], wh[sl], cache, table[r], positions[sl])
        for i, wr in enumerate(want):
            if len(wr):
                g = got[q0 + i, :len(wr)]
                assert np.abs(g - wr).max() <= 1e-4 * max(np.abs(wr).max(), 1e-6), (r, i)


def test_fp8_pool_insert_against_the_bf16_insert(cuda):
    from ssengine_b200 import indexer

    rng = np.random.default_rng(1)
    starts, lens = [0, 5, 130, 0], [40, 67, 9, 3]                # chunks starting inside a pool take the tail ring
    R = len(starts)
    T = sum(lens)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).to(cuda)
    k, gate = bf(rng.standard_normal((T, 128))), bf(rng.standard_normal((T, 128)))
    ape = torch.from_numpy(rng.standard_normal((4, 128)).astype(np.float32)).to(cuda)
    first = np.cumsum([0] + lens)[:-1]
    reqs = torch.tensor([[int(f), n, s, 1 + r] for r, (f, n, s) in enumerate(zip(first, lens, starts))],
                        dtype=torch.int32, device=cuda)
    table = torch.tensor([[2 + 3 * r, 3 + 3 * r, 4 + 3 * r] for r in range(R)], dtype=torch.int32, device=cuda)
    ring0 = bf(rng.standard_normal((R + 1, 2, 4, 128)))
    pool16 = torch.zeros(16 * 32, 128, dtype=torch.bfloat16, device=cuda)
    pool8 = torch.zeros(16 * 33, 128, dtype=torch.uint8, device=cuda)
    ring_a, ring_b = ring0.clone(), ring0.clone()
    indexer.kpool_insert(k, gate, ape, reqs, max(lens), table, pool16, ring_a)
    indexer.kpool_insert_fp8(k, gate, ape, reqs, max(lens), table, pool8, ring_b)
    torch.cuda.synchronize()
    assert torch.equal(ring_a, ring_b)                            # the tail ring stays bf16, the same
    p16, p8 = pool16.float().cpu().numpy(), pool8.cpu().numpy().reshape(16, 33 * 128)
    written = np.abs(p16).sum(axis=1) > 0
    rows = np.flatnonzero(written)
    assert len(rows) > 20
    codes, scales = oidx.read_pool_pages(p8, rows)
    vals = e4m3_decode(codes) * scales[:, None]
    ref = p16[rows]
    want_s = oidx.ue8m0(np.maximum(np.float32(1e-4), np.abs(ref).max(axis=1)) / np.float32(448))
    assert np.mean(scales == want_s) > 0.95
    assert (np.abs(vals - ref) <= (2.0 ** -3) * np.abs(ref) + scales[:, None] * 2.0 ** -9 + 1e-2 * np.abs(ref)).all()
