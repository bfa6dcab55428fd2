"""Host logic of the stage boundary on CPU: row order, graph buckets and table widths against the reference's rules
(pinned by the golden bucket fixture), and the message fields."""

import json

import pytest

from oracle import pages as opages
from tests.conftest import GOLDEN


def test_row_order_puts_decode_class_chunks_first_stably():
    from ssengine_b200 import stage

    assert stage.row_order([300, 10, 50, 1000, 256, 257]) == [1, 2, 4, 0, 3, 5]
    assert stage.row_order([]) == []
    assert stage.row_order([5, 4]) == opages.row_order([5, 4]) == [0, 1]


def test_graph_bucket_matches_reference_fixture():
    from ssengine_b200 import stage

    g = json.loads((GOLDEN / "buckets.json").read_text())
    assert list(stage.GRAPH_BUCKETS) == g["GRAPH_BUCKETS"]
    assert [stage.graph_bucket(n) for n in g["probe"]] == g["bucket"]


def test_table_width_is_a_power_of_two_of_blocks():
    from ssengine_b200 import stage

    assert [stage.table_width(b) for b in (1, 2, 3, 4, 5, 8)] == [134 * w for w in (1, 2, 4, 4, 8, 8)]


def test_plan_fields_mirror_the_reference_messages():
    from ssengine_b200.messages import Chunk, Plan

    c = Chunk("r", 0, 3, [1], [0] * 6, True, [1, 2, 3])
    assert Plan(7, [c, c]).num_tokens == 6
    assert list(Chunk.__dataclass_fields__) == ["req_id", "start", "num_tokens", "kv_pages", "state_blocks", "is_last",
                                                "token_ids"]


def test_kda_state_groups_match_the_reference_known_answer():
    """The reference's known answer for its 45-layer split (tests/test_model_cpu.py:147-160 of the reference): KDA
    state group 0 (g2, state_blocks[0]) holds layers 0, 6, 13, 20, 26, 33, 40; every KDA layer has a group 0..4."""
    from ssengine_b200.kvpages import kda_group

    dsa = lambda i: i % 4 == 3
    groups = {i: kda_group(i, dsa) for i in range(45) if not dsa(i)}
    assert [i for i, g in groups.items() if g == 0] == [0, 6, 13, 20, 26, 33, 40]
    assert set(groups.values()) == {0, 1, 2, 3, 4}


def test_state_pages_alias_the_dsa_latent_blocks():
    """Stage 0 of the 12/11/11/11 split: the i-th KDA layer of group g keeps its state in the i-th DSA layer's latent
    tensor, block state_blocks[g]: conv state at the block's start, recurrent state after it (256-byte aligned: 3 x 3 x 256 bf16 = 4,608 bytes for 2 heads)."""
    import torch

    from ssengine_b200.kvpages import BLOCK_TOKENS, LATENT_ROW, StageKv

    kv = StageKv(range(12), lambda i: i % 4 == 3, 3, 2, "cpu")
    assert kv.dsa_layers == [3, 7, 11] and len(kv.pages) == 3
    assert [kv.group[i] for i in kv.kda_layers] == [0, 1, 2, 3, 4, 0, 1, 2, 3]
    assert [kv.slot[i] for i in kv.kda_layers] == [0, 0, 0, 0, 0, 1, 1, 1, 1]
    page = BLOCK_TOKENS * LATENT_ROW
    base = kv.pages[1].data_ptr()
    conv, rec = kv.conv_state(6), kv.rec_state(6)          # layer 6: group 0, second of its group -> DSA layer 7
    assert conv[2].data_ptr() - base == 2 * page and kv.state_offsets(6, 2) == (2 * page, 2 * page + 4608)
    assert rec[2].data_ptr() - base == 2 * page + 4608
    assert conv.shape == (3, 3, 768) and rec.shape == (3, 2, 128, 128) and rec[1].is_contiguous()
    assert kv.latent(7).shape == (3 * BLOCK_TOKENS, LATENT_ROW) and kv.latent(7).data_ptr() == base
    rec[1].fill_(1.0)
    conv[1].fill_(2.0)
    raw = kv.pages[1][1]
    assert torch.equal(raw[4608:4608 + 2 * 128 * 128 * 4].view(torch.float32), torch.ones(2 * 128 * 128))
    assert (raw[:4608].view(torch.bfloat16) == 2.0).all() and not raw[4608 + 2 * 128 * 128 * 4:].any()


def test_block_contract_is_checked():
    import pytest

    from ssengine_b200.messages import Chunk
    from ssengine_b200.stage import check_blocks

    ok = [Chunk("a", 0, 3, [67], [2, 3, 4, 5, 6, 7], True, None), Chunk("b", 0, 3, [68], [8, 9, 10, 11, 12, 13], True,
                                                                     None)]
    check_blocks(ok, 14)
    check_blocks([Chunk("w", 0, 3, [1], [0] * 6, True, None)], 2)           # the null block for a dummy request
    with pytest.raises(ValueError, match="held twice"):
        check_blocks([ok[0], Chunk("b", 0, 3, [68], [2, 9, 10, 11, 12, 13], True, None)], 14)
    with pytest.raises(ValueError, match="both KV and state"):
        check_blocks([Chunk("a", 0, 3, [67 * 2], [2, 3, 4, 5, 6, 7], True, None)], 14)
    with pytest.raises(ValueError, match="outside the pool"):
        check_blocks([Chunk("a", 0, 3, [67], [2, 3, 4, 5, 6, 70], True, None)], 14)


def test_microbatch_former_covers_every_token_and_keeps_the_block_contract():
    import numpy as np

    from ssengine_b200.schedule import blocks_needed, microbatches, prompt_lengths
    from ssengine_b200.stage import check_blocks

    lens = prompt_lengths(40, seed=3)
    assert lens.max() <= 131072 and 4000 < np.median(lens) < 16000
    plans, high = microbatches(lens, 8192, 10_000, vocab=100)
    assert blocks_needed(plans) <= high + 1
    seen = {}
    for p in plans:
        assert sum(c.num_tokens for c in p.chunks) <= 8192
        check_blocks(p.chunks, high + 1)
        for c in p.chunks:
            assert c.start == seen.get(c.req_id, 0) and len(c.token_ids) == c.num_tokens
            assert len(c.kv_pages) * 128 >= c.start + c.num_tokens
            seen[c.req_id] = c.start + c.num_tokens
            if c.is_last:
                assert seen[c.req_id] == lens[int(c.req_id[1:])]
    assert sorted(seen.values()) == sorted(lens.tolist())          # every prompt fully prefilled
    assert all(sum(c.num_tokens for c in p.chunks) == 8192 for p in plans[:-1])


def test_head_batched_gemm_reads_and_writes_token_major_rows_in_place():
    """The DSA absorb / v_up GEMMs take each head's slice of token-major rows as a strided batch (no transposes):
    q[t, h, :nope] -> head-major latent rows, and o_lat[t, h, :] -> the token-major o_proj input o_in[t, h * v + j]."""
    import torch

    from ssengine_b200.layers import Bf16Grouped

    g = torch.Generator().manual_seed(5)
    T, NH, qh, nope, L, vd = 37, 4, 24, 16, 32, 8
    q = torch.randn(T, NH * qh, generator=g).to(torch.bfloat16)
    uk = Bf16Grouped(g, NH, L, nope, "cpu")
    lat = torch.empty(NH * T, L, dtype=torch.bfloat16)
    uk.bmm(q.view(T, NH, qh)[:, :, :nope].permute(1, 0, 2), lat.view(NH, T, L))
    want = torch.einsum("thk,hlk->htl", q.view(T, NH, qh)[:, :, :nope].float(), uk.w.float())
    torch.testing.assert_close(lat.view(NH, T, L).float(), want, rtol=2e-2, atol=2e-2)
    uv = Bf16Grouped(g, NH, vd, L, "cpu")
    o_lat = torch.randn(T, NH, L, generator=g).to(torch.bfloat16)
    o_in = torch.full((T, NH * vd), float("nan"), dtype=torch.bfloat16)
    uv.bmm(o_lat.permute(1, 0, 2), o_in.view(T, NH, vd).permute(1, 0, 2))
    want = torch.einsum("thl,hvl->thv", o_lat.float(), uv.w.float()).reshape(T, NH * vd)
    torch.testing.assert_close(o_in.float(), want, rtol=2e-2, atol=2e-2)


def test_indexer_work_groups_cover_every_row_with_visible_pools_once():
    """The indexer's host work table: groups of <= 8 consecutive query rows of one request, each row that sees at
    least one complete pool in exactly one group, the group's pool tiles those of its last (furthest) row, longest
    groups first."""
    import numpy as np

    from ssengine_b200.indexer import POOL, TILE, work_groups

    q_lens = np.array([50, 13, 70, 21, 1, 3])
    starts = np.array([0, 37, 300, 1400, 3, 0])
    q_starts = np.concatenate([[0], np.cumsum(q_lens)[:-1]])
    g = work_groups(q_starts, q_lens, starts)
    assert g.dtype == np.int32 and g.shape[1] == 4
    covered = np.zeros(int(q_lens.sum()), np.int32)
    for r, q0, nq, tiles in g:
        assert 1 <= nq <= 8 and q_starts[r] <= q0 and q0 + nq <= q_starts[r] + q_lens[r]
        covered[q0:q0 + nq] += 1
        last_pos = starts[r] + (q0 + nq - 1 - q_starts[r])
        assert tiles == -(-((last_pos + 1) // POOL) // TILE) > 0
    pos = np.concatenate([np.arange(s, s + n) for s, n in zip(starts, q_lens)])
    sees = (pos + 1) // POOL > 0
    # every row that sees a pool is in exactly one group (a row that sees none may ride along in a group whose last
    # row sees one; its logits columns are outside its key range)
    assert covered.max() <= 1 and (covered[sees] == 1).all()
    assert (np.diff(g[:, 3]) <= 0).all()


def test_tier_ranges_cover_the_stage_views_block_by_block():
    """`StageKv.tier_ranges`: every range's rows stay inside their tensor; KV ranges of different views are disjoint;
    each KDA layer's conv and recurrent ranges lie inside the latent block they alias, at `state_offsets`; every DSA
    layer has its latent, pool-key and tail ranges; state groups are the layers' KDA groups (tail: 5)."""
    from ssengine_b200.kvpages import PAGES_PER_BLOCK, StageKv

    dsa = lambda i: i % 4 == 3
    for layers in (list(range(12)), list(range(12, 23)), list(range(45))):
        nb = 3
        kv = StageKv(layers, dsa, nb, 4, "cpu")
        rs = kv.tier_ranges(2)
        spans = [(t.data_ptr(), t.data_ptr() + t.numel() * t.element_size()) for t in kv.pages + kv.pool + kv.tail]

        def inside(a, b):
            return any(lo <= a and b <= hi for lo, hi in spans)

        for r in rs:
            assert r.stage == 2 and r.kind in ("kv", "state") and r.nbytes <= r.stride
            for b in range(nb):
                assert inside(r.base + b * r.stride, r.base + b * r.stride + r.nbytes), r
        kvr = sorted((r.base + b * r.stride, r.base + b * r.stride + r.nbytes) for r in rs if r.kind == "kv"
                     for b in range(nb))
        assert all(a[1] <= b[0] for a, b in zip(kvr, kvr[1:]))
        n_dsa = len(kv.dsa_layers)
        assert [r.kind for r in rs].count("kv") == 2 * n_dsa
        assert sum(r.name.endswith(".tail") and r.group == 5 for r in rs) == n_dsa
        for layer in kv.kda_layers:
            conv = next(r for r in rs if r.name == f"layers.{layer}.conv")
            rec = next(r for r in rs if r.name == f"layers.{layer}.recurrent")
            page = kv.pages[kv.slot[layer]]
            assert conv.group == rec.group == kv.group[layer]
            for b in range(nb):
                c, q = kv.state_offsets(layer, b)
                assert conv.base + b * conv.stride == page.data_ptr() + c
                assert rec.base + b * rec.stride == page.data_ptr() + q
                assert rec.base + b * rec.stride + rec.nbytes <= page.data_ptr() + (b + 1) * page.shape[1]
        pk = next(r for r in rs if r.name.endswith(".pool_keys"))
        assert pk.nbytes == PAGES_PER_BLOCK * 32 * 128 * 2


def test_fp8_pool_pages_have_the_reference_entry_layout():
    """`StageKv(pool_fp8=True)`: each DSA layer's pool keys in pages of 33 rows of 128 bytes (the reference's 32
    entries of 132 bytes: codes, then scales), the same bytes the oracle's page writer produces; block bytes and tier
    ranges follow."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import numpy as np
    import torch

    from oracle import indexer as oidx
    from ssengine_b200.kvpages import PAGES_PER_BLOCK, StageKv, block_bytes

    dsa = lambda i: i % 4 == 3
    layers = list(range(12))
    kv = StageKv(layers, dsa, 3, 4, "cpu", pool_fp8=True)
    assert kv.pool[0].shape == (3 * PAGES_PER_BLOCK * 33, 128) and kv.pool[0].dtype == torch.uint8
    per_block = sum(t.numel() * t.element_size() for t in kv.pages + kv.pool + kv.tail) // 3
    assert per_block == block_bytes(layers, dsa, 4, pool_fp8=True) < block_bytes(layers, dsa, 4)
    pk = next(r for r in kv.tier_ranges(0) if r.name.endswith(".pool_keys"))
    assert pk.nbytes == pk.stride == PAGES_PER_BLOCK * 132 * 32
    rng = np.random.default_rng(0)
    codes, scales = oidx.quant_pool_rows(rng.standard_normal((40, 128)).astype(np.float32))
    pages = np.array([70, 71])                         # pool p of the request at page pages[p // 32], entry p % 32
    rows = oidx.pool_rows(pages, 40)
    ref = oidx.write_pool_pages(np.zeros((3 * PAGES_PER_BLOCK, 33 * 128), np.uint8), rows, codes, scales)
    mine = kv.pool[0].numpy().reshape(-1, 33 * 128)
    oidx.write_pool_pages(mine, rows, codes, scales)
    np.testing.assert_array_equal(mine, ref)
    got_c, got_s = oidx.read_pool_pages(mine, rows)
    np.testing.assert_array_equal(got_c, codes)
    np.testing.assert_array_equal(got_s, scales)


def test_kda_tables_cover_every_chunk_once_longest_first():
    """The KDA sequence tables a microbatch's prepare builds: per state group, every chunk's rows exactly once (the
    tables tile [0, T) with no overlap), longest first, each row with the chunk's state block of that group and its
    has-state flag (the chunk continues its request)."""
    import numpy as np

    from ssengine_b200.messages import Chunk
    from ssengine_b200.stage import kda_tables, row_order

    rng = np.random.default_rng(4)
    for trial in range(30):
        R = int(rng.integers(1, 12))
        lens = [int(x) for x in rng.choice([1, 3, 17, 64, 65, 256, 257, 3000, 8192], R)]
        starts = [int(x) for x in rng.choice([0, 0, 5, 4096, 70000], R)]
        chunks = [Chunk(f"r{i}", s, n, [], [10 * i + g + 1 for g in range(6)], True, None)
                  for i, (s, n) in enumerate(zip(starts, lens))]
        order = row_order(lens)
        qsl = np.concatenate([[0], np.cumsum([lens[i] for i in order])])
        t = kda_tables(chunks, order, qsl)
        assert t.shape == (5, R, 4) and t.dtype == np.int32
        for g in range(5):
            spans = sorted((int(a), int(b)) for a, b in t[g, :, :2])
            assert spans[0][0] == 0 and spans[-1][1] == qsl[-1]
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))            # a tiling: no gap, no overlap
            sizes = t[g, :, 1] - t[g, :, 0]
            assert (np.diff(sizes) <= 0).all()                                      # longest first
            for a, b, blk, has in t[g]:
                r = int(np.searchsorted(qsl, a))
                c = chunks[order[r]]
                assert b - a == c.num_tokens and blk == c.state_blocks[g] and has == int(c.start > 0)


def test_the_reference_run_config_builds_a_stage_config():
    """`StageModel(run_cfg, ...)` reads the reference's run config through `stage_settings` (its five fields, read
    directly); a `StageConfig` passes through as it is."""
    from types import SimpleNamespace

    from ssengine_b200.stage import REFERENCE_MODEL, StageConfig, bench_config, stage_settings

    own = StageConfig(layer_split=(4,), hidden=256)
    assert stage_settings(own) is own
    cfg = stage_settings(bench_config(4096))
    assert cfg.layer_split == (12, 11, 11, 11) and cfg.mb_tokens == 8192 and not cfg.cuda_graphs
    assert cfg.num_blocks == StageConfig().num_blocks
    assert all(getattr(cfg, k) == v for k, v in REFERENCE_MODEL.items())
    assert (cfg.experts, cfg.top_k, cfg.inter, cfg.routing) == (288, 8, 2048, "sigmoid")
    run = bench_config(16384, cuda_graphs=True, split=(23, 22))
    run.pool_tokens = 20_000                                     # 3 blocks of 8,576 tokens, plus the null block
    cfg = stage_settings(run)
    assert (cfg.layer_split, cfg.mb_tokens, cfg.cuda_graphs, cfg.num_blocks) == ((23, 22), 16384, True, 4)
    with pytest.raises(ValueError):
        stage_settings(bench_config(8192, checkpoint="/models/glm"))
    with pytest.raises(AttributeError):                          # a field missing from the run config
        stage_settings(SimpleNamespace(layer_split=[45], checkpoint=None, cuda_graphs=False, pool_tokens=None))
