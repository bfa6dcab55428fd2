"""The DRAM tier on CPU: the copy runs of a tier op move exactly a context's page slices and state rows between a
stage's cache views and their host mirror; and under random session churn, applying the recorded ops in order before
each forward always leaves a resumed context's pages and state where its round reads them."""

import ctypes
import random

import numpy as np
import pytest
import torch

from ssengine_b200.kvpages import PAGES_PER_BLOCK, StageKv
from ssengine_b200.pagepool import KvManager, kv_pages_for
from ssengine_b200.scheduler import Request
from ssengine_b200.tier import DramTier, TierArena, TierOp, op_runs


def memmove_copier(runs, stream=None):
    for s, d, n in runs.tolist():
        ctypes.memmove(d, s, n)


def test_runs_are_aligned_merged_and_cut():
    kv = StageKv(list(range(12)), lambda i: i % 4 == 3, 4, 4, "cpu")
    arena = TierArena(kv, 0, 3, copier=memmove_copier)
    op = TierOp("write", [67, 68, 69, 200], [1, 2, 3, 1, 2, 3], [0 + 67, 1 + 67, 2 + 67, 134], [2, 1, 3, 2, 1, 3])
    runs = op_runs(op, arena.hbm_ranges, arena.dram_ranges, piece=64 * 1024)
    assert runs.dtype == np.int64 and (runs % 16 == 0).all() and (runs[:, 2] <= 64 * 1024).all()
    # 3 latent + 3 pool-key views x (pages 67-69 contiguous on both sides, page 200 alone), 3 tails, 9 KDA x 2 states
    lat = kv.tier_ranges(0)[0]
    page = lat.nbytes // PAGES_PER_BLOCK
    total = 3 * (4 * page) + 3 * 4 * (PAGES_PER_BLOCK * 32 * 256 // PAGES_PER_BLOCK)
    total += sum(r.nbytes for r in arena.hbm_ranges if r.kind == "state")
    assert int(runs[:, 2].sum()) == total
    with pytest.raises(ValueError):
        op_runs(TierOp("move", [], [], [], []), arena.hbm_ranges, arena.dram_ranges)


@pytest.mark.parametrize("layers", [list(range(12)), list(range(12, 23)), list(range(39, 45))])
def test_write_then_read_moves_the_context_bytes(layers):
    g = torch.Generator().manual_seed(1)
    # HBM blocks 1-9, DRAM blocks 1-9; as the page pool hands them out, a state block is never a KV page's block
    hbm = StageKv(layers, lambda i: i % 4 == 3, 10, 4, "cpu")
    for t in hbm.pages + hbm.pool + hbm.tail:
        t.view(torch.uint8).copy_(torch.randint(0, 256, t.view(torch.uint8).shape, dtype=torch.uint8, generator=g))
    arena = TierArena(hbm, 1, 9, copier=memmove_copier)
    pages, old_states = [70, 71, 140, 141, 142], [3, 4, 5, 6, 7, 8]
    dram_pages, dram_states = [70, 71, 72, 73, 74], [2, 3, 4, 5, 6, 7]
    ref = {id(t): t.clone() for t in hbm.pages + hbm.pool + hbm.tail}
    arena.apply([TierOp("write", pages, old_states, dram_pages, dram_states)])
    for t in hbm.pages + hbm.pool + hbm.tail:                    # HBM reuses everything
        t.zero_()
    new_pages, new_states = [150, 151, 152, 153, 154], [9, 8, 7, 6, 5, 3]
    arena.apply([TierOp("read", new_pages, new_states, dram_pages, dram_states)])
    # every KV page slice and every state row came back at its new place
    for j, layer in enumerate(hbm.dsa_layers):
        lat_old, lat = ref[id(hbm.pages[j])], hbm.pages[j]
        pb = lat.shape[1] // PAGES_PER_BLOCK
        for po, pn in zip(pages, new_pages):
            a = lat_old[po // PAGES_PER_BLOCK, (po % PAGES_PER_BLOCK) * pb:(po % PAGES_PER_BLOCK + 1) * pb]
            b = lat[pn // PAGES_PER_BLOCK, (pn % PAGES_PER_BLOCK) * pb:(pn % PAGES_PER_BLOCK + 1) * pb]
            assert torch.equal(a, b)
            bits = lambda t: t.view(torch.int16)                 # random bytes as bf16 include NaNs
            assert torch.equal(bits(ref[id(hbm.pool[j])][po * 32:(po + 1) * 32]), bits(hbm.pool[j][pn * 32:(pn + 1) * 32]))
        assert torch.equal(ref[id(hbm.tail[j])][old_states[5]].view(torch.int16),
                           hbm.tail[j][new_states[5]].view(torch.int16))
    for layer in hbm.kda_layers:
        gi = hbm.group[layer]
        t_old, t = ref[id(hbm.pages[hbm.slot[layer]])], hbm.pages[hbm.slot[layer]]
        c_o, r_o = hbm.state_offsets(layer, old_states[gi])
        c_n, r_n = hbm.state_offsets(layer, new_states[gi])
        flat_old, flat = t_old.reshape(-1), t.reshape(-1)
        assert torch.equal(flat_old[c_o:c_o + hbm.conv_bytes], flat[c_n:c_n + hbm.conv_bytes])
        rec = hbm.kda_heads * 128 * 128 * 4
        assert torch.equal(flat_old[r_o:r_o + rec], flat[r_n:r_n + rec])
    assert arena.bytes_moved > 0
    with pytest.raises(ValueError):                              # block 10 is outside the 10 HBM rows
        arena.apply([TierOp("read", [10 * 67], new_states, [70], dram_states)])
    with pytest.raises(ValueError):                              # block 0 is the null block
        arena.apply([TierOp("write", [70], [0, 2, 3, 4, 5, 6], [70], dram_states)])


def _churn(seed: int, steps: int = 1500, hbm_blocks: int = 40, dram_blocks: int = 30):
    """Random sessions over HBM + DRAM. Every page and state block carries a tag of what it holds; ops are applied in
    the order recorded (before the next forward), a forward writes its request's pages and final state; at every
    admission with a hit, the pages and state the round resumes from must hold its context."""
    rng = random.Random(seed)
    kv = KvManager(hbm_blocks, keep_sessions=True)
    kv.lower = tier = DramTier(dram_blocks)
    hbm, dram, hst, dst = {}, {}, {}, {}
    ctx = {}                                              # session -> (epoch, tokens of its last prompt)
    running = []
    hits = {"hbm": 0, "tier": 0}

    def apply_ops():
        for op in kv.take_ops():
            if op.kind == "write":
                for p, q in zip(op.hbm_pages, op.dram_pages):
                    dram[q] = hbm.get(p)
                for p, q in zip(op.hbm_states, op.dram_states):
                    dst[q] = hst.get(p)
            else:
                for p, q in zip(op.hbm_pages, op.dram_pages):
                    hbm[p] = dram.get(q)
                for p, q in zip(op.hbm_states, op.dram_states):
                    hst[p] = dst.get(q)

    for step in range(steps):
        if running and rng.random() < 0.45:
            r = running.pop(rng.randrange(len(running)))
            kv.release(r)
            ctx[r.session] = (r.epoch, r.num_tokens)
            apply_ops()
            continue
        s = rng.randrange(24)
        if any(r.session == s for r in running):
            continue
        epoch, prev = ctx.get(s, (0, 0))
        if prev and rng.random() < 0.1:
            epoch, prev = epoch + 1, 0                   # the session starts over
        n = (prev + 1 if prev else 0) + rng.choice([rng.randrange(1, 400), rng.randrange(1, 2 * 8576)])
        r = Request(f"r{step}", n, session=s, prefix_tokens=prev + 1 if prev else 0, epoch=epoch)
        if not kv.fits(r):
            continue
        r.cached = kv.allocate(r)
        apply_ops()
        a = kv.held[r.req_id]
        if r.cached:
            hits["tier" if r.admit_info["hit_kind"] == "tier" else "hbm"] += 1
            for i in range(kv_pages_for(r.cached)):
                assert hbm.get(a.kv_pages[i]) == (s, epoch, i), (step, i, r.admit_info)
            for gidx, b in enumerate(a.state_blocks):
                assert hst.get(b) == (s, epoch, r.cached, gidx), (step, gidx)
        for i in range(kv_pages_for(n)):                  # the forward writes the prompt's pages and final state
            hbm[a.kv_pages[i]] = (s, epoch, i)
        for gidx, b in enumerate(a.state_blocks):
            hst[b] = (s, epoch, n, gidx)
        running.append(r)
    return kv, tier, hits


def test_resumed_contexts_find_their_pages_and_states_after_in_order_copies():
    tot = {"hbm": 0, "tier": 0}
    for seed in range(4):
        kv, tier, hits = _churn(seed)
        for k in tot:
            tot[k] += hits[k]
        assert tier.stats["stored"] > 10 and tier.stats["read"] > 5
        assert kv.stats["tier_hits"] == tier.stats["read"]
    assert tot["tier"] > 20 and tot["hbm"] > 20


def test_fp8_pool_pages_move_with_the_context():
    g = torch.Generator().manual_seed(2)
    hbm = StageKv(list(range(12)), lambda i: i % 4 == 3, 10, 4, "cpu", pool_fp8=True)
    for t in hbm.pages + hbm.pool + hbm.tail:
        t.view(torch.uint8).copy_(torch.randint(0, 256, t.view(torch.uint8).shape, dtype=torch.uint8, generator=g))
    arena = TierArena(hbm, 0, 9, copier=memmove_copier)
    assert arena.dram.pool_fp8
    ref = [t.clone() for t in hbm.pool]
    arena.apply([TierOp("write", [70, 141], [3, 4, 5, 6, 7, 8], [75, 76], [2, 3, 4, 5, 6, 7])])
    for t in hbm.pool:
        t.zero_()
    arena.apply([TierOp("read", [150, 80], [9, 8, 7, 6, 5, 4], [75, 76], [2, 3, 4, 5, 6, 7])])
    for old, new in zip(ref, hbm.pool):
        for po, pn in ((70, 150), (141, 80)):
            assert torch.equal(old[po * 33:(po + 1) * 33], new[pn * 33:(pn + 1) * 33])


def _runs_reference(op, hbm_ranges, dram_ranges, piece):
    """The copy runs restated slice by slice (the vectorized op_runs must give exactly these)."""
    runs = []
    write = op.kind == "write"
    for hr, dr in zip(hbm_ranges, dram_ranges):
        if hr.kind == "kv":
            pb = hr.nbytes // PAGES_PER_BLOCK
            sl = [(hr.base + (h // 67) * hr.stride + (h % 67) * pb, dr.base + (d // 67) * dr.stride + (d % 67) * pb,
                   pb) for h, d in zip(op.hbm_pages, op.dram_pages)]
        elif 0 <= hr.group < len(op.hbm_states):
            sl = [(hr.base + op.hbm_states[hr.group] * hr.stride, dr.base + op.dram_states[hr.group] * dr.stride,
                   hr.nbytes)]
        else:
            sl = []
        for h, d, n in sl:
            a, b = (h, d) if write else (d, h)
            if runs and runs[-1][0] + runs[-1][2] == a and runs[-1][1] + runs[-1][2] == b:
                runs[-1][2] += n
            else:
                runs.append([a, b, n])
    return [(a + o, b + o, min(piece, n - o)) for a, b, n in runs for o in range(0, n, piece)]


def test_vectorized_runs_equal_the_slice_by_slice_restatement():
    rng = np.random.default_rng(9)
    kv = StageKv(list(range(12)), lambda i: i % 4 == 3, 40, 4, "cpu")
    arena = TierArena(kv, 0, 30, copier=memmove_copier)
    for trial in range(20):
        n = int(rng.integers(0, 300))
        hb = rng.choice(np.arange(67, 39 * 67), n, replace=False)
        if trial % 3 == 0:
            hb = np.sort(hb)                                      # runs of consecutive pages merge
        db = rng.choice(np.arange(67, 30 * 67), n, replace=False)
        if trial % 2 == 0:
            db = np.sort(db)
        op = TierOp("write" if trial % 2 else "read", hb.tolist(), [1, 2, 3, 4, 5, 6], db.tolist(),
                    [7, 8, 9, 10, 11, 12])
        for piece in (64 * 1024, 256 * 1024):
            got = op_runs(op, arena.hbm_ranges, arena.dram_ranges, piece)
            want = np.asarray(_runs_reference(op, arena.hbm_ranges, arena.dram_ranges, piece), np.int64).reshape(-1, 3)
            np.testing.assert_array_equal(got, want)


def test_a_batch_prepared_early_still_carries_its_tier_copies():
    """The pipeline prepares batches ahead and steps them: the plan's copies ride the batch, not the plan object."""
    from ssengine_b200.messages import Plan
    from ssengine_b200.stage import Batch
    from ssengine_b200.worker import StageWorker

    op = TierOp("write", [70], [1, 2, 3, 4, 5, 6], [70], [1, 2, 3, 4, 5, 6], 10)

    class Stage:
        first = last = True

        def prepare(self, plan):
            return Batch(0, [], None, None, None, None, None, tier_ops=list(plan.tier_ops))

        def run(self, batch, hidden):
            return "tokens"

    class Arena:
        applied = []

        def apply(self, ops, stream=None):
            self.applied.append(list(ops))

    plan = Plan(3, [], tier_ops=[op])
    w = StageWorker(Stage(), tier=Arena())
    assert w.step(Stage().prepare(plan)) == "tokens" and Arena.applied == [[op]]
    assert w.step(plan) == "tokens" and Arena.applied == [[op], [op]]
    with pytest.raises(RuntimeError):
        StageWorker(Stage()).step(plan)                          # copies and no tier: refused


def test_the_copy_kernel_path_refuses_host_views():
    kv = StageKv(list(range(4)), lambda i: i % 4 == 3, 3, 4, "cpu")
    arena = TierArena(kv, 0, 2, copier=memmove_copier)          # (pinned DRAM views need a driver)
    arena.copier = arena._cuda_copier                            # the default: ssb_copy_runs, which needs device views
    with pytest.raises(ValueError):
        arena.apply([TierOp("write", [70], [1, 1, 1, 1, 1, 1], [70], [1, 1, 1, 1, 1, 1])])
