"""`StageModel.prepare`'s host tables on the CPU (the pinned copy and the device metadata kernel stubbed, the packed
arrays read back as they would land on the device), each against a plain loop restatement of its rule on seeded
random plans: row order (chunks of <= 256 tokens first, stably), the KDA sequence tables per state group (longest
first, ties in row order), the DSA page table (each request's first pages, -1 after), the kpool requests, the
indexer work groups, the stage-0 token ids and the finished rows."""

import numpy as np
import pytest
import torch

import __graft_entry__

__graft_entry__.import_package()
from ssengine_b200 import stage as S  # noqa: E402
from ssengine_b200.messages import Chunk, Plan  # noqa: E402


class _Meta:
    def ssb_stage_metadata(self, *args):
        return 0


@pytest.fixture
def host_stage(monkeypatch):
    def copy(self, device):                     # the packed buffer, unpinned, standing in for the device copy
        host = torch.zeros(max(self.size, 8), dtype=torch.uint8)
        hv = host.numpy()
        for off, a in self.items:
            hv[off:off + a.nbytes] = a.view(np.uint8).reshape(-1)
        return host, host.clone()

    monkeypatch.setattr(S._Pack, "copy", copy)
    monkeypatch.setattr(S.lib, "stream_ptr", lambda stream=None: 0)
    st = object.__new__(S.StageModel)
    st.cuda_graphs, st.kda, st.num_blocks, st.first, st.device, st._lib = False, True, 4000, True, "cpu", _Meta()
    st.is_dsa = [i % 4 == 3 for i in range(12)]
    return st


def _plan(rng, R):
    chunks = []
    for r in range(R):
        n = int(rng.choice([1, 3, 17, 256, 257, int(rng.integers(1, 900))]))
        start = int(rng.integers(0, 30_000)) if rng.random() < 0.6 else 0
        need = -(-(start + n) // 128)
        first_page = 67 * (1 + 3 * r)
        chunks.append(Chunk(f"r{r}", start, n, list(range(first_page, first_page + need + int(rng.integers(0, 3)))),
                            [3000 + 6 * r + g if rng.random() < 0.9 else 0 for g in range(6)], bool(rng.random() < 0.6),
                            rng.integers(0, 1000, n).tolist()))
    return Plan(0, chunks)


def _groups(qs, lens, starts):
    g = []
    for r, (q, n, s) in enumerate(zip(qs, lens, starts)):
        for q0 in range(q, q + n, 8):
            nq = min(8, q + n - q0)
            tiles = -(-((s + q0 + nq - 1 - q + 1) // 4) // 128)
            if tiles > 0:
                g.append((r, q0, nq, tiles))
    g.sort(key=lambda e: -e[3])
    return np.asarray(g, np.int64).reshape(-1, 4)


@pytest.mark.parametrize("seed", range(6))
def test_prepare_packs_the_tables_its_rules_give(host_stage, seed):
    rng = np.random.default_rng(seed)
    plan = _plan(rng, int(rng.integers(1, 60)))
    b = host_stage.prepare(plan)
    ch = plan.chunks
    order = [i for i, c in enumerate(ch) if c.num_tokens <= 256] + [i for i, c in enumerate(ch) if c.num_tokens > 256]
    assert list(b.order) == order
    lens = [ch[i].num_tokens for i in order]
    qsl = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    starts = [ch[i].start for i in order]
    assert b.num_tokens == qsl[-1]
    lpt = sorted(range(len(order)), key=lambda r: -lens[r])
    for g in range(5):
        want = [(qsl[r], qsl[r + 1], ch[order[r]].state_blocks[g], int(ch[order[r]].start > 0)) for r in lpt]
        assert b.kda_seqs[g].numpy().tolist() == [list(map(int, w)) for w in want]
    ptab = b.dsa["page_table"].numpy()
    for r, i in enumerate(order):
        need = -(-(starts[r] + lens[r]) // 128)
        assert ptab[r, :need].tolist() == ch[i].kv_pages[:need] and (ptab[r, need:] == -1).all()
    kreq = [[int(qsl[r]), lens[r], starts[r], ch[i].state_blocks[5]] for r, i in enumerate(order)]
    assert b.dsa["kpool_reqs"].numpy().tolist() == kreq
    assert np.array_equal(b.dsa["groups"].numpy(), _groups(qsl[:-1].tolist(), lens, starts))
    assert b.dsa["max_rows"] == max(lens)
    assert b.token_ids.numpy().tolist() == [t for i in order for t in ch[i].token_ids]
    row_end = {i: int(qsl[r + 1]) - 1 for r, i in enumerate(order)}
    assert b.last_rows.numpy().tolist() == [row_end[i] for i, c in enumerate(ch) if c.is_last]


def test_prepare_refuses_a_chunk_short_of_pages_and_a_shared_block(host_stage):
    rng = np.random.default_rng(1)
    plan = _plan(rng, 3)
    c = plan.chunks[0]
    c.kv_pages = c.kv_pages[:-(len(c.kv_pages) - (-(-(c.start + c.num_tokens) // 128)) + 1)]
    with pytest.raises(ValueError, match="KV pages"):
        host_stage.prepare(plan)
    plan = _plan(rng, 3)
    plan.chunks[1].state_blocks = [plan.chunks[0].kv_pages[0] // 67] * 6       # a KV block of request 0
    with pytest.raises(ValueError, match="held twice|both KV and state"):
        host_stage.prepare(plan)
