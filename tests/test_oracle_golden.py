"""The CPU oracle pinned against fixtures produced by the reference's own functions (tests/golden/make_golden.py):
canonical top-k (ssengine/model/topk_canon.py:33-52), g0 page table and slots (ssengine/model/metadata.py:79-96),
graph rows (:65-76), graph buckets (ssengine/model/stage.py:63-69), block pages (ssengine/engine/kv.py:60-75)."""

import json

import numpy as np
import pytest

from oracle import pages, topk
from tests.conftest import GOLDEN


@pytest.mark.parametrize("case", ["ties", "dense", "wide_ties"])
def test_canonical_topk_matches_reference_fixture(case):
    z = np.load(GOLDEN / "topk_canon.npz")
    g = {k.split("__", 1)[1]: z[k] for k in z.files if k.startswith(case + "__")}
    out = topk.canonical_topk(g["logits"], g["ks"], g["ke"], int(g["k"]))
    np.testing.assert_array_equal(out, g["out"])


def test_canonical_topk_reference_known_answer():
    # the reference's own known-answer test (tests/test_graphs_cpu.py:48-66 of the reference)
    logits = np.array([[9., 2., 7., 2., 0., 2.], [5., 5., 1., 3., 8., 8.], [1., 6., 4., 0., 5., 3.]], dtype=np.float32)
    out = topk.canonical_topk(logits, [0, 2, 0], [6, 4, 6], 3)
    assert out.tolist() == [[0, 1, 2], [0, 1, -1], [1, 2, 4]]


def test_g0_table_and_graph_rows_match_reference_fixture():
    z = np.load(GOLDEN / "g0_table.npz")
    counts = z["page_counts"]
    flat = z["pages"]
    pg = np.split(flat, np.cumsum(counts)[:-1])
    starts, n = z["starts"], z["num_tokens"]
    seq = starts + n
    pos = np.concatenate([np.arange(s, s + m) for s, m in zip(starts, n)])
    qsl = np.r_[0, np.cumsum(n)]
    table, slots = pages.g0_table(pg, seq, pos, qsl, int(z["width"]))
    np.testing.assert_array_equal(table, z["table"])
    np.testing.assert_array_equal(slots, z["slots"])
    np.testing.assert_array_equal(pages.graph_rows(pos, slots, z["token_ids"], int(z["bucket"])), z["graph_rows"])
    np.testing.assert_array_equal(pages.block_pages([1, 3]), z["block_pages_1_3"])


def test_buckets_match_reference_fixture():
    g = json.loads((GOLDEN / "buckets.json").read_text())
    assert list(pages.GRAPH_BUCKETS) == g["GRAPH_BUCKETS"]
    assert [pages.graph_bucket(n) for n in g["probe"]] == g["bucket"]
    assert {str(n): pages.kv_pages_for(int(n)) for n in g["kv_pages_for"]} == g["kv_pages_for"]
