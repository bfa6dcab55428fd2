"""Host logic of the stage boundary on CPU: row order, graph buckets and table widths against the reference's rules
(pinned by the golden bucket fixture), and the message fields."""

import json

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
