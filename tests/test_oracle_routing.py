"""The oracle's sigmoid + correction-bias routing (the reference model's rule) pinned to:

- the reference's own routing check (fixture tests/golden/routing_ref.npz from ssengine/model/moe_tuning.py
  `scale_hist` / `forced_logits` and the rule `(logits.sigmoid() + bias).topk(8)` as the reference's
  tests/test_moe_tuning_cpu.py:55-64 runs it): the same experts for every token and the same histogram;
- vLLM 0.22.0's DeepSeek-V2/V3 router `grouped_topk` (fixture tests/golden/routing_vllm.npz, CPU): one ungrouped case
  with the reference's dims (288 experts, top-8, scale 2.5) and one grouped case (256 experts in 8 groups, 4 kept):
  the same expert sets and, per expert, weights within 5e-7 relative (measured 2.8e-7 on 3 of 768: vLLM evaluates the
  sigmoid in fp32 and sums the selected scores in its own order).

Made by tests/golden/make_golden.py --parts routing and tests/golden/make_vllm_golden.py --parts routing."""

import sys
from pathlib import Path

import numpy as np

from oracle import moe as omoe

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_vllm_golden as gen  # noqa: E402


def test_sigmoid_routing_matches_the_reference_rule():
    f = np.load(GOLDEN / "routing_ref.npz")
    sel = np.unpackbits(f["selected"], axis=1)[:, :288].astype(bool)
    logits = np.where(sel, np.float32(30.0), np.float32(-30.0))
    ids, w = omoe.route_sigmoid_bias(logits, 8, f["bias"], 1, 1, 2.5)
    np.testing.assert_array_equal(np.sort(ids, axis=1), f["ids_sorted"])
    np.testing.assert_array_equal(np.bincount(ids.reshape(-1), minlength=288), f["hist"])
    np.testing.assert_allclose(w.sum(axis=1), 2.5, rtol=1e-6)


def test_sigmoid_routing_matches_vllm_grouped_topk():
    f = np.load(GOLDEN / "routing_vllm.npz")
    for name, c in gen.ROUTING_CASES.items():
        inp = gen.routing_inputs(name)
        ids, w = omoe.route_sigmoid_bias(inp["logits"], c["k"], inp["bias"], c["n_group"], c["topk_group"],
                                         c["scale"])
        order = np.argsort(ids, axis=1)
        np.testing.assert_array_equal(np.take_along_axis(ids, order, 1), f[f"{name}_ids"], err_msg=name)
        np.testing.assert_allclose(np.take_along_axis(w, order, 1), f[f"{name}_weights"], rtol=5e-7, atol=0,
                                   err_msg=name)


def test_slots_are_in_rank_order_with_ties_to_the_lower_expert():
    logits = np.zeros((1, 8), np.float32)
    bias = np.array([0, 1, 1, 0, 2, 0, 1, 0], np.float32)
    ids, w = omoe.route_sigmoid_bias(logits, 4, bias, 1, 1, 1.0)
    assert ids.tolist() == [[4, 1, 2, 6]]
    np.testing.assert_allclose(w, 0.25)
    # groups of 2 over choices 0.5 + bias: sums (2, 2, 3, 2) -> group 2, then group 0 (the lowest of the tied) kept;
    # among experts 0, 1, 4, 5: 4, 1, then 0 (tied with 5)
    ids, _ = omoe.route_sigmoid_bias(logits, 3, bias, 4, 2, 1.0)
    assert ids.tolist() == [[4, 1, 0]]
