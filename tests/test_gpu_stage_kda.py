"""GPU checks of `StageModel` with KDA + MoE decoder layers on the 4-stream mHC residual (`layer_kind="kda"`): a model
split into two stages (stage 0 sends its [T, 4H] rows after a post-only boundary, stage 1 starts with a pre-only
boundary: the reference's edge_send / edge_recv, ssengine/model/pp_patch.py:156-163) returns the same tokens and
bit-identical logits as the unsplit stage, for a first microbatch and for a second one that continues a request
from its KDA state blocks."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def plans(vocab):
    from ssengine_b200.messages import Chunk, Plan

    rng = np.random.default_rng(9)
    ta = rng.integers(0, vocab, 60).tolist()
    tb = rng.integers(0, vocab, 30).tolist()
    # KV pages in block 1; six distinct state blocks per request (the reference's block contract)
    p1 = Plan(0, [Chunk("a", 0, 40, [67], [2, 3, 4, 5, 6, 7], False, ta[:40]),
                  Chunk("b", 0, 30, [69], [8, 9, 10, 11, 12, 13], True, tb)])
    p2 = Plan(1, [Chunk("a", 40, 20, [67], [2, 3, 4, 5, 6, 7], True, ta[40:])])
    return p1, p2


def test_two_stages_equal_one(cuda):
    from ssengine_b200.stage import StageConfig, StageModel

    base = dict(hidden=512, inter=256, experts=16, top_k=4, vocab=1000, num_blocks=14, mb_tokens=256, seed=4,
                layer_kind="kda", kda_heads=2)
    whole = StageModel(StageConfig(layer_split=(2,), **base), 0, cuda)
    s0 = StageModel(StageConfig(layer_split=(1, 1), **base), 0, cuda)
    s1 = StageModel(StageConfig(layer_split=(1, 1), **base), 1, cuda)
    for plan in plans(1000):
        t_whole = whole.forward(plan)
        hidden = s0.forward(plan)
        assert hidden.shape == (plan.num_tokens, 4 * 512)
        t_split = s1.forward(plan, hidden)
        torch.cuda.synchronize()
        assert int(whole.status[0]) == 0 and int(s1.status[0]) == 0
        assert torch.equal(t_whole, t_split)
        assert torch.equal(whole.last_logits, s1.last_logits)
        assert torch.isfinite(whole.last_logits).all()


def test_hybrid_two_stages_equal_one(cuda):
    """The hybrid split (layer 3 DSA + MoE, the others KDA + MoE): two stages reproduce one, across a continuation."""
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig, StageModel

    base = dict(hidden=512, inter=256, experts=16, top_k=4, vocab=1000, num_blocks=14, mb_tokens=256, seed=6,
                layer_kind="hybrid", kda_heads=2, q_lora=256, mla_nope=64)
    whole = StageModel(StageConfig(layer_split=(4,), **base), 0, cuda)
    s0 = StageModel(StageConfig(layer_split=(2, 2), **base), 0, cuda)
    s1 = StageModel(StageConfig(layer_split=(2, 2), **base), 1, cuda)
    assert whole.is_dsa == [False, False, False, True] and s1.is_dsa == [False, True]
    rng = np.random.default_rng(10)
    ta, tb = rng.integers(0, 1000, 170).tolist(), rng.integers(0, 1000, 30).tolist()
    plans = [Plan(0, [Chunk("a", 0, 130, [67, 68], [2, 3, 4, 5, 6, 7], False, ta[:130]),
                      Chunk("b", 0, 30, [69], [8, 9, 10, 11, 12, 13], True, tb)]),
             Plan(1, [Chunk("a", 130, 40, [67, 68], [2, 3, 4, 5, 6, 7], True, ta[130:])])]
    for plan in plans:
        t_whole = whole.forward(plan)
        t_split = s1.forward(plan, s0.forward(plan))
        torch.cuda.synchronize()
        assert int(whole.status[0]) == 0 and int(s1.status[0]) == 0
        assert torch.equal(t_whole, t_split)
        assert torch.equal(whole.last_logits, s1.last_logits)
        assert torch.isfinite(whole.last_logits).all()
