"""The CPU oracle's MoE routing rule and permutation contract (known answers and invariants), and the generator."""

import numpy as np

from oracle import moe


def test_route_ties_go_to_the_lower_expert_and_weights_are_a_softmax():
    logits = np.array([[1.0, 3.0, 3.0, 0.5, 3.0, -1.0],
                       [0.0, 0.0, 0.0, 0.0, 0.0, 0.0]], dtype=np.float32)
    ids, w = moe.route_softmax_topk(logits, 2)
    assert ids.tolist() == [[1, 2], [0, 1]]
    np.testing.assert_allclose(w, 0.5, rtol=1e-7)
    ids3, w3 = moe.route_softmax_topk(logits, 4)
    assert ids3[0].tolist() == [1, 2, 4, 0]
    e = np.exp(np.array([3, 3, 3, 1.0]) - 3)
    np.testing.assert_allclose(w3[0], e / e.sum(), rtol=1e-6)


def test_permutation_contract():
    rng = np.random.default_rng(0)
    T, E, k = 1000, 12, 3
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    counts, offsets, rows, srows = moe.permutation(ids, E)
    assert counts[:E].tolist() == np.bincount(ids.ravel(), minlength=E).tolist() and counts[E] == T
    assert (offsets % 128 == 0).all() and offsets[-1] == sum(-(-c // 128) * 128 for c in counts)
    # every (token, slot) has its own row inside its expert's range, tokens ascending inside an expert
    for e in range(E):
        t, j = np.nonzero(ids == e)
        r = rows[t, j]
        assert sorted(r.tolist()) == list(range(offsets[e], offsets[e] + counts[e]))
        assert (np.diff(r[np.argsort(t)]) == 1).all()
    assert srows.tolist() == list(range(offsets[E], offsets[E] + T))


def test_moe_forward_runs_and_is_consistent_with_its_parts():
    import torch

    from ssengine_b200 import weights

    T, H, F, E, k = 64, 256, 128, 8, 2
    p = weights.to_numpy(weights.moe_logical(3, H, F, E))
    x = weights.hidden_states(4, T, H).float().numpy()
    out, parts = moe.moe_forward(x, p, k, return_parts=True)
    assert out.shape == (T, H) and np.isfinite(out).all()
    re = (parts["weights"][:, :, None] * parts["y_routed"]).sum(1) + parts["y_shared"]
    np.testing.assert_allclose(out, re, rtol=1e-5, atol=1e-5)
    # the generator's scales give unit-variance logits and O(1) outputs
    assert 0.5 < parts["logits"].std() < 2.0
    assert 0.3 < out.std() < 5.0
    assert torch.equal(weights.hidden_states(4, T, H), weights.hidden_states(4, T, H))
