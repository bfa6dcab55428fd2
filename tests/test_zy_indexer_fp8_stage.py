"""A whole stage with the FP8 indexer (`StageConfig(indexer_fp8=True)`: e4m3 queries with per-(token, head) scales,
pool keys in the reference's 132-byte entries) on the GPU against the oracle's composition with its FP8 indexer branch
(oracle/model.py, oracle/indexer.py, pinned to vLLM's own quantizers and `fp8_mqa_logits_torch`). Its three kernels
are checked one by one in tests/test_gpu_indexer_fp8.py; this file is collected after the other GPU tests, so that a
run stopping at its first failure has run them all."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_stage_with_the_fp8_indexer_matches_the_oracle(cuda):
    """BASELINE config 1's model with `indexer_fp8` on, over a 2,600-token prompt (650 pools: the 512-pool top-k
    drops some), against the oracle's composition with its FP8 indexer branch, teacher-forced: every layer within 3e-2
    of the oracle's layer on the device layer's own inputs, the logits within 2e-2 of the oracle's head on the
    device's own final residual (each oracle layer runs once: a chained oracle pass doubles the test's time)."""
    from model_params import row_chunks, stage_params, stage_states
    from oracle import mhc as omhc
    from oracle import model as omodel
    from ssengine_b200 import weights
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig, StageModel

    rel = lambda a, b: float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))
    cfg = StageConfig(layer_split=(4,), hidden=256, inter=128, experts=8, top_k=2, vocab=4096, mb_tokens=4096,
                      num_blocks=8, seed=0, layer_kind="hybrid", kda_heads=2, q_lora=256, mla_nope=64, mla_v_dim=256,
                      routing="sigmoid", weight_init="normal", init_std=0.02, indexer_fp8=True)
    st = StageModel(cfg, 0, cuda)
    caught = []
    st.layer_hook = lambda layer, res, x_prev, post, comb: caught.append(
        tuple(t.float().cpu().numpy() for t in (res, x_prev, post, comb)))
    params, states = stage_params(st), stage_states(st)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, 2600)
    plan = Plan(0, [Chunk("p0", 0, 2600, list(range(67, 67 + 21)), [2, 3, 4, 5, 6, 7], True, prompt.tolist())])
    st.forward(plan)
    torch.cuda.synchronize()
    assert int(st.status.item()) == 0
    rows, _ = row_chunks(plan)
    inp = (np.repeat(params["embed"][prompt][:, None, :], 4, axis=1), None, None, None)
    for li, (L, stt) in enumerate(zip(params["layers"], states)):
        res, _, _, _ = omodel.layer_forward(L, stt, rows, *inp, weights.GS_X, weights.GS_H)
        assert rel(caught[li][0], res) < 3e-2, (li, rel(caught[li][0], res))
        inp = caught[li]
    res, x_prev, post, comb = caught[-1]
    o_logits, _ = omodel.head(params, rows, omhc.post(x_prev, res, post, comb))
    assert rel(st.last_logits.cpu().numpy(), o_logits) < 2e-2
