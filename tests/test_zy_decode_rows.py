"""Decode-class rows (chunks of at most 256 tokens: 1-token appends and short continuations) mixed with long prefill
chunks in the same microbatches, through `StageModel` on the GPU against the oracle's composition of the same stage.

The reference routes such chunks through vLLM's decode indexer path and canonicalizes its top-k to the prefill rule
(ssengine/model/pp_patch.py:369-413), and every stage orders them first (ssengine/model/metadata.py:6-9, 214); here
every row goes through the same kernels, so a decode row must match the oracle like any other. Model: BASELINE config
1's (the tiny 4-layer Glm5Next of tests/test_gpu_model.py). Three microbatches over five requests: prefills of
300 / 200 / 100 / 5 tokens; then appends of 1, 3 and 17 tokens with a new 400-token prompt; then 1, 256 and 1 tokens.

Judged teacher-forced throughout, so that each check isolates the rows of one microbatch: the oracle starts every
microbatch from the device's own states (KDA conv / recurrent, latent cache bytes, pool keys, tail ring, read back
before the forward), every layer's residual is held within 3e-2 of the oracle's layer run on the device layer's own
inputs, and the head's logits within 2e-2 of the oracle's head on the device's own final residual, with the greedy
tokens equal wherever the oracle's top-1 margin is clear (in the plan's chunk order). Chained logits are not held to
2e-2 here: the first microbatch's only finishing prompt has 5 tokens, and attention over a few tokens averages
little requantization noise away (measured 5.9e-2 chained on a B200, with every layer inside its bar; the whole-model
test's short-prompt note gives the same effect)."""

import numpy as np
import pytest
import torch

from model_params import row_chunks, stage_params, stage_states
from oracle import mhc as omhc
from oracle import model as omodel

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


LENGTHS = {"p0": 302, "p1": 203, "p2": 117, "p3": 261, "p4": 401}          # each request's tokens over the run
SCHEDULE = [[("p0", 0, 300), ("p1", 0, 200), ("p2", 0, 100), ("p3", 0, 5)],
            [("p0", 300, 1), ("p1", 200, 3), ("p2", 100, 17), ("p4", 0, 400)],
            [("p0", 301, 1), ("p3", 5, 256), ("p4", 400, 1)]]


def test_decode_class_rows_match_the_oracle(cuda):
    from ssengine_b200 import weights
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig, StageModel

    cfg = StageConfig(layer_split=(4,), hidden=256, inter=128, experts=8, top_k=2, vocab=4096, mb_tokens=1024,
                      num_blocks=40, seed=0, layer_kind="hybrid", kda_heads=2, q_lora=256, mla_nope=64,
                      mla_v_dim=256, routing="sigmoid", weight_init="normal", init_std=0.02)
    st = StageModel(cfg, 0, cuda)
    caught = []
    st.layer_hook = lambda layer, res, x_prev, post, comb: caught.append(
        tuple(t.float().cpu().numpy() for t in (res, x_prev, post, comb)))
    params = stage_params(st)
    gs_x, gs_h = weights.GS_X, weights.GS_H
    rng = np.random.default_rng(5)
    prompts = {r: rng.integers(0, cfg.vocab, n) for r, n in LENGTHS.items()}
    # request r: KV pages of block 1 + r (4 pages), state blocks 10 + 6 r ..
    res_of = {r: (list(range(67 * (1 + j), 67 * (1 + j) + 4)), [10 + 6 * j + g for g in range(6)])
              for j, r in enumerate(LENGTHS)}
    decode_rows = judged = 0
    for k, mb in enumerate(SCHEDULE):
        chunks = []
        for r, start, n in mb:
            pages, sblocks = res_of[r]
            last = k > 0 or n <= 5                       # appends return a token; of the prefills only the 5-token one
            chunks.append(Chunk(r, start, n, pages, sblocks, last, prompts[r][start:start + n].tolist()))
            decode_rows += n if n <= 256 else 0
        plan = Plan(k, chunks)
        before = stage_states(st)                        # the device's own states entering this microbatch
        caught.clear()
        tokens = st.forward(plan)
        torch.cuda.synchronize()
        assert int(st.status.item()) == 0
        assert len(caught) == 4
        rows, order = row_chunks(plan)
        tok = np.concatenate([np.asarray(c["token_ids"], np.int64) for c in rows])
        inp = (np.repeat(params["embed"][tok][:, None, :], 4, axis=1), None, None, None)
        for li, (L, stt) in enumerate(zip(params["layers"], before)):
            res, _, _, _ = omodel.layer_forward(L, stt, rows, *inp, gs_x, gs_h)
            g = caught[li]
            assert rel(g[0], res) < 3e-2, (k, li, rel(g[0], res))
            inp = g
        res, x_prev, post, comb = caught[-1]
        o_logits, o_tok = omodel.head(params, rows, omhc.post(x_prev, res, post, comb))
        # the device returns the finished prompts' logits and tokens in the plan's chunk order, the oracle in row order
        in_rows = {c: j for j, c in enumerate(i for i in order if plan.chunks[i].is_last)}
        sel = [in_rows[i] for i in range(len(plan.chunks)) if plan.chunks[i].is_last]
        got = st.last_logits.cpu().numpy()
        assert rel(got, o_logits[sel]) < 2e-2, (k, rel(got, o_logits[sel]))
        # greedy tokens equal wherever the oracle's top-1 margin is outside the logit tolerance band (4 x the 2e-2
        # relative bar x the row's logit RMS, the whole-model greedy test's rule); near ties are not judged
        ol = o_logits[sel].astype(np.float64)
        top2 = np.sort(ol, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 4 * 2e-2 * np.sqrt((ol ** 2).mean(axis=1))
        dev, ref = tokens.cpu().numpy(), np.asarray(o_tok)[sel]
        assert (dev[clear] == ref[clear]).all(), (k, dev, ref, clear)
        judged += int(clear.sum())
    assert decode_rows > 250
    print(f"decode rows {decode_rows}, greedy tokens judged {judged}")
