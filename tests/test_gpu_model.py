"""Whole-stage parity: a Glm5Next stage through `StageModel` on the GPU against the oracle's composition of the same
stage (oracle/model.py) on the same seeded random-init weights, read back from the device objects.

- BASELINE config 1 (the tiny Glm5Next: 4 layers KDA, KDA, KDA, DSA; hidden 256; vocab 4096; MoE of 8 routed experts
  top-2 + 1 shared, 256 -> 2 x 128 -> 256, with the reference model's routing: sigmoid + correction bias, scale 5/2;
  weights N(0, 0.02) quantized to NVFP4, the BF16 lm_head N(0, 0.02); one prompt of 512 uniform token ids, seed 0;
  one greedy token), once as one 512-token chunk and once as two chunks
  in two microbatches (300 + 212: the KDA states, kpool tail and latent cache carried across). The attention dims are
  the kernels' (KDA 2 heads of 128 = the config's 4 x 64 channels; MLA 64 heads, latent 512 + rope 64; the config's
  4 heads / 128 + 32 are not built). Checks the north star's bars: every layer's hidden state (the residual after
  its attention sub-block, and a KDA layer's final recurrent / conv state) within 3e-2 relative L2 of the oracle's
  layer run on the device layer's own inputs; the final-position logits within 2e-2 and the greedy token equal
  through the whole chain. (Chained, the per-layer residuals drift further than the per-layer bar: every NVFP4 /
  e4m3 requantization of a slightly different input turns a sub-ulp difference into code flips, so differences grow
  layer by layer -- measured 0.2 %, 0.5 %, 0.7 %, 2.8 % over the four layers; they are bounded at 6e-2 here.)
- Greedy agreement over 200 seeded synthetic prompts (8-40 tokens, four microbatches) on config 1's model (and on a
  wider variant: hidden 512, 16 experts top-4 + shared, one leading dense-FFN layer, with a lower bar explained at
  GREEDY_MODELS): agreement >= 99.5 % over the prompts whose
  oracle top-1 margin is above the logit tolerance band; prompts inside it (near ties) are counted and reported, not
  judged -- the reference's own token check rule (near ties below 3 nats are reported, not judged,
  benchmarks/check_tokens.py:10-12, 45), with the band scaled to this random model's logits: 4 x the 2e-2 relative
  logit bar times the row's logit RMS."""

import copy

import numpy as np
import pytest
import torch

from model_params import row_chunks, stage_params, stage_states
from oracle import model as omodel

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def _stage(cfg, cuda):
    from ssengine_b200.stage import StageModel

    st = StageModel(cfg, 0, cuda)
    caught = []
    st.layer_hook = lambda layer, res, x_prev, post, comb: caught.append(
        tuple(t.float().cpu().numpy() for t in (res, x_prev, post, comb)))
    return st, caught


def _gs():
    from ssengine_b200 import weights

    return weights.GS_X, weights.GS_H


@pytest.mark.parametrize("split", [(512,), (300, 212)])
def test_config1_tiny_model(cuda, split):
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig

    cfg = StageConfig(layer_split=(4,), hidden=256, inter=128, experts=8, top_k=2, vocab=4096, mb_tokens=512,
                      num_blocks=8, seed=0, layer_kind="hybrid", kda_heads=2, q_lora=256, mla_nope=64, mla_v_dim=256,
                      routing="sigmoid", weight_init="normal", init_std=0.02)
    st, caught = _stage(cfg, cuda)
    params, states = stage_params(st), stage_states(st)
    gs_x, gs_h = _gs()
    prompt = np.random.default_rng(0).integers(0, cfg.vocab, 512)
    pages = list(range(67, 67 + 4))                    # block 1's first pages
    sblocks = [2, 3, 4, 5, 6, 7]                      # state blocks g2..g6 and the kpool tail
    kv = st.kv
    at = 0
    for i, n in enumerate(split):
        plan = Plan(i, [Chunk("p0", at, n, pages, sblocks, at + n == 512, prompt[at:at + n].tolist())])
        at += n
        caught.clear()
        tokens = st.forward(plan)
        torch.cuda.synchronize()
        assert int(st.status.item()) == 0
        chunks, _ = row_chunks(plan)
        before = copy.deepcopy(states)
        (o_logits, o_tok), o_res = omodel.stage_forward(params, chunks, None, states, gs_x, gs_h, first=True,
                                                        last=True)
        assert len(caught) == len(o_res) - 1 == 4
        chained = [rel(c[0], o) for c, o in zip(caught, o_res)]
        print(f"split {split} microbatch {i}: chained residual rel L2 per layer {[round(v, 4) for v in chained]}")
        assert max(chained) < 6e-2
        # every layer on the device layer's own inputs (the stage's embedded rows for layer 0)
        x0 = params["embed"][np.asarray(chunks[0]["token_ids"])]
        inp = (np.repeat(x0[:, None, :], 4, axis=1), None, None, None)
        for li, (L, stt) in enumerate(zip(params["layers"], before)):
            res, x_b, post, comb = omodel.layer_forward(L, stt, chunks, *inp, gs_x, gs_h)
            g = caught[li]
            assert rel(g[0], res) < 3e-2, (split, i, li, rel(g[0], res))
            if L["kind"] == "kda":
                blk = sblocks[kv.group[li]]
                assert rel(st.kda_states[li][1][blk].cpu().numpy(), stt[1][blk]) < 3e-2
                assert rel(st.kda_states[li][0][blk].float().cpu().numpy(), stt[0][blk]) < 3e-2
            inp = g
        if at == 512:
            g_logits = st.last_logits.cpu().numpy()
            assert rel(g_logits, o_logits) < 2e-2, rel(g_logits, o_logits)
            assert tokens.cpu().numpy().tolist() == o_tok.tolist()
    # every KDA layer's state sits at the reference's offsets: block state_blocks[g] of the latent tensor its group
    # slot aliases (here the stage's only DSA layer), the conv state first, the recurrent state after it
    P = cfg.kda_heads * 128
    for li in kv.kda_layers:
        blk = sblocks[kv.group[li]]
        conv_off, rec_off = kv.state_offsets(li, blk)
        raw = kv.pages[kv.slot[li]].cpu().numpy().reshape(-1)
        conv = raw[conv_off:conv_off + 9 * P * 2].view(np.uint16)
        recs = raw[rec_off:rec_off + cfg.kda_heads * 128 * 128 * 4].view(np.float32)
        own_conv, own_rec = st.kda_states[li][0][blk], st.kda_states[li][1][blk]
        np.testing.assert_array_equal(conv, own_conv.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
                                      .reshape(-1))
        np.testing.assert_array_equal(recs, own_rec.contiguous().cpu().numpy().reshape(-1))
    assert kv.slot[0] == 0 and kv.group[0] == 0 and [kv.group[i] for i in (1, 2)] == [1, 2]


GREEDY_MODELS = {
    # BASELINE config 1's model, prompts of 48-160 tokens; the north star's bar
    "config1": (dict(hidden=256, inter=128, experts=8, top_k=2, routing="sigmoid"), (48, 161), 0.995),
    # a wider variant with a leading dense-FFN layer on short prompts (8-40 tokens): its DSA layer's e4m3 latent
    # cache and query requantize rows that differ by ~1 % after three layers, and attention over a few dozen tokens
    # averages little of it away: ~6 % at that layer's output and ~4e-2 in the logits (measured), so a lower
    # agreement bar is asserted and the measured figure reported
    "h512_dense": (dict(hidden=512, inter=256, experts=16, top_k=4, dense_layers=1, dense_inter=512), (8, 41), 0.97),
}


def _oracle_microbatch(args):
    """One microbatch of fresh requests through the oracle (a separate process: microbatches of fresh requests do not
    depend on each other's states)."""
    params, rows, states, gs_x, gs_h = args
    (o_logits, o_tok), o_res = omodel.stage_forward(params, rows, None, states, gs_x, gs_h, first=True, last=True)
    return o_logits, o_tok, o_res


@pytest.mark.parametrize("model", list(GREEDY_MODELS))
def test_greedy_agreement_over_synthetic_prompts(cuda, model):
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig

    dims, lengths, bar = GREEDY_MODELS[model]
    cfg = StageConfig(layer_split=(4,), vocab=4096, mb_tokens=8192, num_blocks=8 + 6 * 50, seed=3,
                      layer_kind="hybrid", kda_heads=2, q_lora=256, mla_nope=64, mla_v_dim=256, weight_init="normal",
                      init_std=0.02, **dims)
    st, caught = _stage(cfg, cuda)
    params, states = stage_params(st), stage_states(st)
    gs_x, gs_h = _gs()
    rng = np.random.default_rng(1234)
    lens = rng.integers(*lengths, 200)
    gpu = []
    for m in range(4):
        chunks = []
        for j in range(50):
            r = 50 * m + j
            n = int(lens[r])
            # KV: pages in blocks 1-3; state blocks: 6 distinct blocks per request of this microbatch
            chunks.append(Chunk(f"p{r}", 0, n, [67 + 2 * j, 68 + 2 * j], [8 + 6 * j + g for g in range(6)], True,
                                rng.integers(0, cfg.vocab, n).tolist()))
        plan = Plan(m, chunks)
        caught.clear()
        tokens = st.forward(plan).cpu().numpy()
        gpu.append((plan, tokens, st.last_logits.cpu().numpy(), [c[0] for c in caught]))
    import multiprocessing as mp

    jobs = [(params, row_chunks(plan)[0], copy.deepcopy(states), gs_x, gs_h) for plan, _, _, _ in gpu]
    with mp.get_context("spawn").Pool(4) as pool:
        oracle = pool.map(_oracle_microbatch, jobs)
    judged = agree = near = 0
    worst = 0.0
    for m, ((plan, tokens, g_logits, g_res), (o_logits, o_tok, o_res)) in enumerate(zip(gpu, oracle)):
        order = row_chunks(plan)[1]
        print(f"microbatch {m}: chained residual rel L2 per layer "
              f"{[round(rel(g, o), 4) for g, o in zip(g_res, o_res)]}")
        inv = np.argsort(order)                     # the oracle's rows are in row order, the device's in plan order
        o_logits, o_tok = o_logits[inv], o_tok[inv]
        worst = max(worst, rel(g_logits, o_logits))
        for i in range(len(tokens)):
            srt = np.sort(o_logits[i])
            band = 4 * 2e-2 * np.sqrt((o_logits[i] ** 2).mean())
            if srt[-1] - srt[-2] < band:
                near += 1
                continue
            judged += 1
            agree += int(tokens[i] == o_tok[i])
    print(f"{model}: greedy agreement {agree}/{judged} judged, {near} near ties reported, worst logits rel L2 "
          f"{worst:.2e}")
    assert judged >= 150 and agree >= bar * judged, (agree, judged, near, worst)
