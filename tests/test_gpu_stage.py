"""GPU parity of the stage boundary: device metadata (`ssb_stage_metadata`) bit-exact against fixtures produced by
the reference's `g0_table` / `graph_rows`; `StageModel` prepare / run on a 2-stage tiny model against the oracle."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import stage as ostage
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


def test_stage_metadata_matches_reference_fixture(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    z = np.load(GOLDEN / "g0_table.npz")
    starts, n, counts = z["starts"], z["num_tokens"], z["page_counts"]
    R, T, width, bucket = len(starts), int(n.sum()), int(z["width"]), int(z["bucket"])
    qsl = np.r_[0, np.cumsum(n)].astype(np.int32)
    page_ptr = np.r_[0, np.cumsum(counts)].astype(np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    q, st, pp, pg = dev(qsl), dev(starts.astype(np.int32)), dev(page_ptr), dev(z["pages"].astype(np.int32))
    pos = torch.full((bucket,), -5, dtype=torch.int64, device=cuda)
    slots = torch.full((bucket,), -5, dtype=torch.int64, device=cuda)
    table = torch.full((R, width), -5, dtype=torch.int32, device=cuda)
    rc = so.ssb_stage_metadata(q.data_ptr(), st.data_ptr(), pp.data_ptr(), pg.data_ptr(), R, T, bucket, 128, width,
                               pos.data_ptr(), slots.data_ptr(), table.data_ptr(),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    lib.check("ssb_stage_metadata", rc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(table.cpu().numpy(), z["table"])
    np.testing.assert_array_equal(slots.cpu().numpy()[:T], z["slots"])
    np.testing.assert_array_equal(pos.cpu().numpy(), z["graph_rows"][0])
    np.testing.assert_array_equal(slots.cpu().numpy(), z["graph_rows"][1])


def tiny_cfg(**kw):
    from ssengine_b200.stage import StageConfig

    base = dict(layer_split=(1, 1), hidden=256, inter=128, experts=8, top_k=2, vocab=4096, mb_tokens=1024,
                num_blocks=16, seed=3)
    base.update(kw)
    return StageConfig(**base)


def plan_of(rng, lens, vocab):
    from ssengine_b200.messages import Chunk, Plan

    chunks, page = [], 1
    for j, n in enumerate(lens):
        npg = -(-n // 128)
        chunks.append(Chunk(f"r{j}", 0, n, list(range(page, page + npg)), [0] * 6, j != 1,
                            rng.integers(0, vocab, size=n).tolist()))
        page += npg
    return Plan(0, chunks)


def test_two_stage_forward_matches_oracle(cuda):
    from ssengine_b200.stage import StageModel

    cfg = tiny_cfg()
    s0, s1 = StageModel(cfg, 0, cuda), StageModel(cfg, 1, cuda)
    assert s0.first and not s0.last and s1.last and not s1.first
    assert list(s0.layer_range) == [0] and list(s1.layer_range) == [1] and s0.hidden_width == 256
    rng = np.random.default_rng(0)
    plan = plan_of(rng, [300, 10, 90, 257], cfg.vocab)   # chunk 1 is decode-class: rows go first
    b0 = s0.prepare(plan)
    assert b0.order == [1, 2, 0, 3] and b0.num_tokens == 657
    hidden = s0.run(b0, None)
    tokens = s1.forward(plan, hidden)
    torch.cuda.synchronize()
    for s in (s0, s1):
        for layer in s.layers:
            layer.check_status()

    # stage 0 in the oracle: embedding rows in row order, then x + MoE(x)
    ids = np.concatenate([np.asarray(plan.chunks[i].token_ids) for i in b0.order])
    x0 = s0.embed.float().cpu().numpy()[ids]
    p0 = s0.layers[0].logical()
    ref0 = x0 + omoe.moe_forward(x0, p0, cfg.top_k)
    h = hidden.float().cpu().numpy()
    assert np.linalg.norm(h - ref0) / np.linalg.norm(ref0) < 3e-2

    # last stage head: its own normed rows -> logits (tolerance) -> tokens (bit-exact argmax of its logits)
    last_rows = [int(np.cumsum([plan.chunks[i].num_tokens for i in b0.order])[b0.order.index(i)]) - 1
                 for i, c in enumerate(plan.chunks) if c.is_last]
    assert s1.prepare(plan).last_rows.cpu().tolist() == last_rows
    logits = s1.last_logits.cpu().numpy()
    np.testing.assert_array_equal(tokens.cpu().numpy(), ostage.argmax_lowest(logits))
    # the BF16 lm_head: fp32 logits of the bf16 normed rows against float64 (cuBLAS accumulates in fp32)
    ref_logits = s1.last_normed.double().cpu().numpy() @ s1.head_w.double().cpu().numpy().T
    assert np.linalg.norm(logits - ref_logits) / np.linalg.norm(ref_logits) < 1e-4
    normed_ref = ostage.rmsnorm(s1.layers[0](hidden).float().cpu().numpy()[last_rows], np.ones(cfg.hidden), 1e-5)
    assert np.abs(s1.last_normed.float().cpu().numpy() - normed_ref).max() < 2e-2 * np.abs(normed_ref).max()
    assert tokens.dtype == torch.int64 and tokens.shape == (3,)


def test_single_stage_with_graph_buckets(cuda):
    from ssengine_b200.stage import StageModel

    s = StageModel(tiny_cfg(layer_split=(2,), cuda_graphs=True), 0, cuda)
    assert s.first and s.last
    plan = plan_of(np.random.default_rng(1), [200, 57], 4096)
    b = s.prepare(plan)
    assert b.bucket == 512 and b.positions.shape == (512,)
    assert (b.slots[257:] == -1).all() and (b.positions[257:] == 0).all()
    tok = s.run(b, None)
    again = s.forward(plan)
    torch.cuda.synchronize()
    assert tok.shape == (1,) and torch.equal(tok, again)     # deterministic, chunk 1 is not last
