"""Host-side logic of the pipeline benchmark on CPU: the layer splits, the config-4 microbatch stream that
`--steps 20 --warmup 5` times (100 microbatches), the block contract of every plan against the pool it sizes, and the
algorithmic FLOP count."""

import numpy as np


def test_layer_splits_are_the_reference_ones():
    import bench

    assert bench.split_for(1) == (45,)
    assert bench.split_for(2) == (23, 22)
    assert bench.split_for(4) == (12, 11, 11, 11)
    assert bench.split_for(8) == (6, 6, 6, 6, 6, 5, 5, 5)
    assert all(sum(bench.split_for(n)) == 45 for n in (1, 2, 3, 4, 5, 6, 7, 8))


def test_stream_of_the_timed_microbatches_keeps_the_block_contract():
    import bench
    from ssengine_b200.kvpages import BLOCK_TOKENS, PAGE_TOKENS
    from ssengine_b200.stage import check_blocks

    W, K, M = 5, 20, bench.MB_PER_STEP
    plans, nb = bench.pipeline_plans((W + K) * M, bench.MB_TOKENS, None)
    assert len(plans) == (W + K) * M
    seen = {}
    for p in plans:
        n = sum(c.num_tokens for c in p.chunks)
        assert 0 < n <= bench.MB_TOKENS
        check_blocks(p.chunks, nb)
        for c in p.chunks:
            # the pages cover the chunk's positions; a request's chunks continue where the last one ended
            assert len(c.kv_pages) * PAGE_TOKENS >= c.start + c.num_tokens
            assert max(c.kv_pages) // (BLOCK_TOKENS // PAGE_TOKENS) < nb
            assert seen.get(c.req_id, 0) == c.start
            seen[c.req_id] = c.start + c.num_tokens
    # the timed microbatches reach long contexts (the stream's 128k-token prompt)
    ctx = [max(c.start + c.num_tokens for c in p.chunks) for p in plans[W * M:]]
    assert max(ctx) == 131_072


def test_microbatch_flops_count_the_projections_and_attention():
    import bench
    from ssengine_b200.messages import Chunk, Plan
    from ssengine_b200.stage import StageConfig

    cfg = StageConfig(layer_split=(45,), **bench.MODEL)
    short = Plan(0, [Chunk("a", 0, 8192, list(range(64)), [1] * 6, True, None)])
    long = Plan(1, [Chunk("b", 100_000, 8192, list(range(900)), [1] * 6, True, None)])
    f_short, f_long = bench.microbatch_flops(short, cfg, 45), bench.microbatch_flops(long, cfg, 45)
    # at least the MoE experts of 42 layers (9 rows of 25.17 MFLOP a token) and at most a few times that
    moe = 42 * 8192 * 9 * 25.17e6
    assert moe < f_short < 4 * moe
    assert f_long > f_short                               # the indexer and the selected tokens grow with the context
    assert np.isfinite(f_long)


def test_session_pool_is_sized_by_the_costliest_stage():
    """The session run's pool: what the memory budget holds on the stage whose blocks cost the most, capped at the
    reference's 7,143 usable blocks."""
    import bench
    from ssengine_b200.kvpages import block_bytes

    dsa = lambda i: i % 4 == 3
    stage0 = block_bytes(list(range(12)), dsa, bench.MODEL["kda_heads"])       # 3 DSA layers
    assert bench.session_pool_blocks(bench.split_for(4), 100e9) == int(100e9 // stage0)
    whole = block_bytes(list(range(45)), dsa, bench.MODEL["kda_heads"])        # 11 DSA layers
    assert bench.session_pool_blocks(bench.split_for(1), 100e9) == int(100e9 // whole) < 2000
    assert bench.session_pool_blocks(bench.split_for(8), 1e15) == 7143


def test_session_workload_glue_runs_end_to_end_on_fakes(monkeypatch, capsys):
    """`bench.run_sessions` at N = 1 with the device pieces replaced (no GPU here): the scheduler, page pool,
    controller and reporter run for real, the stage's forward is a fake that takes a modeled time, and the JSON line
    carries the TTFT fields."""
    import json
    import time
    import types

    import torch

    import bench
    from ssengine_b200 import controller, stage

    class FakeStageModel:
        def __init__(self, cfg, rank, device):
            self.cfg, self.first, self.last = cfg, rank == 0, True
            self.hidden_width = 4 * cfg.hidden
            self.status = torch.zeros(1, dtype=torch.int32)
            self.kv = None

    def fake_step(worker, device):
        def step(plan):
            n = plan.num_tokens
            done_last = [c for c in plan.chunks if c.is_last]

            def done():
                time.sleep(2e-4 + n * 1e-8)
                return int(n * 1e4)

            return done, (lambda: [7] * len(done_last))
        return step

    class FakeArena:                                          # the pinned host mirror needs a CUDA context
        def __init__(self, stage_kv, rank, blocks, device=None):
            self.blocks, self.bytes_moved = blocks, 0

        def apply(self, ops, stream=None):
            self.bytes_moved += len(ops)

        def check(self):
            pass

    from ssengine_b200 import tier

    monkeypatch.setattr(torch.cuda, "set_device", lambda *a: None)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    monkeypatch.setattr(stage, "StageModel", FakeStageModel)
    monkeypatch.setattr(controller, "cuda_step", fake_step)
    monkeypatch.setattr(tier, "TierArena", FakeArena)
    for dram in (0.0, 2.0):
        args = types.SimpleNamespace(sessions=6, session_s=0.8, session_warm_s=0.2, think_s=0.02, start_ctx=2000,
                                     pool_gb=1.0, force_after_ms=500.0, dram_gb=dram, tokens=8192, layers=45,
                                     forming="rule" if dram else "limits")
        bench.run_sessions(args, 0, 1, 0)
        line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert line["metric"].startswith("TTFT") and line["unit"] == "s" and line["higher_is_better"] is False
        assert line["rounds"] > 5 and line["unfinished"] == 0 and line["ttft_s"]["p50"] > 0
        assert line["config"]["parallelism"] == "pp1" and line["kv"]["admitted"] >= line["rounds"]
        assert (line["dram_tier"] is not None) == (dram > 0)


def _sessions_rank(rank: int, port: int, out):
    import io
    import os
    import sys
    import time
    import types
    from contextlib import redirect_stdout

    sys.path.insert(0, os.environ["SSB_ROOT"])
    import __graft_entry__

    __graft_entry__.import_package()
    import torch

    import bench
    from ssengine_b200 import controller, edge, stage

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")

    class FakeStageModel:
        def __init__(self, cfg, r, device):
            self.cfg, self.first, self.last = cfg, r == 0, r == 1
            self.hidden_width = 4 * cfg.hidden
            self.status = torch.zeros(1, dtype=torch.int32)
            self.kv = None

    class FakePipe:
        def __init__(self, *a, **k):
            pass

        def check(self):
            pass

        def close(self):
            pass

    def fake_step(worker, device):
        def step(plan):
            n_last = sum(c.is_last for c in plan.chunks)

            def done():
                time.sleep(2e-4)
                return 100_000

            return done, ((lambda: [3] * n_last) if worker.stage.last else None)
        return step

    torch.cuda.set_device = lambda *a: None
    torch.cuda.synchronize = lambda *a: None
    stage.StageModel = FakeStageModel
    edge.P2pPipe = FakePipe
    controller.cuda_step = fake_step
    args = types.SimpleNamespace(sessions=6, session_s=0.8, session_warm_s=0.2, think_s=0.02, start_ctx=2000,
                                 pool_gb=1.0, force_after_ms=500.0, dram_gb=0.0, tokens=8192, layers=45,
                                 forming="rule")
    buf = io.StringIO()
    with redirect_stdout(buf):
        bench.run_sessions(args, rank, 2, rank)
    out.put((rank, buf.getvalue()))


def test_session_workload_glue_two_ranks():
    import json
    import multiprocessing as mp
    import os
    import socket
    from pathlib import Path

    os.environ["SSB_ROOT"] = str(Path(__file__).resolve().parent.parent)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sessions_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[1] == ""                                      # only rank 0 prints
    line = json.loads(res[0].strip().splitlines()[-1])
    assert line["n_gpus"] == 2 and line["config"]["parallelism"] == "pp2"
    assert line["rounds"] > 5 and line["unfinished"] == 0 and line["ttft_s"]["p50"] > 0
