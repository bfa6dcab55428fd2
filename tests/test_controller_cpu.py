"""The serving loop on CPU: stage 0's `Controller` (session load -> scheduler -> plans -> reports -> TTFT) and
`serve_stage`, with fake stages that take a modeled time per microbatch and keep the stage edge's order and in-flight
gate through store keys; one process (N = 1) and two gloo processes over a TCP store on 127.0.0.1."""

import multiprocessing as mp
import socket
import time
from datetime import timedelta

import numpy as np
import pytest

import __graft_entry__

__graft_entry__.import_package()            # also in the spawned stage processes, which import this module

from ssengine_b200.controller import (Controller, Reporter, SessionLoad, StoreChannel, context_ids,
                                     for_later_stages, serve_stage, wait_key)
from ssengine_b200.pagepool import KvManager, kv_pages_for
from ssengine_b200.scheduler import Scheduler, SchedulerConfig

GATE = 3


class FakeStage:
    """Stage `stage` of `n`: microbatch k starts once stage - 1 finished it (stage 0: once the last stage finished
    k - GATE), takes base + per-token time, and marks itself done in `store`. Checks every plan it gets."""

    def __init__(self, stage: int, n: int, store, num_blocks: int, us_per_token: float = 2.0, base_us: float = 400.0):
        self.stage, self.last, self.store = stage, n - 1, store
        self.num_blocks, self.per, self.base = num_blocks, us_per_token, base_us
        self.k = 0
        self.seen_tokens = 0
        self.tier_ops = 0

    def step(self, plan):
        from ssengine_b200.stage import check_blocks

        k = self.k
        assert plan.mb_id == k
        self.k += 1
        check_blocks(plan.chunks, self.num_blocks + 1)
        for c in plan.chunks:
            assert len(c.kv_pages) == kv_pages_for(c.start + c.num_tokens)
            if self.stage == 0:
                assert c.token_ids is not None and len(c.token_ids) == c.num_tokens
            else:
                assert c.token_ids is None
        n = plan.num_tokens
        self.seen_tokens += n
        self.tier_ops += len(plan.tier_ops)
        n_last = sum(c.is_last for c in plan.chunks)

        def done():
            if self.stage > 0:
                wait_key(self.store, f"d/{self.stage - 1}/{k}", 60)
            elif k >= GATE:
                wait_key(self.store, f"d/{self.last}/{k - GATE}", 60)
            t = (self.base + n * self.per) * 1e-6
            time.sleep(t)
            self.store.set(f"d/{self.stage}/{k}", b"1")
            return t * 1e9

        toks = (lambda: [(k * 31 + j) % 1000 for j in range(n_last)]) if self.stage == self.last else None
        return done, toks


def small_load(seed=3):
    return SessionLoad(sessions=12, seed=seed, vocab=5000, append_median=200, append_max=1000, ctx_cap=8000,
                       think_s=0.05, start_ctx_max=3000, stagger_s=0.2)


CFG = SchedulerConfig(order="srpt", mb_tokens=8192, force_after_ms=500.0)
NUM_BLOCKS = 60


def test_context_ids_are_a_fixed_stream_per_session_and_epoch():
    a = context_ids(1, 2, 0, 0, 1000, 151_552)
    assert np.array_equal(a[100:300], context_ids(1, 2, 0, 100, 300, 151_552))       # positions, not calls
    assert not np.array_equal(a, context_ids(1, 3, 0, 0, 1000, 151_552))
    assert not np.array_equal(a, context_ids(1, 2, 1, 0, 1000, 151_552))
    assert a.min() >= 0 and a.max() < 151_552 and len(np.unique(a)) > 990


def test_session_rounds_extend_their_context_and_start_over_at_the_cap():
    load = SessionLoad(sessions=3, seed=0, append_median=600, append_max=8192, ctx_cap=20_000, start_ctx_max=0)
    last = [0, 0, 0]
    restarts = 0
    for step in range(60):
        i = step % 3
        r = load.next_request(i, step)
        assert 1 <= r.num_tokens <= 20_000 and r.session == i
        if r.prefix_tokens == 0:
            restarts += last[i] > 0
            assert r.num_tokens <= 8192
        else:
            assert r.prefix_tokens == last[i] + 1 and r.num_tokens > r.prefix_tokens
        last[i] = r.num_tokens
    assert restarts > 0


def test_plans_for_later_stages_drop_only_the_token_ids():
    from ssengine_b200.messages import Chunk, Plan

    p = Plan(4, [Chunk("a", 0, 3, [67], [1, 2, 3, 4, 5, 6], True, [1, 2, 3])])
    q = for_later_stages(p)
    assert q.mb_id == 4 and q.chunks[0].token_ids is None and q.chunks[0].kv_pages == [67]


def test_one_stage_serves_the_session_load():
    import torch.distributed as dist

    store = dist.HashStore()
    kv = KvManager(NUM_BLOCKS, keep_sessions=True)
    sched = Scheduler(kv, CFG, None, GATE + 1, 1)
    ctl = Controller(sched, small_load(), 1)
    stage = FakeStage(0, 1, store, NUM_BLOCKS)
    rep = Reporter(0, ctl.local.put)
    s = ctl.run(stage.step, rep, None, duration_s=1.5, warm_s=0.4)
    rep.close()
    assert s["unfinished"] == 0 and s["rounds"] > 50
    assert 0 < s["ttft_s"]["p50"] <= s["ttft_s"]["p90"] <= s["ttft_s"]["max"] < 5.0
    assert 0 < s["prefix_hit_share"] < 1                # later rounds resume their session's kept context
    assert stage.k == s["microbatches"] and sched.in_flight == 0
    assert kv.hard == 0 and kv.stats["evicted_sessions"] > 0         # the pool is too small to keep them all
    assert sum(r["tokens"] - r["cached"] for r in ctl.rounds) == stage.seen_tokens


def test_one_stage_with_a_dram_tier_resumes_evicted_contexts():
    import torch.distributed as dist

    from ssengine_b200.tier import DramTier

    store = dist.HashStore()
    kv = KvManager(NUM_BLOCKS, keep_sessions=True)
    kv.lower = DramTier(80)
    sched = Scheduler(kv, CFG, None, GATE + 1, 1)
    ctl = Controller(sched, small_load(), 1)
    stage = FakeStage(0, 1, store, NUM_BLOCKS)
    rep = Reporter(0, ctl.local.put)
    s = ctl.run(stage.step, rep, None, duration_s=1.5, warm_s=0.4)
    rep.close()
    assert s["unfinished"] == 0 and kv.stats["tier_hits"] > 0 and stage.tier_ops > 0
    assert kv.lower.stats["read"] == kv.stats["tier_hits"] and kv.lower.stats["stored"] >= kv.lower.stats["read"]
    assert not kv.take_ops()                            # every recorded copy rode a plan
    assert sum(r["tokens"] - r["cached"] for r in ctl.rounds) == stage.seen_tokens


def test_one_stage_with_the_dispatch_rule_forming_plans():
    import torch.distributed as dist

    from ssengine_b200.dispatch import DispatchRule

    store = dist.HashStore()
    rule = DispatchRule(max_in_flight=GATE, lead_ms=3.0, num_stages=1)
    kv = KvManager(NUM_BLOCKS, keep_sessions=True)
    sched = Scheduler(kv, CFG, None, *rule.sched_limits)
    ctl = Controller(sched, small_load(), 1, rule=rule)
    stage = FakeStage(0, 1, store, NUM_BLOCKS)
    rep = Reporter(0, ctl.local.put)
    s = ctl.run(stage.step, rep, None, duration_s=1.5, warm_s=0.4)
    rep.close()
    assert s["unfinished"] == 0 and s["rounds"] > 50 and sched.in_flight == 0
    assert s["forming"] == "dispatch rule" and s["microbatches"] == stage.k
    assert s["decisions"]["now"] >= s["microbatches"]               # a NOW with nothing waiting forms nothing
    assert s["decisions"]["wait"] + s["decisions"]["no"] > 0
    assert 0 < s["ttft_s"]["p50"] <= s["ttft_s"]["p90"] < 5.0


def _rank(rank: int, port: int, out, use_rule: bool = False):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=60))
    try:
        store = dist.distributed_c10d._get_default_store()
        chan = StoreChannel(dist.PrefixStore("ctl/", store), give_up_s=60)
        stage = FakeStage(rank, 2, dist.PrefixStore("fake/", store), NUM_BLOCKS)
        if rank == 0:
            from ssengine_b200.dispatch import DispatchRule

            kv = KvManager(NUM_BLOCKS, keep_sessions=True)
            rule = DispatchRule(max_in_flight=GATE, lead_ms=3.0, num_stages=2) if use_rule else None
            sched = Scheduler(kv, CFG, None, *(rule.sched_limits if rule else (GATE + 1, 1)))
            ctl = Controller(sched, small_load(), 2, rule=rule)
            rep = Reporter(0, ctl.local.put)
            s = ctl.run(stage.step, rep, chan, duration_s=1.5, warm_s=0.4)
            rep.close()
            s["in_flight"], s["hard"] = sched.in_flight, kv.hard
            out.put((0, s, stage.k))
        else:
            n = serve_stage(stage.step, chan, Reporter(1, chan.put_report))
            out.put((1, None, n))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("use_rule", [False, True])
def test_two_stage_processes_serve_the_session_load(use_rule):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, out, use_rule)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, s, n = out.get(timeout=120)
        res[r] = (s, n)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    s, n0 = res[0]
    _, n1 = res[1]
    assert n0 == n1 == s["microbatches"] >= 5           # every plan reached both stages
    assert s["unfinished"] == 0 and s["in_flight"] == 0 and s["hard"] == 0 and s["rounds"] > 30
    assert 0 < s["ttft_s"]["p50"] <= s["ttft_s"]["p90"] < 5.0 and 0 < s["prefix_hit_share"] < 1
    if use_rule:                                          # both stages' reports reached the rule
        assert s["decisions"]["now"] >= s["microbatches"] and s["decisions"]["wait"] + s["decisions"]["no"] > 0


def test_a_stage_that_stops_reporting_trips_the_watchdog():
    """A stage whose microbatches never complete: the controller raises after `stall_s` instead of waiting forever."""
    import threading

    never = threading.Event()
    kv = KvManager(NUM_BLOCKS, keep_sessions=True)
    sched = Scheduler(kv, CFG, None, GATE + 1, 1)
    ctl = Controller(sched, small_load(), 1)
    rep = Reporter(0, ctl.local.put)

    def stuck_step(plan):
        return (lambda: never.wait(5.0) and 0), None

    with pytest.raises(RuntimeError, match="no stage report"):
        ctl.run(stuck_step, rep, None, duration_s=0.5, warm_s=0.1, stall_s=0.5)
    never.set()


def _failing_rank(rank: int, port: int, out, failing: int):
    """A two-stage run in which stage `failing` raises at microbatch 3 (a host-side failure: the exception of a
    stage's loop, no device involved); every rank reports how its own loop ended and after how long."""
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=60))
    try:
        store = dist.distributed_c10d._get_default_store()
        chan = StoreChannel(dist.PrefixStore("ctl/", store), give_up_s=60)
        stage = FakeStage(rank, 2, dist.PrefixStore("fake/", store), NUM_BLOCKS)

        def step(plan):
            if rank == failing and plan.mb_id == 3:
                raise ValueError("planted failure at microbatch 3")
            return stage.step(plan)

        t0 = time.monotonic()
        try:
            if rank == 0:
                sched = Scheduler(KvManager(NUM_BLOCKS, keep_sessions=True), CFG, None, GATE + 1, 1)
                ctl = Controller(sched, small_load(), 2)
                ctl.run(step, Reporter(0, ctl.local.put), chan, duration_s=30.0, warm_s=0.4)
            else:
                serve_stage(step, chan, Reporter(1, chan.put_report))
            out.put((rank, "finished", time.monotonic() - t0))
        except Exception as e:                       # noqa: BLE001 -- the test reads which exception ended the loop
            out.put((rank, f"{type(e).__name__}: {e}", time.monotonic() - t0))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failing", [0, 1])
def test_a_failing_stage_ends_every_stage_loop_promptly(failing):
    """A stage whose loop raises tells the others through the store: a later stage's failure ends stage 0's
    controller (`StageFailed`, within its 50 ms check, not after the stall watchdog's minutes), and stage 0's failure
    ends the later stage's loop (the failure, then the stop plan) instead of leaving it waiting for plans."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, port, out, failing)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, how, secs = out.get(timeout=120)
        res[r] = (how, secs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    other = 1 - failing
    assert res[failing][0] == "ValueError: planted failure at microbatch 3", res
    assert res[other][0].startswith(f"StageFailed: stage {failing} failed: ValueError: planted failure"), res
    assert res[other][1] < 20.0, res                # the 30 s run ends at the failure, far below the watchdog
