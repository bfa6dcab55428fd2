"""The control plane (scheduler, page pool + prefix cache, dispatch rule) on CPU.

Parity: the reference's own control plane ran the scenarios of control_sim.py and recorded every microbatch (chunks,
KV pages, state blocks), every admission and the forming decisions (tests/golden/control_ref.json.gz, made by
tests/golden/make_control_golden.py); this package must reproduce them exactly. Known answers: the cases of the
reference's tests/test_scheduler.py, tests/test_kv.py and tests/test_prefix.py, restated with their expected values.
"""

import gzip
import json
import random
from types import SimpleNamespace

import numpy as np
import pytest

import control_sim
from conftest import GOLDEN
from ssengine_b200 import dispatch, pagepool, scheduler
from ssengine_b200.pagepool import (PAGES_PER_BLOCK, STATE_BLOCKS, STATE_PAGES, KvManager, PagePool, kv_blocks_for,
                                    kv_pages_for, pages_for, pool_size)
from ssengine_b200.scheduler import PlainScheduler, Request, Scheduler, SchedulerConfig

BLOCK_TOKENS = 8576
NS = SimpleNamespace(Request=Request, KvManager=KvManager, Scheduler=Scheduler, SchedulerConfig=SchedulerConfig,
                     kv_pages_for=kv_pages_for)


@pytest.fixture(scope="module")
def golden():
    with gzip.open(GOLDEN / "control_ref.json.gz", "rt") as f:
        return json.load(f)


def _first_diff(got, exp):
    for i, (a, b) in enumerate(zip(got, exp)):
        if a != b:
            return i, a, b
    return min(len(got), len(exp)), None, None


@pytest.mark.parametrize("name", list(control_sim.SCENARIOS))
def test_microbatches_pages_and_admissions_match_the_reference(golden, name):
    got = json.loads(json.dumps(control_sim.run(NS, **control_sim.SCENARIOS[name])))
    exp = golden["scenarios"][name]
    i, a, b = _first_diff(got["microbatches"], exp["microbatches"])
    assert got["microbatches"] == exp["microbatches"], f"microbatch {i}: got {a} want {b}"
    assert got["requests"] == exp["requests"]
    assert got["kv_stats"] == exp["kv_stats"] and got["kept"] == exp["kept"]


@pytest.mark.parametrize("name,kw", [("host_stamps", dict(seed=11)), ("no_stamps", dict(seed=12, with_host=False)),
                                     ("pp8", dict(seed=13, stages=8))])
def test_dispatch_decisions_match_the_reference(golden, name, kw):
    got = json.loads(json.dumps(control_sim.dispatch_trace(dispatch.DispatchRule,
                                                           (dispatch.NOW, dispatch.WAIT, dispatch.NO), **kw)))
    i, a, b = _first_diff(got, golden["dispatch"][name])
    assert got == golden["dispatch"][name], f"decision {i}: got {a} want {b}"


def test_golden_scenarios_reach_the_rules_they_pin(golden):
    """The recorded runs exercise admission waits, LRU evictions, states short of whole blocks, superseded and
    content-keyed contexts, and every forming decision kind."""
    sc = golden["scenarios"]
    waits = {k: sum(r.get("room_wait") is not None for r in v["requests"].values()) for k, v in sc.items()}
    assert waits["plain_cold"] > 0 and waits["good_sessions"] > 0
    assert sc["srpt8k_sessions"]["kv_stats"]["dropped_stale"] > 0
    assert all(sc[k]["kv_stats"]["evicted_sessions"] > 0 for k in ("srpt8k_sessions", "good_sessions",
                                                                    "content_keys"))
    assert sc["good_sessions"]["kv_stats"]["states_short"] > 0
    assert sc["content_keys"]["kv_stats"]["hits"] > 0
    assert {d[1] for d in golden["dispatch"]["host_stamps"]} == {"now", "wait", "no"}


# --- known answers of the reference's tests/test_scheduler.py --------------------------------------------------------

def _make(lengths, mb=8192, in_flight=4, ahead=10, blocks=10_000):
    s = PlainScheduler(KvManager(blocks), mb, in_flight, ahead)
    reqs = [Request(f"r{i}", n) for i, n in enumerate(lengths)]
    for r in reqs:
        s.add(r)
    return s, reqs


def _drain(s, last_stage=3):
    out = []
    while (mb := s.next_microbatch()) is not None:
        out.append([(c.req.req_id, c.start, c.num_tokens, c.is_last) for c in mb])
        for st in range(last_stage + 1):
            s.stage_done(st, last_stage)
    return out


def test_fills_to_the_budget_in_arrival_order():                     # test_scheduler.py:24-29
    s, _ = _make([1024] * 20)
    mbs = _drain(s)
    assert [sum(c[2] for c in mb) for mb in mbs] == [8192, 8192, 4096]
    assert [c[0] for mb in mbs for c in mb] == [f"r{i}" for i in range(20)]


def test_long_prompts_are_cut_into_budget_chunks():                  # test_scheduler.py:32-44
    s, _ = _make([20000, 3000])
    assert _drain(s) == [[("r0", 0, 8192, False)], [("r0", 8192, 8192, False)],
                         [("r0", 16384, 3616, True), ("r1", 0, 3000, True)]]
    s, _ = _make([5000, 5000, 5000])
    assert _drain(s) == [[("r0", 0, 5000, True), ("r1", 0, 3192, False)],
                         [("r1", 3192, 1808, True), ("r2", 0, 5000, True)]]
    s, _ = _make([131072], mb=131072)
    assert _drain(s) == [[("r0", 0, 131072, True)]]


def test_in_flight_limit_and_stage0_dispatch_ahead():                # test_scheduler.py:52-75
    s, _ = _make([8192] * 10, ahead=1)
    assert s.next_microbatch() is not None and s.next_microbatch() is not None
    assert s.next_microbatch() is None
    s.stage_done(0, 3)
    assert s.next_microbatch() is not None
    s.stage_done(0, 3)
    assert s.next_microbatch() is not None
    s.stage_done(0, 3)
    assert s.in_flight == 4 and s.next_microbatch() is None
    s.stage_done(3, 3)
    assert s.next_microbatch() is not None
    s, _ = _make([8192] * 3, ahead=0)
    assert s.next_microbatch() is not None and s.next_microbatch() is None
    s.stage_done(0, 3)
    assert s.next_microbatch() is not None


def test_admission_waits_in_arrival_order_and_resumes():             # test_scheduler.py:78-86
    per = -(-20000 // BLOCK_TOKENS) + STATE_BLOCKS
    s, reqs = _make([20000, 20000, 1000], blocks=per + 7)
    mbs = _drain(s)
    assert {c[0] for mb in mbs for c in mb} == {"r0"}
    assert [r.req_id for r in s.waiting] == ["r1", "r2"]
    s.finish(reqs[0])
    assert _drain(s) == [[("r1", 0, 8192, False)], [("r1", 8192, 8192, False)],
                         [("r1", 16384, 3616, True), ("r2", 0, 1000, True)]]
    assert s.kv.pool.num_free == (per + 7) * PAGES_PER_BLOCK - pages_for(20000) - pages_for(1000)


# --- known answers of the reference's tests/test_kv.py ----------------------------------------------------------------

def _check_pool(kv: KvManager):
    """The charge is exactly the pages handed out, every page and state block once, never the null block."""
    allocs = list(kv.held.values()) + [k.alloc for k in kv.kept.values()]
    used = sum(a.num_pages for a in allocs)
    assert used + kv.pool.num_free == kv.num_blocks * PAGES_PER_BLOCK
    assert kv.hard + kv.kept_charge == used
    pages = [p for a in allocs for p in a.kv_pages]
    pages += [b * PAGES_PER_BLOCK + i for a in allocs for b in a.state_blocks for i in range(PAGES_PER_BLOCK)]
    assert len(set(pages)) == len(pages) and min(pages, default=PAGES_PER_BLOCK) >= PAGES_PER_BLOCK
    assert max(pages, default=0) < (kv.num_blocks + 1) * PAGES_PER_BLOCK
    assert not any(kv.pool.is_free(p) for p in pages)


def test_block_and_page_counts():                                    # test_kv.py:11-19
    assert PAGES_PER_BLOCK * 128 == BLOCK_TOKENS and PAGES_PER_BLOCK == 67
    assert kv_blocks_for(1) == 1 and kv_blocks_for(BLOCK_TOKENS) == 1 and kv_blocks_for(BLOCK_TOKENS + 1) == 2
    assert kv_blocks_for(131072) == 16
    assert kv_pages_for(1) == 1 and kv_pages_for(128) == 1 and kv_pages_for(129) == 2
    assert pages_for(8192) == 64 + STATE_PAGES and STATE_PAGES == STATE_BLOCKS * PAGES_PER_BLOCK


def test_pool_size_counts_out_the_null_block():                      # test_kv.py:22-28
    assert pool_size([7144, 7200, 7144, 7300]) == 7143
    assert pool_size([7144] * 4) * BLOCK_TOKENS == 61_258_368
    assert pool_size([7144] * 4, pool_tokens=15_273_856) == 1781
    with pytest.raises(ValueError):
        pool_size([1, 5])


def test_admit_release_never_hands_out_the_null_block():             # test_kv.py:44-62
    kv = KvManager(20)
    ra, rb, rc = Request("a", 3 * BLOCK_TOKENS), Request("b", 6 * BLOCK_TOKENS), Request("c", 5 * BLOCK_TOKENS)
    a = kv.admit(ra)
    assert len(a.kv_pages) == 3 * PAGES_PER_BLOCK and len(a.state_blocks) == STATE_BLOCKS
    assert 0 not in a.state_blocks and min(a.kv_pages) >= PAGES_PER_BLOCK
    _check_pool(kv)
    assert kv.pool.num_free == 11 * PAGES_PER_BLOCK
    assert kv.admit(rb) is None
    assert kv.admit(rc) is not None and kv.pool.num_free == 0
    kv.release(ra)
    assert kv.pool.num_free == 9 * PAGES_PER_BLOCK
    kv.release(rc)
    assert kv.pool.num_free == 20 * PAGES_PER_BLOCK
    assert kv.fits_ever(14 * BLOCK_TOKENS) and not kv.fits_ever(14 * BLOCK_TOKENS + 1)
    _check_pool(kv)


def test_charge_is_the_prompt_rounded_to_a_page():                   # test_kv.py:65-80
    kv = KvManager(100)
    lens = [1, 127, 128, 129, BLOCK_TOKENS - 1, BLOCK_TOKENS + 1, 3 * BLOCK_TOKENS + 4000]
    for i, n in enumerate(lens):
        a = kv.admit(Request(f"r{i}", n))
        assert len(a.kv_pages) == kv_pages_for(n) and kv._charge[f"r{i}"] == kv_pages_for(n) + STATE_PAGES
        _check_pool(kv)
    assert kv.used_tokens == sum(kv_pages_for(n) * 128 for n in lens) + 7 * STATE_PAGES * 128


def test_short_contexts_share_a_block_of_pages():                    # test_kv.py:83-96
    kv = KvManager(20, keep_sessions=True)
    for i in range(3):
        r = Request(f"r{i}", 1000, session=i)
        assert kv.admit(r) is not None
        kv.release(r)
    assert len(kv.kept) == 3 and kv.stats["evicted_sessions"] == 0
    assert len({p // PAGES_PER_BLOCK for k in kv.kept.values() for p in k.alloc.kv_pages}) == 1
    _check_pool(kv)


def test_page_pool_order_fullest_split_block_first_oldest_whole_block_first():   # test_kv.py:99-118
    pool = PagePool(6)
    a = pool.take_pages(10)
    assert a == list(range(PAGES_PER_BLOCK, PAGES_PER_BLOCK + 10)) and pool.num_whole == 5
    b = pool.take_pages(PAGES_PER_BLOCK)
    assert {p // PAGES_PER_BLOCK for p in b} == {1, 2} and pool.num_whole == 4
    assert pool.take_states(2) == [3, 4] and pool.num_whole == 2
    pool.give_pages(a[:4])
    c = pool.take_pages(5)
    assert c[:4] == a[:4] and c[4] // PAGES_PER_BLOCK == 2
    pool.give_states([3])
    assert pool.num_whole == 3 and pool.take_states(1) == [5]
    pool.give_pages(a[4:] + b + c)
    pool.give_states([4, 5])
    assert pool.num_free == 6 * PAGES_PER_BLOCK and pool.num_whole == 6
    assert pool.can_take(6 * PAGES_PER_BLOCK, 0) and pool.can_take(0, 6) and not pool.can_take(1, 6)


def _churn(seed: int, steps: int = 600, num_blocks: int = 40, keep: bool = True) -> KvManager:
    """Random sessions on a small pool (the reference's test_kv.py:121-150 driver, restated)."""
    rng = random.Random(seed)
    kv = KvManager(num_blocks, keep_sessions=keep)
    running, ctx = [], {}
    for step in range(steps):
        if running and rng.random() < 0.5:
            r = running.pop(rng.randrange(len(running)))
            kv.release(r)
            ctx[r.session] = r.num_tokens
        else:
            s = rng.randrange(16)
            if any(r.session == s for r in running):
                continue
            prev = ctx.get(s, 0)
            n = prev + rng.choice([rng.randrange(1, 600), rng.randrange(1, 3 * BLOCK_TOKENS)])
            r = Request(f"r{step}", n, session=s, prefix_tokens=prev)
            charge_fits = kv.hard + kv.kept_charge + kv.footprint(n) <= kv.capacity
            if kv.fits(r):
                r.cached = kv.allocate(r)
                assert len(kv.held[r.req_id].kv_pages) == kv_pages_for(n)
                running.append(r)
            elif not keep and charge_fits:
                assert kv.pool.num_whole < STATE_BLOCKS
        _check_pool(kv)
        assert kv.hard + kv.kept_charge <= kv.capacity
    return kv


def test_random_sessions_keep_the_charge_equal_to_the_pages_held():  # test_kv.py:153-161
    short = 0
    for seed in range(6):
        kv = _churn(seed)
        assert kv.stats["admitted"] > 150 and kv.stats["hits"] > 10
        short += kv.stats["states_short"]
    assert short > 0


def test_without_kept_contexts_a_request_short_of_whole_blocks_waits():          # test_kv.py:164-171
    for seed in (18, 47):
        kv = _churn(seed, keep=False)
        assert kv.stats["states_short"] > 0 and not kv.kept and kv.stats["evicted_sessions"] == 0


# --- known answers of the reference's tests/test_prefix.py ------------------------------------------------------------

def _rnd(name, session, prefix, new, token_ids=None):
    return Request(name, prefix + new, session=session, prefix_tokens=prefix, token_ids=token_ids)


def _serve(kv, req):
    assert kv.fits(req)
    req.cached = kv.allocate(req)
    kv.release(req)
    return req.cached


@pytest.mark.parametrize("P,A", [(8192, 1024), (32768, 8192), (131072, 1024), (524288, 8192)])
def test_hit_is_the_whole_previous_prompt(P, A):                     # test_prefix.py:34-43
    kv = KvManager(1000, keep_sessions=True)
    assert _serve(kv, _rnd("r0", 1, 0, P)) == 0
    r1 = _rnd("r1", 1, P + 1, A - 1)
    assert kv.peek_hit(r1) == P
    assert _serve(kv, r1) == P and r1.num_tokens - r1.cached == A
    _check_pool(kv)


def test_kept_pages_and_states_move_to_the_next_round():             # test_prefix.py:46-58
    kv = KvManager(100, keep_sessions=True)
    _serve(kv, _rnd("r0", 1, 0, BLOCK_TOKENS + 100))
    kept = kv.kept[1].alloc
    kv_ids, state_ids = list(kept.kv_pages), list(kept.state_blocks)
    r1 = _rnd("r1", 1, BLOCK_TOKENS + 101, 3 * BLOCK_TOKENS)
    r1.cached = kv.allocate(r1)
    a = kv.held["r1"]
    assert len(kv_ids) == PAGES_PER_BLOCK + 1
    assert a.kv_pages[:len(kv_ids)] == kv_ids and a.state_blocks == state_ids
    assert len(a.kv_pages) == kv_pages_for(4 * BLOCK_TOKENS + 101) and 1 not in kv.kept
    _check_pool(kv)


def test_the_kda_state_is_only_at_the_prompt_end():                  # test_prefix.py:61-73 (exact hits)
    kv = KvManager(100, keep_sessions=True)
    _serve(kv, _rnd("r0", 1, 0, 50_000))
    shrunk = _rnd("r1", 1, 49_000, 10)
    assert kv.peek_hit(shrunk) == 0
    assert _serve(kv, shrunk) == 0 and kv.stats["dropped_stale"] == 1
    assert kv.kept[1].tokens == 49_010
    assert kv.peek_hit(_rnd("r2", 1, 49_010, 0)) == 0


def test_content_match_by_token_ids():                               # test_prefix.py:76-82
    kv = KvManager(100, keep_sessions=True)
    ids = list(range(1000))
    _serve(kv, Request("r0", 1000, session="k", token_ids=ids))
    assert kv.peek_hit(Request("r1", 1500, session="k", token_ids=ids + [7] * 500)) == 1000
    assert kv.peek_hit(Request("r2", 1500, session="k", token_ids=ids[:999] + [5] + [7] * 500)) == 0


def test_lru_evicts_whole_sessions_for_running_requests():           # test_prefix.py:85-103
    n = 2 * BLOCK_TOKENS - 100
    per, rest = divmod(pages_for(n), PAGES_PER_BLOCK)
    assert rest == 0
    kv = KvManager(3 * per, keep_sessions=True)
    for s in (1, 2, 3):
        _serve(kv, _rnd(f"s{s}", s, 0, n))
    assert list(kv.kept) == [1, 2, 3] and kv.pool.num_free == 0
    _serve(kv, _rnd("s1b", 1, n + 1, 9))
    assert list(kv.kept) == [2, 3, 1]
    big = _rnd("new", 4, 0, BLOCK_TOKENS * 2 + 5000)
    assert kv.fits(big)
    big.cached = kv.allocate(big)
    assert list(kv.kept) == [1] and kv.stats["evicted_sessions"] == 2 and kv.stats["evicted_tokens"] == 2 * n
    _check_pool(kv)
    assert not kv.fits(_rnd("x", 5, 0, 30 * BLOCK_TOKENS))


def test_chunked_continuation_after_a_hit():                         # test_prefix.py:120-140
    kv = KvManager(1000, keep_sessions=True)
    s = Scheduler(kv, SchedulerConfig(mb_tokens=8192), dispatch_ahead=0)
    r0 = _rnd("r0", 9, 0, 20_000)
    s.add(r0, 0)
    mbs = []
    while (mb := s.next_microbatch(0)) is not None:
        mbs.append([(c.req.req_id, c.start, c.num_tokens, c.is_last) for c in mb])
        s.stage_done(0, 3)
        s.stage_done(3, 3)
    assert mbs == [[("r0", 0, 8192, False)], [("r0", 8192, 8192, False)], [("r0", 16384, 3616, True)]]
    s.finish(r0)
    r1 = _rnd("r1", 9, 20_001, 9000)
    s.add(r1, 0)
    mb1 = s.next_microbatch(0)
    s.stage_done(0, 3)
    mb2 = s.next_microbatch(0)
    assert [(c.start, c.num_tokens) for c in mb1] == [(20_000, 8192)]
    assert [(c.start, c.num_tokens, c.is_last) for c in mb2] == [(28_192, 809, True)]
    assert r1.cached == r1.hbm_tokens == 20_000


def test_server_backlog_counts_new_tokens_without_a_declared_prefix():            # test_prefix.py:143-163
    n = 2 * BLOCK_TOKENS - 100
    per = pages_for(n) // PAGES_PER_BLOCK
    kv = KvManager(2 * per, keep_sessions=True, content_keys=True)
    s = Scheduler(kv, SchedulerConfig(order="srpt", mb_tokens=32768, load_budget=True), dispatch_ahead=0)
    ids = {k: [k * 100_000 + i for i in range(n)] for k in (1, 2, 3)}
    for k in (1, 2, 3):
        _serve(kv, Request(f"s{k}", n, session=kv.find_session(ids[k]), token_ids=ids[k]))
    assert kv.stats["evicted_sessions"] == 1
    for name, k in (("hit", 2), ("evicted", 1), ("first", 9)):
        tok = ids[k] + [7] * 500 if k in ids else [9_000_000 + i for i in range(500)]
        r = Request(name, len(tok), session=kv.find_session(tok), token_ids=tok)
        s.add(r, 0)
        assert r.fresh == 500, (name, r.fresh, r.size)
    assert s.backlog() == 1500


def test_waiting_size_counts_what_is_cached_at_arrival():            # test_prefix.py:166-177
    kv = KvManager(1000, keep_sessions=True)
    s = Scheduler(kv, SchedulerConfig(order="srpt"), dispatch_ahead=0)
    _serve(kv, _rnd("a0", 1, 0, 100_000))
    hit, miss = _rnd("a1", 1, 100_001, 2000), _rnd("b1", 2, 50_001, 500)
    s.add(miss, 0)
    s.add(hit, 0)
    assert (hit.size, miss.size) == (2001, 50_501)
    assert hit.fresh == 2000 and s.backlog() == 2500
    mb = s.next_microbatch(0)
    assert [c.req.req_id for c in mb] == ["a1", "b1"] and mb[0].start == 100_000


# --- this package's additions -------------------------------------------------------------------------------------

def test_budget_rules():
    """The load budget rises linearly from 4,096 tokens at a 1M backlog to mb_tokens at 3M (rounded to nearest);
    the even split caps it at ceil(B / depth) within [512, mb_tokens]."""
    s = Scheduler(KvManager(10), SchedulerConfig(order="srpt", mb_tokens=32768, load_budget=True, even_split=True))
    for backlog, want in [(0, 512), (1_500, 512), (8_000, 2000), (20_000, 4096), (1_000_000, 4096),
                          (2_000_000, 18_432), (3_000_000, 32_768), (9_000_000, 32_768)]:
        s.pending.tokens = backlog
        assert s.budget() == want, (backlog, s.budget(), want)


def test_force_schedule_puts_overdue_requests_first():
    kv = KvManager(1000)
    s = Scheduler(kv, SchedulerConfig(order="srpt", force_after_ms=100.0), dispatch_ahead=10)
    long = Request("long", 20_000)
    s.add(long, 0)
    shorts = [Request(f"s{i}", 1000) for i in range(3)]
    for r in shorts:
        s.add(r, 50_000_000)
    mb = s.next_microbatch(60_000_000)                   # nothing overdue: shortest first, then the long one
    assert [c.req.req_id for c in mb] == ["s0", "s1", "s2", "long"]
    s2 = Scheduler(KvManager(1000), SchedulerConfig(order="srpt", force_after_ms=100.0), dispatch_ahead=10)
    long2 = Request("long", 20_000)
    s2.add(long2, 0)
    for i in range(3):
        s2.add(Request(f"s{i}", 1000), 50_000_000)
    mb = s2.next_microbatch(100_000_000)                 # 100 ms after its arrival the long one goes first
    assert [c.req.req_id for c in mb] == ["long"] and mb[0].num_tokens == 8192


def test_plans_carry_the_pages_the_positions_need():
    """`Scheduler.plan` gives each chunk the KV pages covering [0, start + n), its six state blocks and its token ids,
    and the stage's block contract accepts it."""
    from ssengine_b200.stage import check_blocks

    kv = KvManager(200, keep_sessions=True)
    s = Scheduler(kv, SchedulerConfig(mb_tokens=8192), dispatch_ahead=10)
    rng = np.random.default_rng(0)
    reqs = [Request(f"r{i}", int(n), session=i, token_ids=rng.integers(0, 1000, int(n)).tolist())
            for i, n in enumerate([300, 20_000, 5000])]
    for r in reqs:
        s.add(r, 0)
    k = 0
    while (mb := s.next_microbatch(0)) is not None:
        plan = Scheduler.plan(k, mb)
        check_blocks(plan.chunks, kv.num_blocks + 1)
        for c, spec in zip(plan.chunks, mb):
            assert len(c.kv_pages) == kv_pages_for(c.start + c.num_tokens)
            assert c.kv_pages == spec.req.alloc.kv_pages[:len(c.kv_pages)] and len(c.state_blocks) == STATE_BLOCKS
            assert c.token_ids == spec.req.token_ids[c.start:c.start + c.num_tokens]
        for st in range(4):
            s.stage_done(st, 3)
        k += 1
    assert k == 4


def test_forming_cost_on_the_host():
    """Forming a microbatch over 400 waiting sessions takes well under a millisecond of host time (the plan must
    reach stage 0 ahead of its start)."""
    import time

    kv = KvManager(7143, keep_sessions=True)
    s = Scheduler(kv, scheduler.SCHEDULER_STEPS["good"], dispatch_ahead=10_000, max_in_flight=10_000)
    rng = np.random.default_rng(1)
    for i in range(400):
        s.add(Request(f"q{i}", int(rng.integers(200, 8000)), session=i), 0)
    t = time.perf_counter()
    n = 0
    while s.next_microbatch(0) is not None:
        n += 1
    per = (time.perf_counter() - t) / max(n, 1)
    assert n > 10 and per < 5e-3, (n, per)
