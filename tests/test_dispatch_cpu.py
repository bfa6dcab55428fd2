"""The dispatch rule's known answers: the cases of the reference's tests/test_dispatch.py with their expected values,
restated against `ssengine_b200.dispatch`, and its pipeline behaviour in an event-driven model of four stages with the
GPU in-flight gate, report latency and plan delivery (this file's own model, written to the same description:
stage 0 starts microbatch k at max(plan arrived, stage 0 free, exit of k - 4))."""

import heapq
import random

import pytest

from ssengine_b200.dispatch import NO, NOW, WAIT, DispatchRule, HostPredictor, StagePredictor

MS = 1_000_000


def _report(rule, mb, spans, stages=(0, 1, 2, 3)):
    for s in stages:
        a, b = spans[s]
        rule.stage_done(s, mb, int(a * MS), int(b * MS))


def test_predictor_ewma_per_size_bucket():                            # test_dispatch.py:13-23
    p = StagePredictor(alpha=0.5)
    assert p.predict_ns(8192) is None
    p.observe(8192, 57 * MS)
    assert p.predict_ns(8192) == pytest.approx(57 * MS)
    assert p.predict_ns(4096) == pytest.approx(28.5 * MS)
    p.observe(8192, 59 * MS)
    assert p.predict_ns(8192) == pytest.approx(58 * MS)
    p.observe(1024, 2 * MS)
    assert p.predict_ns(1000) == pytest.approx(1000 * 2 * MS / 1024)
    assert p.predict_ns(8000) == pytest.approx(8000 * 58 * MS / 8192)


def test_cold_start_forms_with_stage0_free_and_room():                # test_dispatch.py:26-33
    r = DispatchRule(4, 3.0)
    assert r.decide(0) == (NOW, None)
    r.dispatched(0, 0, 8192)
    assert r.decide(1 * MS) == (NO, None)
    _report(r, 0, [(0, 50), (50, 100), (100, 150), (150, 200)], stages=(0,))
    assert r.decide(51 * MS) == (NOW, None)


def test_forms_lead_and_host_time_before_the_projected_start():        # test_dispatch.py:41-49
    r = DispatchRule(4, 3.0)
    r.dispatched(0, 0, 8192)
    _report(r, 0, [(1, 51), (51, 101), (101, 151), (151, 201)], stages=(0,))
    r.dispatched(1, 52 * MS, 8192)
    assert r.decide(60 * MS) == (WAIT, 99 * MS)
    assert r.decide(99 * MS) == (NOW, None) and r.exiting == 0


def test_the_gate_moves_the_start_to_the_exit_of_k_minus_4():         # test_dispatch.py:52-68
    r = DispatchRule(4, 0.0)
    r.dispatched(0, 0, 1000)
    _report(r, 0, [(0, 10), (10, 20), (20, 30), (30, 130)])
    r.host.rate = {r.host.bucket(1000): 0.0}
    for k in range(1, 5):
        r.dispatched(k, 10 * MS * k, 1000)
        r.stage_done(0, k, 10 * MS * k, 10 * MS * (k + 1))
    p = r.project()
    assert p["ends"][1][3] == pytest.approx(230 * MS) and p["ends"][4][3] == pytest.approx(530 * MS)
    assert p["start"] == pytest.approx(230 * MS) and p["exiting"] == 1
    assert r.decide(100 * MS) == (WAIT, 230 * MS)


def test_host_time_learned_only_when_stage0_was_ready():              # test_dispatch.py:222-229
    r = DispatchRule(4, 3.0)
    r.dispatched(0, 0, 8192)
    _report(r, 0, [(0.7, 50), (50, 100), (100, 150), (150, 200)], stages=(0,))
    assert r.host.predict_ns(8192) == pytest.approx(0.7 * MS)
    r.dispatched(1, 10 * MS, 8192)
    _report(r, 1, [(50, 100), (100, 150), (150, 200), (200, 250)], stages=(0,))
    assert r.host.predict_ns(8192) == pytest.approx(0.7 * MS)


def test_a_stage0_report_after_the_last_stages_report():              # test_dispatch.py:232-244
    r = DispatchRule(4, 3.0)
    for k in range(3):
        r.dispatched(k, k * MS, 4096)
    _report(r, 0, [(0, 10), (10, 20), (20, 30), (30, 40)])
    _report(r, 1, [(10, 20), (20, 30), (30, 40), (40, 50)], stages=(1, 2, 3))
    assert 1 not in r.flight and list(r.on_stage0) == [2]
    _report(r, 2, [(20, 30), (30, 40), (40, 50), (50, 60)], stages=(0,))
    _report(r, 1, [(10, 20), (20, 30), (30, 40), (40, 50)], stages=(0,))
    assert not r.on_stage0 and list(r.flight) == [2]
    assert r.decide(61 * MS)[0] in (NOW, WAIT)


def test_host_time_from_worker_stamps_on_every_microbatch():           # test_dispatch.py:261-271
    r = DispatchRule(4, 3.0)
    r.dispatched(0, 0, 8192)
    r.stage_done(0, 0, int(20 * MS), int(100 * MS), (int(1 * MS), int(1 * MS), int(16 * MS), int(16 * MS), 0))
    assert r.host.predict_ns(8192) == pytest.approx(20 * MS)
    r.dispatched(1, int(50 * MS), 8192)
    r.stage_done(0, 1, int(102 * MS), int(180 * MS), (int(51 * MS), int(51 * MS), int(70 * MS), int(70 * MS), 0))
    assert r.host.predict_ns(8192) == pytest.approx(0.75 * 20 * MS + 0.25 * 22 * MS)


def test_host_time_leaves_out_the_in_flight_gate_wait():              # test_dispatch.py:274-289
    r = DispatchRule(4, 3.0)
    for k in range(4):
        r.dispatched(k, k * int(MS), 4096)
    for k in range(4):
        r.stage_done(0, k, int((10 + 30 * k) * MS), int((40 + 30 * k) * MS))
    r.stage_done(3, 0, int(150 * MS), int(200 * MS))
    r.dispatched(4, int(150 * MS), 4096)
    before = r.host.predict_ns(4096)
    r.stage_done(0, 4, int(200 * MS) + 10_000, int(230 * MS),
                 (int(151 * MS), int(151 * MS), int(155 * MS), int(155 * MS), 0))
    want = int(1 * MS) + int(4 * MS) + 10_000
    assert r.host.predict_ns(4096) == pytest.approx(want if before is None else 0.75 * before + 0.25 * want)


def test_forming_allows_the_host_time_bound_at_the_recent_largest_size():   # test_dispatch.py:292-304
    h = HostPredictor()
    for ns in (10 * MS, 20 * MS, 10 * MS, 20 * MS):
        h.observe(32768, ns)
    assert h.bound_ns(32768) > h.predict_ns(32768) + 5 * MS
    r = DispatchRule()
    r.host.observe(32768, 20 * MS)
    r.host.observe(512, 1 * MS)
    for i, t in enumerate((32768, 512, 512)):
        r.dispatched(i, 0, t)
    assert r.form_host_ns() == pytest.approx(20 * MS)


# --- pipeline behaviour ---------------------------------------------------------------------------------------------

def _targets(n_mb, stage_ns, depth=4):
    """Stage-0 starts of an ideal pipeline: max(stage 0 free, exit of k - depth), no host time."""
    free, starts, exits = [0] * 4, [], []
    for k in range(n_mb):
        t = max(free[0], exits[k - depth] if k >= depth else 0)
        starts.append(t)
        end = t
        for s in range(4):
            end = (end if s == 0 else max(end, free[s])) + stage_ns[s]
            free[s] = end
        exits.append(end)
    return starts


def _pipeline(rule, n_mb=60, stage_ms=10.0, report_ms=0.3, form_ms=0.8, stage_time=None, report_delay=None, depth=4):
    """Run `n_mb` microbatches through the model; rule None forms on reports (stage 0 free, < depth in flight).
    Returns (stage-0 starts, peak in flight on the GPU, ends per microbatch)."""
    base = [int(x * MS) for x in (stage_ms if isinstance(stage_ms, list) else [stage_ms] * 4)]
    ev, seq = [], [0]
    free, last_rep = [0] * 4, [0] * 4
    starts, ends = {}, {}
    st = dict(k=0, in_flight=0, timer=None, on0=[])

    def push(t, kind, data=None):
        seq[0] += 1
        heapq.heappush(ev, (int(t), seq[0], kind, data))

    def form(now):
        while st["k"] < n_mb:
            if rule is None:
                if st["in_flight"] >= depth or st["on0"]:
                    return
            else:
                d, at = rule.decide(now)
                if d == WAIT:
                    if st["timer"] != at:
                        st["timer"] = at
                        push(at, "timer")
                    return
                if d == NO:
                    return
                rule.dispatched(st["k"], now, 8192)
            k = st["k"]
            st["k"] += 1
            st["in_flight"] += 1
            st["on0"].append(k)
            push(now + form_ms * MS, "plan", k)

    push(0, "timer")
    while ev:
        t, _, kind, data = heapq.heappop(ev)
        if kind == "timer":
            st["timer"] = None
            form(t)
        elif kind == "plan":
            k = data
            begin = max(t, free[0], ends[k - depth][3] if k >= depth else 0)
            starts[k], ends[k] = [], []
            end = begin
            for s in range(4):
                b = begin if s == 0 else max(end, free[s])
                end = b + (int(stage_time(k, s) * MS) if stage_time else base[s])
                free[s] = end
                starts[k].append(b)
                ends[k].append(end)
                at = max(end + int((report_delay(k, s) if report_delay else report_ms) * MS), last_rep[s])
                last_rep[s] = at
                push(at, "done", (s, k))
        else:
            s, k = data
            if s == 0:
                st["on0"].remove(k)
            if s == 3:
                st["in_flight"] -= 1
            if rule is not None:
                rule.stage_done(s, k, starts[k][s], ends[k][s])
            form(t)
    marks = sorted([(starts[k][0], 1) for k in starts] + [(ends[k][3], -1) for k in starts])
    cur = peak = 0
    for _, d in marks:
        cur += d
        peak = max(peak, cur)
    return [starts[k][0] for k in range(n_mb)], peak, ends


def _gaps(starts, first):
    return [b - a for a, b in zip(starts[first:], starts[first + 1:])]


def test_stage0_starts_back_to_back_as_an_ideal_pipeline():           # test_dispatch.py:181-188
    s0, peak, _ = _pipeline(DispatchRule(4, 3.0))
    want = _targets(60, [10 * MS] * 4)
    assert peak <= 4
    assert _gaps(s0, 8) == pytest.approx(_gaps(want, 8), abs=1)
    old, old_peak, _ = _pipeline(None)
    assert old_peak <= 4 and old[-1] - want[-1] > 50 * MS       # forming on reports pays latency every microbatch


def test_a_slower_later_stage_sets_the_pace_through_the_gate():       # test_dispatch.py:191-197
    sts = [10.0, 10.0, 12.0, 10.0]
    s0, peak, _ = _pipeline(DispatchRule(4, 3.0), n_mb=80, stage_ms=sts)
    want = _targets(80, [int(x * MS) for x in sts])
    assert peak <= 4 and _gaps(s0, 10) == pytest.approx(_gaps(want, 10), abs=1)


def test_reports_slower_than_a_microbatch():                          # test_dispatch.py:200-205
    s0, peak, _ = _pipeline(DispatchRule(4, 1.0), n_mb=80, stage_ms=2.0, report_ms=3.0, form_ms=0.8)
    want = _targets(80, [2 * MS] * 4)
    assert peak <= 4 and _gaps(s0, 20) == pytest.approx(_gaps(want, 20), abs=1)


def test_noisy_stage_times_leave_stage0_almost_never_idle():          # test_dispatch.py:208-219
    rnd = random.Random(7)
    table = {(k, s): 10.0 * rnd.uniform(0.9, 1.1) for k in range(80) for s in range(4)}
    s0, peak, ends = _pipeline(DispatchRule(4, 2.0), n_mb=80, stage_time=lambda k, s: table[(k, s)])
    assert peak <= 4
    idle = sum(max(s0[k] - max(ends[k - 1][0], ends[k - 4][3] if k >= 4 else 0), 0) for k in range(10, 80))
    assert idle < 0.002 * (s0[79] - s0[10])


def test_reports_in_any_order_across_stages():                        # test_dispatch.py:247-258
    rnd = random.Random(11)
    table = {(k, s): 10.0 * rnd.uniform(0.7, 1.3) for k in range(300) for s in range(4)}
    delay = {(k, s): (rnd.uniform(50, 500) if s == 0 and rnd.random() < 0.05 else rnd.uniform(0.1, 3.0))
             for k in range(300) for s in range(4)}
    rule = DispatchRule(4, 3.0)
    s0, peak, _ = _pipeline(rule, n_mb=300, stage_time=lambda k, s: table[(k, s)],
                            report_delay=lambda k, s: delay[(k, s)])
    assert len(s0) == 300 and peak <= 4 and not rule.flight and not rule.on_stage0
