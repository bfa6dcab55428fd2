"""A deterministic event-driven driver of a control plane (scheduler + KV manager) over a model pipeline: test
infrastructure shared by the golden-fixture script (which runs the reference's control plane) and the tests (which run
this package's).

`run(ns, **scenario)`: `ns` carries the implementation's `Request`, `KvManager`, `Scheduler`, `SchedulerConfig` and
`kv_pages_for`. Sessions arrive closed-loop (each round after the previous round's token plus a think time); every
stage runs microbatches in order, stage 0 starting microbatch k no earlier than microbatch k - max_in_flight leaves
the last stage (the GPU gate); a stage's time is a fixed cost plus per-token and per-(token x context) terms. The
record lists every formed microbatch (time, chunks with run-length encoded KV pages and state blocks), every request's
admission and finish, and the final counters: two control planes that decide alike give identical records.
"""

from __future__ import annotations

import heapq

import numpy as np

HOST_NS = 1_000_000           # plan formed -> stage 0 may start
EDGE_NS = 300_000             # stage s end -> stage s + 1 may start
STAGE_SCALE = (12, 11, 11, 11, 11, 11, 11, 11)


def rle(pages) -> list[list[int]]:
    """[[first, length], ...] of runs of consecutive page ids."""
    out: list[list[int]] = []
    for p in pages:
        p = int(p)
        if out and out[-1][0] + out[-1][1] == p:
            out[-1][1] += 1
        else:
            out.append([p, 1])
    return out


def stage_ns(stage: int, chunks) -> int:
    tok = sum(n for _, s, n in chunks)
    att = sum(n * (2 * s + n) for _, s, n in chunks) // 40
    return (150_000 + 6_000 * tok + att) * STAGE_SCALE[stage] // 12


def run(ns, *, seed: int, sessions: int, rounds: int, cfg: dict, num_blocks: int, keep_sessions: bool,
        content_keys: bool = False, max_in_flight: int = 4, dispatch_ahead: int = 1, stages: int = 4,
        first_median: int = 8192, first_max: int = 131_072, append_median: int = 600, append_max: int = 8192,
        ctx_cap: int = 131_072, think_ms: float = 500.0, stagger_ms: float = 20.0, restart_p: float = 0.0,
        max_mb: int = 100_000) -> dict:
    rng = np.random.default_rng(seed)
    kv = ns.KvManager(num_blocks, keep_sessions=keep_sessions, **({"content_keys": True} if content_keys else {}))
    sched = ns.Scheduler(kv, ns.SchedulerConfig(**cfg), None, max_in_flight, dispatch_ahead)
    last = stages - 1
    events: list = []
    order = [0]

    def push(t, kind, payload):
        heapq.heappush(events, (int(t), order[0], kind, payload))
        order[0] += 1

    # per session: rounds left, previous prompt (token ids or length)
    sess = [{"left": rounds, "ids": None, "len": 0, "n": 0} for _ in range(sessions)]

    def new_round(i: int, now: int):
        s = sess[i]
        if s["left"] == 0:
            return
        s["left"] -= 1
        if s["len"] == 0:
            new = int(np.clip(rng.lognormal(np.log(first_median), 1.0), 1, first_max))
            prev = 0
        else:
            new = int(np.clip(rng.lognormal(np.log(append_median), 1.0), 1, append_max))
            prev = s["len"] + 1                        # the previous prompt and its output token
            if prev + new > ctx_cap or rng.random() < restart_p:
                prev = 0                               # the context starts over (its kept one is superseded)
        name = f"s{i}r{s['n']}"
        s["n"] += 1
        if content_keys:
            base = s["ids"] + [int(s["tok"])] if prev else []
            ids = base + [int(x) for x in rng.integers(0, 150_000, new)]
            r = ns.Request(name, len(ids), token_ids=ids)
            r.session = kv.find_session(ids)
            s["ids"], s["len"] = ids, len(ids)
        else:
            r = ns.Request(name, prev + new, session=i if keep_sessions else None, prefix_tokens=prev)
            s["len"] = prev + new
        r.output_token = (i * 7919 + s["n"] * 104_729) % 150_000
        s["tok"] = r.output_token
        sched.add(r, now)
        info[name] = {"arrival": now}

    info: dict = {}
    mbs: list = []
    exits: list[int] = []
    free = [0] * stages
    owner = {}
    for i in range(sessions):
        push(i * stagger_ms * 1e6, "arrive", i)
    now = 0
    while events or sched.has_work():
        if events:
            now = events[0][0]
            while events and events[0][0] == now:
                _, _, kind, payload = heapq.heappop(events)
                if kind == "arrive":
                    new_round(payload, now)
                elif kind == "stage":
                    st, k = payload
                    sched.stage_done(st, last)
                    if st == last:
                        for r in mbs[k]["done"]:
                            sched.finish(r)
                            info[r.req_id]["finish"] = now
                            push(now + int(rng.exponential(think_ms) * 1e6), "arrive", owner[r.req_id])
        elif not sched.can_dispatch():
            raise RuntimeError("no event pending and no room in flight")
        formed_any = False
        while len(mbs) < max_mb and (mb := sched.next_microbatch(now)) is not None:
            formed_any = True
            k = len(mbs)
            chunks = []
            for c in mb:
                r, end = c.req, c.start + c.num_tokens
                owner.setdefault(r.req_id, int(r.req_id[1:].split("r")[0]))
                chunks.append([r.req_id, int(c.start), int(c.num_tokens), bool(c.is_last),
                               rle(r.alloc.kv_pages[:ns.kv_pages_for(end)]), [int(b) for b in r.alloc.state_blocks]])
                if r.req_id in info and "admit" not in info[r.req_id]:
                    info[r.req_id].update(admit=now, cached=int(r.cached), size=int(r.size), fresh=int(r.fresh),
                                          hit_kind=(r.admit_info or {}).get("hit_kind"), room_wait=r.room_wait_ns)
            spec = [(c[0], c[1], c[2]) for c in chunks]
            t0 = max(now + HOST_NS, free[0], exits[k - max_in_flight] if k >= max_in_flight else 0)
            ends = []
            for st in range(stages):
                begin = t0 if st == 0 else max(ends[-1] + EDGE_NS, free[st])
                ends.append(begin + stage_ns(st, spec))
                free[st] = ends[-1]
                push(ends[-1], "stage", (st, k))
            exits.append(ends[-1])
            mbs.append({"t": now, "chunks": chunks, "done": [c.req for c in mb if c.is_last],
                        "kv": [int(kv.hard), int(kv.kept_charge), int(kv.pool.num_free), int(kv.pool.num_whole)],
                        "budget_backlog": int(sched.backlog())})
        if not events and not formed_any and sched.has_work():
            raise RuntimeError("control plane stalled: work waiting, nothing in flight")
        if len(mbs) >= max_mb:
            break
    return {"microbatches": [{k: v for k, v in m.items() if k != "done"} for m in mbs],
            "requests": info,
            "kv_stats": {k: int(kv.stats[k]) for k in ("admitted", "hits", "hit_tokens", "evicted_sessions",
                                                       "evicted_tokens", "dropped_stale", "peak_hard",
                                                       "states_short")},
            "kept": len(kv.kept)}


# The scenarios the golden fixture records (small enough to run in seconds on the host).
SCENARIOS = {
    # BASELINE config 4's cold prompts through the plain scheduler on a pool that makes admissions wait
    "plain_cold": dict(seed=1, sessions=48, rounds=1, cfg=dict(), num_blocks=30, keep_sessions=False),
    # kept sessions, SRPT at 8k, a pool that evicts kept contexts and runs short of whole blocks
    "srpt8k_sessions": dict(seed=2, sessions=24, rounds=6, cfg=dict(order="srpt"), num_blocks=70, keep_sessions=True,
                            first_median=4096, ctx_cap=65_536, restart_p=0.15),
    # the reference's "good" step (load budget, even split, force-schedule), force bound short enough to bind
    "good_sessions": dict(seed=3, sessions=40, rounds=5, num_blocks=120, keep_sessions=True, first_median=6000,
                          cfg=dict(order="srpt", mb_tokens=32768, load_budget=True, even_split=True,
                                   force_after_ms=400.0, backlog_lo=20_000, backlog_hi=200_000), think_ms=200.0),
    # FIFO forming only when stage 0 is free, two in flight
    "fifo_gate": dict(seed=4, sessions=16, rounds=4, cfg=dict(), num_blocks=90, keep_sessions=True,
                      max_in_flight=2, dispatch_ahead=0, first_median=3000),
    # server mode: prompts carry token ids, kept contexts found by content
    "content_keys": dict(seed=5, sessions=10, rounds=4, cfg=dict(order="srpt", mb_tokens=16384), num_blocks=48,
                         keep_sessions=True, content_keys=True, first_median=2000, first_max=12_000,
                         append_max=4000, ctx_cap=24_000, restart_p=0.2),
}


def dispatch_trace(rule_cls, consts, *, seed: int, steps: int = 160, stages: int = 4, max_in_flight: int = 4,
                   with_host: bool = True) -> list:
    """Drive a dispatch rule over a noisy model pipeline (reports arrive late and out of stage order) and record every
    decision: [now, decision, at, exiting, projected start]. `consts`: (NOW, WAIT, NO)."""
    NOW, WAIT, NO = consts
    rng = np.random.default_rng(seed)
    rule = rule_cls(max_in_flight=max_in_flight, lead_ms=3.0, num_stages=stages)
    events: list = []
    order = [0]

    def push(t, kind, payload):
        heapq.heappush(events, (int(t), order[0], kind, payload))
        order[0] += 1

    free = [0] * stages
    exits: dict[int, int] = {}
    ticks: set[int] = set()
    out = []
    mb = 0
    now = 0
    push(0, "tick", None)
    while events and mb < steps:
        now, _, kind, payload = heapq.heappop(events)
        if kind == "report":
            rule.stage_done(*payload)
        else:
            ticks.discard(now)
        d, at = rule.decide(now)
        proj = rule.projected["start"] if rule.projected else None
        out.append([int(now), d, at, rule.exiting, proj])
        if d == NOW:
            tokens = int(rng.choice([512, 2048, 4096, 8192, 8192, 16384, 32768]))
            rule.dispatched(mb, now, tokens)
            host = int(rng.uniform(0.5, 3.0) * 1e6)
            start = max(now + host, free[0], exits.get(mb - max_in_flight, 0))
            for st in range(stages):
                dur = int(tokens * rng.uniform(5_000, 7_000) * (12 if st == 0 else 11) / 12) + 200_000
                begin = start if st == 0 else max(end + EDGE_NS, free[st])
                end = begin + dur
                free[st] = end
                if st == stages - 1:
                    exits[mb] = end
                stamps = None
                if st == 0 and with_host:
                    plan = now + int(host * 0.3)
                    call = plan + 10_000
                    stamps = (plan, call, call + int(host * 0.4), now + host)
                push(end + int(rng.uniform(0.7, 1.2) * 1e6) + st * 1000, "report", (st, mb, begin, end, stamps))
            mb += 1
            if now + 1 not in ticks:
                ticks.add(now + 1)
                push(now + 1, "tick", None)
        elif d == WAIT and at not in ticks:
            ticks.add(at)
            push(at, "tick", None)
    return out
