"""Serving a session load through the pipeline: stage 0's host loop and the loop of the other stages (host only).

The reference's controller process (ssengine/runtime/controller.py) forms microbatches with its scheduler and sends
each plan to every stage worker; the workers report stage ends, and the last stage's tokens close the requests. Here
the same roles run inside the stage processes of one `torch.distributed` job:
- stage 0's host runs `Controller`: arrivals of a `SessionLoad` -> `Scheduler.add`; `next_microbatch` -> a `Plan`
  (token ids for stage 0 only) -> every other stage through the job's c10d store (`StoreChannel`) -> stage 0's own
  forward; reports -> `stage_done` / `finish`; a finished round's token time minus its arrival is its TTFT, and the
  session's next round arrives a think time later (closed loop);
- every other stage runs `serve_stage`: take plan k from the store, run it, repeat until the stop plan;
- a `Reporter` thread per stage waits for each microbatch's completion in order (a CUDA event, or whatever `done`
  waits on) and emits {mb, stage, start_ns, end_ns, tokens}; the other stages' reports go back to stage 0 through
  the store (the last stage's carry the tokens; all of them feed the dispatch rule when one forms the plans), stage
  0's own stay local.
Plans and reports are small host messages; the activations never leave the GPUs (the P2P stage edge, `edge.py`),
and stage 0's GPU holds itself to the edge's in-flight limit whatever the host forms ahead.

`SessionLoad` is BASELINE config 5's synthetic load: closed-loop sessions; each round appends lognormal (median 600,
max 8k) new token ids to the session's growing context (cap 128k, then the context starts over); think time
exponential (mean 5 s). Token ids are a counter-based hash of (seed, session, epoch, position), so the same position
always carries the same id and prefix-cache hits are exact.
"""

from __future__ import annotations

import heapq
import pickle
import queue
import threading
import time
from dataclasses import dataclass, field

import numpy as np

from .messages import Chunk, Plan
from .scheduler import Request, Scheduler


def context_ids(seed: int, session: int, epoch: int, start: int, end: int, vocab: int) -> np.ndarray:
    """Token ids at positions [start, end) of a session's context: splitmix64 of (seed, session, epoch, position)
    modulo the vocabulary, int64."""
    key = np.uint64((((seed * 1_000_003 + session) * 65_537 + epoch) & 0xFFFFFFFF) << 32)
    z = np.arange(start, end, dtype=np.uint64) + key
    z = z * np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    z = z ^ (z >> np.uint64(31))
    return (z % np.uint64(vocab)).astype(np.int64)


@dataclass
class SessionLoad:
    """Closed-loop synthetic sessions (see the module docstring). `start_ctx_max`: a session's first round brings a
    context uniform in [0, start_ctx_max) plus one append (so that contexts are spread from the start);
    `stagger_s`: first arrivals spread uniformly over [0, stagger_s)."""
    sessions: int = 400
    seed: int = 0
    vocab: int = 151_552
    append_median: int = 600
    append_max: int = 8192
    ctx_cap: int = 131_072
    think_s: float = 5.0
    start_ctx_max: int = 16_384
    stagger_s: float = 5.0
    _rng: np.random.Generator = field(init=False, repr=False)

    def __post_init__(self):
        self._rng = np.random.default_rng(self.seed)
        self._ctx = [0] * self.sessions
        self._epoch = [0] * self.sessions
        self._round = [0] * self.sessions

    def first_arrivals(self, t0_ns: int) -> list[tuple[int, int]]:
        return [(t0_ns + int(self._rng.uniform(0.0, self.stagger_s) * 1e9), i) for i in range(self.sessions)]

    def think_ns(self) -> int:
        return int(self._rng.exponential(self.think_s) * 1e9)

    def next_request(self, i: int, arrival_ns: int) -> Request:
        add = int(np.clip(self._rng.lognormal(np.log(self.append_median), 1.0), 1, self.append_max))
        if self._round[i] == 0:
            prev = 0
            n = (int(self._rng.integers(0, self.start_ctx_max)) if self.start_ctx_max > 0 else 0) + add
        else:
            prev = self._ctx[i] + 1                      # the previous prompt and the token it got
            n = prev + add
            if n > self.ctx_cap:                         # the context starts over: the kept one is superseded
                self._epoch[i] += 1
                prev, n = 0, add
        self._ctx[i] = n
        r = Request(f"s{i}.{self._round[i]}", n, arrival_ns=arrival_ns, session=i, prefix_tokens=prev,
                    epoch=self._epoch[i])
        self._round[i] += 1
        return r

    def ids(self, req: Request, start: int, end: int) -> np.ndarray:
        return context_ids(self.seed, req.session, req.epoch, start, end, self.vocab)


def for_later_stages(plan: Plan) -> Plan:
    """The plan without token ids (only stage 0 embeds them)."""
    return Plan(plan.mb_id, [Chunk(c.req_id, c.start, c.num_tokens, c.kv_pages, c.state_blocks, c.is_last, None)
                             for c in plan.chunks], list(plan.tier_ops))


class Reporter(threading.Thread):
    """Waits, in order, for each submitted microbatch to finish on this stage and hands `sink` a report
    {mb, stage, start_ns, end_ns, tokens}. `done()` blocks until the microbatch is done and returns its busy time in
    ns; `tokens()` (last stage) returns its greedy tokens on the host."""

    def __init__(self, stage: int, sink, clock=time.monotonic_ns, init=None):
        super().__init__(daemon=True, name=f"reporter-{stage}")
        self.stage, self.sink, self.clock, self._init = stage, sink, clock, init
        self.q: queue.Queue = queue.Queue()
        self.error: BaseException | None = None
        self.start()

    def submit(self, mb: int, done, tokens=None):
        self.q.put((mb, done, tokens))

    def close(self):
        self.q.put(None)
        self.join()
        if self.error is not None:
            raise self.error

    def run(self):
        try:
            if self._init is not None:
                self._init()
            while (item := self.q.get()) is not None:
                mb, done, tokens = item
                busy = int(done())
                end = self.clock()
                toks = None if tokens is None else [int(t) for t in tokens()]
                self.sink({"mb": mb, "stage": self.stage, "start_ns": end - busy, "end_ns": end, "tokens": toks})
        except BaseException as e:                       # surfaced by the owner's loop and by close()
            self.error = e


def wait_key(store, key: str, give_up_s: float, poll_s: float = 2e-4) -> None:
    """Wait until `key` exists by polling `check` (a c10d store client holds its lock for the whole of a blocking
    `wait`, which would stall the other threads of this process that share the client, such as a stage's
    `Reporter`). The poll interval grows to 2 ms while nothing comes."""
    t0, dt = time.monotonic(), poll_s
    while not store.check([key]):
        if time.monotonic() - t0 > give_up_s:
            raise TimeoutError(f"store key {key!r} not set within {give_up_s:.0f} s")
        time.sleep(dt)
        dt = min(2 * dt, 2e-3)


class StageFailed(RuntimeError):
    """Another stage's loop failed (its message came through the store)."""


class StoreChannel:
    """Plans from stage 0 to the other stages, and the other stages' reports back, over a c10d store (the job's
    rendezvous store, or any `torch.distributed.Store`). Keys: plan/<k>, rep/<stage>/<k>, and err/<stage> for a
    stage whose loop failed."""

    def __init__(self, store, give_up_s: float = 900.0):
        self.store = store
        self.give_up_s = give_up_s
        self.next_report: dict[int, int] = {}

    def put_plan(self, k: int, plan: Plan | None):
        self.store.set(f"plan/{k}", pickle.dumps(plan))

    def get_plan(self, k: int) -> Plan | None:
        """Plan k, or None for the stop plan; raises `StageFailed` when stage 0 reports a failure first, and
        TimeoutError after `give_up_s` without either."""
        key, t0, dt = f"plan/{k}", time.monotonic(), 2e-4
        while not self.store.check([key]):
            if self.store.check(["err/0"]):
                raise StageFailed(f"stage 0 failed: {self.store.get('err/0').decode()}")
            if time.monotonic() - t0 > self.give_up_s:
                raise TimeoutError(f"store key {key!r} not set within {self.give_up_s:.0f} s")
            time.sleep(dt)
            dt = min(2 * dt, 2e-3)
        return pickle.loads(self.store.get(key))

    def put_error(self, stage: int, what: str):
        self.store.set(f"err/{stage}", what.encode())

    def error(self, stages) -> tuple[int, str] | None:
        """(stage, message) of the first of `stages` that reported a failure, else None."""
        for st in stages:
            if self.store.check([f"err/{st}"]):
                return st, self.store.get(f"err/{st}").decode()
        return None

    def drop_plan(self, k: int):
        self.store.delete_key(f"plan/{k}")

    def put_report(self, rep: dict):
        self.store.set(f"rep/{rep['stage']}/{rep['mb']}", pickle.dumps(rep))

    def poll_reports(self, stages) -> list[dict]:
        """Every report that has arrived from `stages`, each stage's in microbatch order."""
        out = []
        for st in stages:
            k = self.next_report.get(st, 0)
            while self.store.check([f"rep/{st}/{k}"]):
                key = f"rep/{st}/{k}"
                out.append(pickle.loads(self.store.get(key)))
                self.store.delete_key(key)
                k += 1
            self.next_report[st] = k
        return out


class Controller:
    """Stage 0's host loop (see the module docstring). Without `rule` a microbatch is formed whenever the scheduler's
    in-flight limits allow; with a `dispatch.DispatchRule` (built for the GPU's in-flight gate, the scheduler built
    with `rule.sched_limits`), one is formed when the rule's projection of the pipeline says NOW, with the microbatches
    projected to leave by its start not counted (`exiting`): the reference controller's forming
    (ssengine/runtime/dispatch.py), so that rounds arriving until then can ride it."""

    def __init__(self, sched: Scheduler, load: SessionLoad, num_stages: int, clock=time.monotonic_ns,
                 poll_s: float = 2e-4, rule=None):
        self.sched, self.load, self.num_stages = sched, load, num_stages
        self.rule = rule
        self.decisions = {"now": 0, "wait": 0, "no": 0}
        self.last = num_stages - 1
        self.clock, self.poll_s = clock, poll_s
        self.local: queue.Queue = queue.Queue()          # stage 0's own reports
        self.rounds: list[dict] = []
        self.microbatches: list[dict] = []
        self._plans: dict[int, list] = {}
        self._arrivals: list = []
        self._reqs: dict[str, Request] = {}
        self._stop_arrivals = None

    def _arrive(self, t: int, i: int):
        if self._stop_arrivals is None or t < self._stop_arrivals:
            heapq.heappush(self._arrivals, (t, i))

    def _on_report(self, rep: dict):
        k, st = rep["mb"], rep["stage"]
        mb = self.microbatches[k]
        mb[f"end{st}"], mb[f"busy{st}"] = rep["end_ns"], rep["end_ns"] - rep["start_ns"]
        if self.rule is not None:            # stage 0's host stamps (delivered, prepare called, prepared, ready)
            self.rule.stage_done(st, k, rep["start_ns"], rep["end_ns"], mb.get("host_ns") if st == 0 else None)
        if st == 0 or st == self.last:
            self.sched.stage_done(st, self.last)
        if st != self.last:
            return
        done = self._plans.pop(k)
        toks = rep["tokens"] or []
        if len(toks) != len(done):
            raise RuntimeError(f"microbatch {k}: {len(toks)} tokens for {len(done)} finished prompts")
        for req, tok in zip(done, toks):
            req.output_token = tok
            self.sched.finish(req)
            self.rounds.append({"req": req.req_id, "arrival_ns": req.arrival_ns, "token_ns": rep["end_ns"],
                                "tokens": req.num_tokens, "cached": req.cached, "fresh": req.fresh,
                                "admit_ns": req.admit_ns})
            del self._reqs[req.req_id]
            self._arrive(rep["end_ns"] + self.load.think_ns(), req.session)

    def run(self, step, reporter: Reporter, channel: StoreChannel | None, *, duration_s: float, warm_s: float,
            drain_s: float = 60.0, stall_s: float = 300.0) -> dict:
        """Serve the load for `duration_s` (arrivals stop then; rounds already arrived are served, up to `drain_s`
        more), then send the stop plan. `step(plan) -> (done, tokens)` runs stage 0's forward of one plan; `reporter`
        is stage 0's `Reporter` whose sink is `self.local.put`; `channel` reaches the other stages (None at N = 1).
        Watchdog: with microbatches in flight and no report for `stall_s`, raise with the scheduler's state (a stage
        that died or stopped reporting). A stage whose loop failed reports it through the channel (checked every 50
        ms): this raises `StageFailed`. On any failure here the other stages get the failure and a stop plan, so that
        their loops end instead of waiting for plans."""
        try:
            return self._run(step, reporter, channel, duration_s, warm_s, drain_s, stall_s)
        except BaseException as e:
            if channel is not None and self.last > 0:
                channel.put_error(0, f"{type(e).__name__}: {e}")
                channel.put_plan(len(self.microbatches), None)
            raise

    def _run(self, step, reporter, channel, duration_s, warm_s, drain_s, stall_s) -> dict:
        sched, load = self.sched, self.load
        t0 = self.clock()
        last_report = last_check = t0
        end, measure_from = t0 + int(duration_s * 1e9), t0 + int(warm_s * 1e9)
        self._stop_arrivals = end
        for t, i in load.first_arrivals(t0):
            self._arrive(t, i)
        k = 0
        while True:
            now = self.clock()
            busy = False
            while self._arrivals and self._arrivals[0][0] <= now:
                t, i = heapq.heappop(self._arrivals)
                r = load.next_request(i, t)
                self._reqs[r.req_id] = r
                sched.add(r, t)
                busy = True
            reps = []
            while not self.local.empty():
                reps.append(self.local.get())
            if channel is not None and self.last > 0:
                reps += channel.poll_reports(range(1, self.num_stages))
            if channel is not None and self.last > 0 and now - last_check > 50_000_000:
                last_check = now
                err = channel.error(range(1, self.num_stages))
                if err is not None:
                    raise StageFailed(f"stage {err[0]} failed: {err[1]}")
            if reps:
                last_report = now
            elif sched.in_flight and now - last_report > int(stall_s * 1e9):
                raise RuntimeError(f"no stage report for {stall_s:.0f} s with microbatches in flight: "
                                   f"{sched.state()}, {len(self.microbatches)} formed")
            elif not sched.in_flight:
                last_report = now
            for rep in sorted(reps, key=lambda x: (x["mb"], x["stage"])):
                self._on_report(rep)
                if channel is not None and rep["stage"] == self.last and self.last > 0:
                    channel.drop_plan(rep["mb"])
                busy = True
            if reporter.error is not None:
                raise reporter.error
            while True:
                if self.rule is not None:
                    d, _ = self.rule.decide(now)
                    self.decisions[d] += 1
                    if d != "now":
                        break
                    chunks = sched.next_microbatch(now, self.rule.exiting)
                else:
                    chunks = sched.next_microbatch(now)
                if chunks is None:
                    break
                plan = Scheduler.plan(k, chunks, token_ids=load.ids)
                plan.tier_ops = sched.kv.take_ops()              # copies recorded since the last plan, in order
                self._plans[k] = [c.req for c in chunks if c.is_last]
                self.microbatches.append({"mb": k, "formed_ns": now, "tokens": plan.num_tokens,
                                          "chunks": len(plan.chunks)})
                if channel is not None and self.last > 0:
                    channel.put_plan(k, for_later_stages(plan))
                if self.rule is not None:
                    self.rule.dispatched(k, now, plan.num_tokens)
                # stage 0 runs in this process: the plan is delivered and prepared inside `step`, so every stamp is
                # the call and the rule's launch term (GPU start - the later of the call, stage 0's previous end and
                # the gate) measures forming -> first kernel on a free stage 0
                t_call = self.clock()
                self.microbatches[-1]["host_ns"] = (t_call, t_call, t_call, t_call)
                done, tokens = step(plan)
                reporter.submit(k, done, tokens)
                k += 1
                busy = True
                now = self.clock()
            if now >= end and sched.in_flight == 0 and not self._arrivals:
                if not sched.has_work() or now >= end + int(drain_s * 1e9):
                    break
            if not busy:
                time.sleep(self.poll_s)
        if channel is not None and self.last > 0:
            channel.put_plan(k, None)
        return self.summary(t0, measure_from, end)

    def summary(self, t0: int, measure_from: int, end: int) -> dict:
        win = [r for r in self.rounds if measure_from <= r["arrival_ns"] < end]
        span = (end - measure_from) / 1e9
        ttft = np.array([(r["token_ns"] - r["arrival_ns"]) / 1e9 for r in win])
        q = (lambda p: float(np.percentile(ttft, p))) if ttft.size else (lambda p: None)
        tok = sum(r["tokens"] for r in win)
        cached = sum(r["cached"] for r in win)
        mbs = [m for m in self.microbatches if measure_from <= m["formed_ns"] < end]
        return {
            "rounds": len(win), "rounds_per_s": len(win) / span if span > 0 else None,
            "ttft_s": {"p50": q(50), "p90": q(90), "p99": q(99), "max": float(ttft.max()) if ttft.size else None},
            "computed_tok_s": sum(m["tokens"] for m in mbs) / span if span > 0 else None,
            "new_tok_s": sum(r["fresh"] for r in win) / span if span > 0 else None,
            "prefix_hit_share": cached / tok if tok else None,
            "microbatches": len(self.microbatches), "unfinished": len(self._reqs),
            "window_s": span, "all_rounds": len(self.rounds),
            "forming": "dispatch rule" if self.rule is not None else "when the in-flight limits allow",
            "decisions": dict(self.decisions) if self.rule is not None else None,
        }


def serve_stage(step, channel: StoreChannel, reporter: Reporter) -> int:
    """A stage > 0: run plans 0, 1, ... from stage 0 until the stop plan. Returns the microbatches run. A failure
    here is reported to stage 0 through the channel before it propagates; a failure of stage 0 (its message, then
    the stop plan) raises `StageFailed` here."""
    k = 0
    try:
        while (plan := channel.get_plan(k)) is not None:
            if reporter.error is not None:
                raise reporter.error
            done, tokens = step(plan)
            reporter.submit(k, done, tokens)
            k += 1
        err = channel.error([0])
        if err is not None:
            raise StageFailed(f"stage 0 failed: {err[1]}")
        reporter.close()
    except StageFailed:
        raise
    except BaseException as e:
        channel.put_error(reporter.stage, f"{type(e).__name__}: {e}")
        raise
    return k


def cuda_step(worker, device):
    """`step(plan)` over a `StageWorker` built with events=True: launches the stage's work for the plan and returns
    (done, tokens): `done` waits for the forward (and the token copy) and returns the forward's device time; `tokens`
    reads the greedy tokens copied to pinned host memory (last stage)."""
    import torch

    def step(plan):
        out = worker.step(plan)
        e0, e1 = worker.spans.pop()
        host = None
        if out is not None:
            host = torch.empty(out.numel(), dtype=torch.int64, pin_memory=True)
            host.copy_(out, non_blocking=True)
        e2 = torch.cuda.Event()
        e2.record()

        def done():
            e2.synchronize()
            return e0.elapsed_time(e1) * 1e6

        return done, (None if host is None else host.numpy)

    return step
