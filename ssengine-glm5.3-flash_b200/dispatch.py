"""When stage 0's host forms the next microbatch (host only, pure: the caller passes the clock).

The in-flight limit itself is enforced on the GPU: stage 0's stream waits, before microbatch k, until the last stage
has finished microbatch k - `max_in_flight` (the stage edge's exits counter, `edge.py`). A plan may therefore reach
stage 0 early, and forming it on stage-end reports alone would leave stage 0 idle for the report latency plus the
plan's host time every microbatch. So the rule projects the pipeline instead (the reference's
ssengine/runtime/dispatch.py, restated so that the same reports give the same decisions):
- per stage, a per-token EWMA (alpha 0.25) of measured compute time per power-of-two size bucket (`StagePredictor`);
  an unmeasured bucket takes the nearest measured one (ties to the smaller); a later stage without a sample in a
  bucket that stage 0 has takes stage 0's rate for it;
- the host time from forming to the stage-0 start: an EWMA per size bucket of each plan's delivery + prepare + launch,
  GPU waits left out, and of its absolute deviation; forming allows the mean plus two deviations at the largest of
  the last four plans' sizes (`HostPredictor`, default 1 ms before any sample);
- each in-flight plan's stage ends are projected (reported ends where known) through the gate; the next microbatch
  starts at T = max(stage 0 free, exit of microbatch next - `max_in_flight`) and is formed at T - host - `lead_ms`,
  with the plans projected to have left by T counted as `exiting`;
- backstops by reports: form only with at most 2 plans not done on stage 0 and at most `max_in_flight` + 1 in flight;
  before any stage has a sample, only with stage 0 free and fewer than `max_in_flight` in flight.
"""

from __future__ import annotations

NOW, WAIT, NO = "now", "wait", "no"


def size_bucket(tokens: int) -> int:
    return max(tokens, 1).bit_length()


def _nearest(keys, b: int) -> int:
    return min(keys, key=lambda k: (abs(k - b), k))


class StagePredictor:
    """EWMA of ns per token, per power-of-two size bucket."""

    def __init__(self, alpha: float = 0.25):
        self.alpha = alpha
        self.rate: dict[int, float] = {}

    bucket = staticmethod(size_bucket)

    def observe(self, tokens: int, compute_ns: int):
        if tokens <= 0:
            return
        b, r = size_bucket(tokens), compute_ns / tokens
        old = self.rate.get(b)
        self.rate[b] = r if old is None else (1 - self.alpha) * old + self.alpha * r

    def predict_ns(self, tokens: int) -> float | None:
        if not self.rate:
            return None
        return self.rate[_nearest(self.rate, size_bucket(tokens))] * tokens


class HostPredictor:
    """EWMA of a time (not a rate) per size bucket, and of its absolute deviation."""

    def __init__(self, alpha: float = 0.25):
        self.alpha = alpha
        self.rate: dict[int, float] = {}        # bucket -> mean ns
        self.dev: dict[int, float] = {}

    bucket = staticmethod(size_bucket)

    def observe(self, tokens: int, ns: int):
        b, a = size_bucket(tokens), self.alpha
        if b in self.rate:
            d = abs(ns - self.rate[b])
            self.dev[b] = (1 - a) * self.dev.get(b, d) + a * d
            self.rate[b] = (1 - a) * self.rate[b] + a * ns
        else:
            self.rate[b] = ns

    def predict_ns(self, tokens: int) -> float | None:
        return self.rate[_nearest(self.rate, size_bucket(tokens))] if self.rate else None

    def bound_ns(self, tokens: int) -> float | None:
        """The mean plus two deviations."""
        if not self.rate:
            return None
        k = _nearest(self.rate, size_bucket(tokens))
        return self.rate[k] + 2 * self.dev.get(k, 0.0)


class DispatchRule:
    DEFAULT_HOST_NS = 1_000_000

    def __init__(self, max_in_flight: int = 4, lead_ms: float = 3.0, num_stages: int = 4):
        self.max_in_flight = max_in_flight
        self.lead_ns = int(lead_ms * 1e6)
        self.num_stages = num_stages
        self.stage_pred = [StagePredictor() for _ in range(num_stages)]
        self.host = HostPredictor()
        self.on_stage0: dict[int, None] = {}         # formed, stage 0 not reported done (mb order)
        self.flight: dict[int, list] = {}            # mb -> [formed ns, tokens, reported end per stage or None]
        self.exits: dict[int, int] = {}              # mb -> reported last-stage end (the last few)
        self.last_end_ns: int | None = None          # latest stage-0 end reported
        self.stage_end = [0] * num_stages
        self.last_tokens = 0
        self.recent_tokens: list[int] = []
        self.next_mb = 0
        self.projected: dict | None = None

    @property
    def cap(self) -> int:
        """In-flight count by reports the scheduler must allow (reports lag the GPU gate)."""
        return self.max_in_flight + 2

    @property
    def sched_limits(self) -> tuple[int, int]:
        """The scheduler's (max_in_flight, dispatch_ahead)."""
        return self.max_in_flight, 2

    @property
    def exiting(self) -> int:
        return self.projected["exiting"] if self.projected else 0

    # --- events -----------------------------------------------------------------------------------------------------

    def dispatched(self, mb_id: int, now_ns: int, tokens: int):
        self.on_stage0[mb_id] = None
        self.flight[mb_id] = [now_ns, tokens, [None] * self.num_stages]
        self.last_tokens = tokens
        self.recent_tokens = (self.recent_tokens + [tokens])[-4:]
        self.next_mb = mb_id + 1

    def _exit_known(self, mb_id: int):
        """A reported exit time; None: long gone or never existed; False: still in flight."""
        if mb_id < 0:
            return None
        if mb_id in self.flight:
            return False
        return self.exits.get(mb_id)

    def stage_done(self, stage: int, mb_id: int, start_ns: int, end_ns: int, host_ns: tuple | None = None):
        """A stage's report of microbatch `mb_id` (reports of different stages may arrive in any order). `host_ns`:
        stage 0's host stamps (plan received, prepare called, prepared, launch ready), which make every microbatch a
        host-time sample."""
        self.stage_end[stage] = max(self.stage_end[stage], end_ns)
        for k in [k for k in self.on_stage0 if k <= mb_id]:
            del self.on_stage0[k]
        f = self.flight.get(mb_id)
        if f is None:
            return
        formed_ns, tokens, ends = f
        self.stage_pred[stage].observe(tokens, end_ns - start_ns)
        ends[stage] = end_ns
        if stage == 0:
            gate = self._exit_known(mb_id - self.max_in_flight)
            if host_ns is not None:
                plan, call, prep, ready = host_ns[:4]
                launch = start_ns - max(ready, self.last_end_ns or 0, gate or 0)
                self.host.observe(tokens, max(plan - formed_ns, 0) + max(prep - call, 0) + max(launch, 0))
            elif max(self.last_end_ns or 0, gate or 0) <= formed_ns and gate is not False:
                self.host.observe(tokens, max(start_ns - formed_ns, 0))   # it found stage 0 ready
            self.last_end_ns = max(self.last_end_ns or 0, end_ns)
        if stage == self.num_stages - 1:
            del self.flight[mb_id]
            self.exits[mb_id] = end_ns
            for old in [k for k in self.exits if k < mb_id - 2 * self.max_in_flight]:
                del self.exits[old]

    # --- projection -------------------------------------------------------------------------------------------------

    def stage_ns(self, stage: int, tokens: int) -> float | None:
        p, p0 = self.stage_pred[stage], self.stage_pred[0]
        b = size_bucket(tokens)
        if stage > 0 and b not in p.rate and b in p0.rate:
            return p0.rate[b] * tokens
        return p.predict_ns(tokens) if p.rate else p0.predict_ns(tokens)

    def host_ns(self, tokens: int) -> float:
        h = self.host.predict_ns(tokens)
        return self.DEFAULT_HOST_NS if h is None else h

    def form_host_ns(self) -> float:
        h = self.host.bound_ns(max(self.recent_tokens, default=self.last_tokens))
        return self.DEFAULT_HOST_NS if h is None else h

    def project(self) -> dict | None:
        """{"ends": {mb: [end per stage]}, "start": next start ns, "exiting": n}, or None while a stage has no
        sample."""
        n, depth = self.num_stages, self.max_in_flight
        ends: dict[int, list[float]] = {}
        free = [float(t) for t in self.stage_end]

        def exit_of(mb: int) -> float:
            return ends[mb][-1] if mb in ends else float(self.exits.get(mb, 0))

        for mb in sorted(self.flight):
            formed_ns, tokens, rep = self.flight[mb]
            e: list[float] = []
            for s in range(n):
                if rep[s] is not None:
                    t = float(rep[s])
                else:
                    c = self.stage_ns(s, tokens)
                    if c is None:
                        return None
                    begin = (max(formed_ns + self.host_ns(tokens), free[0], exit_of(mb - depth)) if s == 0
                             else max(e[s - 1], free[s]))
                    t = begin + c
                e.append(t)
                free[s] = t
            ends[mb] = e
        start = max(free[0], exit_of(self.next_mb - depth))
        return {"ends": ends, "start": start, "exiting": sum(1 for mb in ends if ends[mb][-1] <= start)}

    def decide(self, now_ns: int) -> tuple[str, int | None]:
        """(NOW, None): form now; (WAIT, t): form at host time t; (NO, None): wait for a report. After NOW, `exiting`
        is the number of in-flight plans (oldest first) that leave before the new one starts."""
        self.projected = None
        in_flight = len(self.flight)
        if len(self.on_stage0) > 2 or in_flight > self.max_in_flight + 1:
            return NO, None
        p = self.project() if self.flight else {"ends": {}, "start": 0.0, "exiting": 0}
        if p is None:
            self.projected = {"start": None, "exiting": 0}
            return (NOW, None) if not self.on_stage0 and in_flight < self.max_in_flight else (NO, None)
        if in_flight - p["exiting"] >= self.max_in_flight:
            return NO, None
        self.projected = {"start": p["start"], "exiting": p["exiting"]}
        at = int(p["start"] - self.form_host_ns() - self.lead_ns)
        return (NOW, None) if now_ns >= at else (WAIT, at)
