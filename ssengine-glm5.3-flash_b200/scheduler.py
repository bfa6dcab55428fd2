"""Microbatch formation on stage 0's host: which prompt chunks ride the next microbatch (host only).

A pure state machine with no clock of its own: the caller passes `now_ns` and feeds it events (`add` an arrival,
`stage_done` a stage report, `finish` a request whose token is out). `next_microbatch` forms and commits one
microbatch as `ChunkSpec`s; `plan` turns them into the `Plan` / `Chunk` messages a `StageModel` runs.

The rules follow the reference's scheduler so that the same events form the same microbatches chunk for chunk
(ssengine/engine/scheduler.py; switches as `SchedulerConfig`, ssengine/config.py:77-97):
- in flight: at most `max_in_flight` microbatches formed and not done on the last stage, and at most
  `dispatch_ahead` + 1 not done on stage 0 (`can_dispatch`, scheduler.py:520-521); a caller forming ahead names the
  `exiting` in-flight microbatches that leave before the new one starts (not counted in flight or in the backlog);
- admission reserves a request's whole footprint once, at its first chunk (`KvManager`); the first waiting request
  that does not fit stops admission for this microbatch; no preemption;
- order `fifo`: started prompts in start order, then waiting ones in arrival order (scheduler.py:580-591); `srpt`:
  (a) overdue requests first, waiting then started, oldest first; (b) started prompts, fewest remaining tokens first,
  each preceded by the waiting prompts needing no more tokens than it has left, shortest first; (c) the other waiting
  prompts shortest first (scheduler.py:593-617); a waiting prompt's size is the tokens it must compute, fixed at
  arrival; ties by arrival;
- budget: `mb_tokens`; `load_budget`: 4,096 tokens up to a backlog of 1M, rising linearly to `mb_tokens` at 3M
  (rounded to nearest); `even_split`: at most ceil(B / depth), kept in [even_min, mb_tokens] (scheduler.py:561-573),
  the backlog B being the started prompts' unscheduled tokens + the waiting prompts' new tokens + the in-flight
  microbatches' tokens;
- force-schedule (`force_after_ms`): a request that has waited that long since its arrival goes first.
Chunks end at any token; a request's next chunk can ride the next microbatch.

Not restated: the DRAM / SSD tier reads and staged loading (the reference's `pool` argument and its landed / reading
queues), which belong to the tier mover.
"""

from __future__ import annotations

import heapq
from collections import deque
from dataclasses import dataclass

from .messages import Chunk, Plan
from .pagepool import Allocation, KvManager, kv_pages_for

MB_TOKENS = 8192
MAX_IN_FLIGHT = 4


@dataclass
class SchedulerConfig:
    """One switch per step of the reference's scheduler (ssengine/config.py:77-89), same names and defaults."""
    order: str = "fifo"                   # "fifo" or "srpt"
    mb_tokens: int = MB_TOKENS            # largest microbatch
    load_budget: bool = False             # 4,096 tokens up to a 1M backlog, mb_tokens at 3M, linear between
    load_budget_low: int = 4096
    backlog_lo: int = 1_000_000
    backlog_hi: int = 3_000_000
    even_split: bool = False              # also at most ceil(B / depth), at least even_min
    even_min: int = 512
    depth: int = MAX_IN_FLIGHT
    force_after_ms: float | None = None   # a request waiting this long goes first


SCHEDULER_STEPS = {
    "plain": SchedulerConfig(),
    "srpt8k": SchedulerConfig(order="srpt"),
    "budget": SchedulerConfig(order="srpt", mb_tokens=32768, load_budget=True),
    "even": SchedulerConfig(order="srpt", mb_tokens=32768, load_budget=True, even_split=True),
    "good": SchedulerConfig(order="srpt", mb_tokens=32768, load_budget=True, even_split=True, force_after_ms=60_000.0),
}


@dataclass(eq=False)
class Request:
    """A prompt to prefill (the reference's `Request` fields the scheduler and the KV manager read and set)."""
    req_id: str
    num_tokens: int                    # the whole prompt
    arrival_ns: int = 0
    token_ids: list[int] | None = None
    session: object = None             # kept-context key (a session id, or a content key from `find_session`)
    prefix_tokens: int = 0             # declared prefix shared with the session's previous context
    backlog_prefix: int | None = None  # no declared prefix: `KvManager.shared_prefix` at arrival
    cached: int = 0                    # prompt tokens already in KV at admission
    computed: int = 0                  # prompt tokens scheduled so far
    alloc: Allocation | None = None
    seq: int = -1
    size: int = 0                      # tokens to compute, as ranked at arrival
    hbm_tokens: int = 0
    admit_ns: int | None = None
    room_wait_ns: int | None = None    # first time it headed the order and did not fit
    hit_memo: tuple | None = None
    admit_info: dict | None = None
    output_token: int | None = None
    epoch: int = 0                     # which of its session's contexts the prompt continues (a session load's token
                                       # stream restarts at its context cap)

    @property
    def remaining(self) -> int:
        return self.num_tokens - self.cached - self.computed

    @property
    def fresh(self) -> int:
        """New tokens: what the request adds to the backlog while it waits (beyond its declared or shared prefix)."""
        return self.num_tokens - (self.prefix_tokens if self.backlog_prefix is None else self.backlog_prefix)


@dataclass
class ChunkSpec:
    req: Request
    start: int                         # tokens of the request already in KV (cached + earlier chunks)
    num_tokens: int

    @property
    def is_last(self) -> bool:
        return self.start + self.num_tokens == self.req.num_tokens


class PendingQueue:
    """Waiting requests in a fixed order (a key fixed at arrival), with lazy removal; `tokens` sums their new
    tokens."""

    def __init__(self, key):
        self._key = key
        self._heap: list = []
        self._members: set[int] = set()
        self.tokens = 0

    def __len__(self) -> int:
        return len(self._members)

    def __iter__(self):
        return (e[-1] for e in sorted(self._heap, key=lambda e: e[:-1]) if id(e[-1]) in self._members)

    def push(self, r: Request):
        heapq.heappush(self._heap, (*self._key(r), r))
        self._members.add(id(r))
        self.tokens += r.fresh

    def peek(self) -> Request | None:
        h = self._heap
        while h and id(h[0][-1]) not in self._members:
            heapq.heappop(h)
        return h[0][-1] if h else None

    def pop(self) -> Request:
        r = self.peek()
        heapq.heappop(self._heap)
        self._members.discard(id(r))
        self.tokens -= r.fresh
        return r

    def remove(self, r: Request) -> bool:
        if id(r) not in self._members:
            return False
        self._members.discard(id(r))
        self.tokens -= r.fresh
        return True


class OverdueQueue:
    """Requests that waited past the force-schedule bound, oldest first, out of the pending order."""

    def __init__(self, after_ms: float):
        self.after_ns = int(after_ms * 1e6)
        self.arrivals: deque[Request] = deque()     # every arrival, in arrival order
        self.q: deque[Request] = deque()
        self.tokens = 0

    def is_overdue(self, r: Request, now_ns: int) -> bool:
        return now_ns - r.arrival_ns >= self.after_ns

    def promote(self, pending: PendingQueue, now_ns: int):
        while self.arrivals and self.is_overdue(self.arrivals[0], now_ns):
            r = self.arrivals.popleft()
            if pending.remove(r):                   # still waiting (not admitted meanwhile)
                self.q.append(r)
                self.tokens += r.fresh

    def pop(self) -> Request:
        r = self.q.popleft()
        self.tokens -= r.fresh
        return r


class Scheduler:
    def __init__(self, kv: KvManager, cfg: SchedulerConfig | None = None, pool=None,
                 max_in_flight: int = MAX_IN_FLIGHT, dispatch_ahead: int = 1):
        if pool is not None:
            raise NotImplementedError("DRAM / SSD tiers are not part of this scheduler")
        self.kv = kv
        self.cfg = cfg = cfg or SchedulerConfig()
        if cfg.order not in ("fifo", "srpt"):
            raise ValueError(f"scheduler order {cfg.order!r} (want 'fifo' or 'srpt')")
        self.srpt = cfg.order == "srpt"
        self.max_in_flight = max_in_flight
        self.dispatch_ahead = dispatch_ahead
        self.pending = PendingQueue((lambda r: (r.size, r.seq)) if self.srpt else (lambda r: (r.seq,)))
        self.overdue = OverdueQueue(cfg.force_after_ms) if cfg.force_after_ms else None
        self.started: list[Request] = []     # admitted, prompt not fully scheduled; start order
        self.in_flight = 0                   # formed, last stage not done
        self.on_stage0 = 0                   # formed, stage 0 not done
        self.in_flight_tokens = 0
        self._mb_tokens: deque[int] = deque()
        self._seq = 0
        self._out: list[ChunkSpec] = []
        self.stats = dict(microbatches=0)

    # --- events ---------------------------------------------------------------------------------------------------

    def add(self, req: Request, now_ns: int | None = None):
        """A request arrived; its rank (tokens to compute beyond its hit) is fixed now."""
        req.seq = self._seq
        self._seq += 1
        if now_ns is not None and not req.arrival_ns:
            req.arrival_ns = now_ns
        req.size = req.num_tokens - self.kv.peek_hit(req)
        if req.token_ids is not None and not req.prefix_tokens:
            req.backlog_prefix = self.kv.shared_prefix(req)
        self.pending.push(req)
        if self.overdue is not None:
            self.overdue.arrivals.append(req)

    def stage_done(self, stage: int, last_stage: int):
        if stage == 0:
            self.on_stage0 -= 1
        if stage == last_stage:
            self.in_flight -= 1
            self.in_flight_tokens -= self._mb_tokens.popleft()

    def finish(self, req: Request):
        """The request's token is out: its context stays kept, or its blocks go back."""
        self.kv.release(req)

    @property
    def waiting(self) -> list[Request]:
        return list(self.pending)

    def has_work(self) -> bool:
        return bool(self.started or len(self.pending) or (self.overdue and self.overdue.q))

    def state(self) -> dict:
        kv = self.kv
        return dict(in_flight=self.in_flight, started=len(self.started), pending=len(self.pending),
                    overdue=len(self.overdue.q) if self.overdue is not None else 0, hard=kv.hard,
                    kept=kv.kept_charge, capacity=kv.capacity)

    # --- decisions ------------------------------------------------------------------------------------------------

    def can_dispatch(self, exiting: int = 0) -> bool:
        return self.in_flight - exiting < self.max_in_flight and self.on_stage0 <= self.dispatch_ahead

    def backlog(self, exiting: int = 0) -> int:
        gone = sum(list(self._mb_tokens)[:exiting])
        return (sum(r.remaining for r in self.started) + self.pending.tokens
                + (self.overdue.tokens if self.overdue else 0) + self.in_flight_tokens - gone)

    def budget(self, exiting: int = 0) -> int:
        cfg = self.cfg
        b = cfg.mb_tokens
        if not (cfg.load_budget or cfg.even_split):
            return b
        backlog = self.backlog(exiting)
        if cfg.load_budget:
            rise = min(max((backlog - cfg.backlog_lo) / (cfg.backlog_hi - cfg.backlog_lo), 0.0), 1.0)
            b = min(b, cfg.load_budget_low + int((cfg.mb_tokens - cfg.load_budget_low) * rise + 0.5))
        if cfg.even_split:
            b = min(b, min(max(-(-backlog // cfg.depth), cfg.even_min), cfg.mb_tokens))
        return b

    def next_microbatch(self, now_ns: int = 0, exiting: int = 0) -> list[ChunkSpec] | None:
        """Form and commit the next microbatch, or None (nothing to run, or no room in flight)."""
        if not self.can_dispatch(exiting):
            return None
        if self.overdue is not None:
            self.overdue.promote(self.pending, now_ns)
        self._out = []
        budget = self.budget(exiting)
        if self.srpt:
            self._form_srpt(budget, now_ns)
        else:
            self._form_fifo(budget, now_ns)
        chunks, self._out = self._out, []
        if not chunks:
            return None
        tokens = sum(c.num_tokens for c in chunks)
        self.in_flight += 1
        self.on_stage0 += 1
        self.in_flight_tokens += tokens
        self._mb_tokens.append(tokens)
        self.stats["microbatches"] += 1
        return chunks

    # --- forming ----------------------------------------------------------------------------------------------------

    def _emit(self, r: Request, n: int):
        self._out.append(ChunkSpec(r, r.cached + r.computed, n))
        r.computed += n

    def _form_fifo(self, budget: int, now_ns: int):
        keep = []
        for r in self.started:
            n = min(r.remaining, budget)
            if n:
                self._emit(r, n)
                budget -= n
            if r.remaining:
                keep.append(r)
        self.started = keep
        self._admit(budget, now_ns)

    def _form_srpt(self, budget: int, now_ns: int):
        od = self.overdue
        ranked = []
        for r in self.started:
            late = od is not None and od.is_overdue(r, now_ns)
            ranked.append((not late, r.arrival_ns if late else r.remaining, r))
        ranked.sort(key=lambda e: (e[0], e[1]))      # stable: ties keep start order
        self.started = []                            # admissions below append here
        if od is not None and budget > 0:
            budget -= self._admit(budget, now_ns, overdue_only=True)
        keep = []
        for not_late, _, r in ranked:
            left = r.remaining
            if not_late and budget > 0:
                budget -= self._admit(budget, now_ns, no_longer_than=left)
            n = min(left, budget)
            if n:
                self._emit(r, n)
                budget -= n
            if n < left:
                keep.append(r)
        if budget > 0:
            self._admit(budget, now_ns)
        self.started = keep + self.started

    def _head(self, overdue_only: bool) -> tuple[bool, Request | None]:
        """(from the overdue queue, the request) heading the admission order."""
        if self.overdue is not None and self.overdue.q:
            return True, self.overdue.q[0]
        if overdue_only:
            return False, None
        return False, self.pending.peek()

    def _admit(self, budget: int, now_ns: int, no_longer_than: int | None = None, overdue_only: bool = False) -> int:
        """Admit waiting prompts into `budget`: overdue ones, then the pending order, stopping at the first pending
        one with more than `no_longer_than` tokens to compute or whose footprint does not fit. Returns the budget
        taken."""
        left = budget
        while left > 0:
            late, r = self._head(overdue_only)
            if r is None:
                break
            need = r.num_tokens - self.kv.peek_hit(r)
            if not late and no_longer_than is not None and need > no_longer_than:
                break
            n = min(need, left)
            if n == 0:
                break
            if not self.kv.fits(r):
                if r.room_wait_ns is None:
                    r.room_wait_ns = now_ns
                break
            (self.overdue.pop() if late else self.pending.pop())
            r.cached = r.hbm_tokens = self.kv.allocate(r)
            r.alloc = self.kv.held[r.req_id]
            r.admit_ns = now_ns
            self._emit(r, n)
            left -= n
            if n < need:
                self.started.append(r)
        return budget - left

    # --- messages ---------------------------------------------------------------------------------------------------

    @staticmethod
    def plan(mb_id: int, chunks: list[ChunkSpec], token_ids=None) -> Plan:
        """The stage message of a formed microbatch: each chunk's KV pages up to its last position, its state blocks,
        and its token ids, as the reference's controller sends them (ssengine/runtime/controller.py:609-614). The ids
        come from the request's `token_ids`, or from `token_ids(req, start, end)` when given."""
        out = []
        for c in chunks:
            r, end = c.req, c.start + c.num_tokens
            if token_ids is not None:
                ids = [int(t) for t in token_ids(r, c.start, end)]
            else:
                ids = None if r.token_ids is None else [int(t) for t in r.token_ids[c.start:end]]
            out.append(Chunk(r.req_id, c.start, c.num_tokens, list(r.alloc.kv_pages[:kv_pages_for(end)]),
                             list(r.alloc.state_blocks), c.is_last, ids))
        return Plan(mb_id, out)


class PlainScheduler(Scheduler):
    """The plain scheduler: first come first served with a fixed budget."""

    def __init__(self, kv: KvManager, mb_tokens: int, max_in_flight: int = MAX_IN_FLIGHT, dispatch_ahead: int = 1):
        super().__init__(kv, SchedulerConfig(mb_tokens=mb_tokens), None, max_in_flight, dispatch_ahead)
