"""The control plane's block pool and exact prefix cache (host only, no device memory).

One block-id space serves every stage (block 0 is the null block). A block is 67 KV pages of 128 tokens, or one KDA
state; a request holds ceil(L / 128) pages for its prompt of L tokens plus six whole state blocks, reserved when its
first chunk is scheduled and never preempted. A finished prompt can stay as its session's kept context (its pages and
the KDA state after its last token): the session's next round takes them over and computes only what follows. Kept
contexts yield to running requests, least recently used first, a whole context at a time.

The rules follow the reference's control plane so that the same arrivals give the same pages (ssengine/engine/kv.py):
- footprint = kv pages + 6 x 67 pages (`pages_for`, kv.py:79-81), charged against num_blocks x 67 pages;
- page hand-out (`PagePool`, kv.py:120-244): KV pages come from partly used blocks first, the fullest first (lowest
  block id on ties, lowest page first inside a block); a whole free block is split only when no partly used block
  has a free page; whole free blocks (for KV or for a state) go out in the order they became whole, oldest first;
  a request's KV pages are taken before its state blocks, and an allocation is given back pages first;
- a hit is exact (kv.py:102-117): the prompt must start with the whole kept context and go beyond it (by token ids
  when the request has them, else by its declared prefix), since the KDA state exists only at the context's end;
- admission (`fits`, kv.py:349-380): the charge must fit once kept contexts (not the request's own) are evicted; when
  it fits without evicting but fewer than six whole blocks are free for new states, one more kept context is evicted
  for them, and with none left the request waits;
- eviction (`_make_room`, kv.py:598-615): least recently used kept contexts go until the charge fits and the pool can
  hand out the pages and states.

Not restated: the simulator-only token ledger and partial hits (kv.py `accounting="tokens"`, `partial_hits`), which
exist to replay another system's targets, and the reference's tier hooks (write-back ahead of eviction, loading area,
pins). A DRAM tier of this package's own design (`tier.DramTier`) can sit below as `lower`: it takes every kept
context HBM evicts, and a round whose session's context it holds is admitted with a miss's footprint and a read of
that context (`peek_hit` and `allocate` count it as a hit); without `lower` every rule above is the reference's.

The pool is implemented with per-block free-page bitmasks, a heap of partly used blocks keyed (free pages, block) and
a heap of whole blocks keyed by the time they became whole, both with lazy invalidation.
"""

from __future__ import annotations

import heapq
from collections import Counter, OrderedDict
from dataclasses import dataclass

import numpy as np

from .kvpages import BLOCK_TOKENS, PAGE_TOKENS, PAGES_PER_BLOCK

NULL_BLOCK = 0
STATE_BLOCKS = 6                                   # state_blocks[0..4]: KDA groups g2..g6; [5]: kpool tail
STATE_PAGES = STATE_BLOCKS * PAGES_PER_BLOCK       # 402
SESSION_KEY_TOKENS = 64                            # content key of a kept context: its first 64 token ids
_FULL = (1 << PAGES_PER_BLOCK) - 1


def kv_pages_for(tokens: int) -> int:
    """KV pages of a context of `tokens` tokens."""
    return -(-int(tokens) // PAGE_TOKENS)


def kv_blocks_for(tokens: int) -> int:
    """Blocks a context of `tokens` tokens spans."""
    return -(-int(tokens) // BLOCK_TOKENS)


def pages_for(tokens: int) -> int:
    """A request's footprint in pages: its KV pages plus its state blocks' pages."""
    return kv_pages_for(tokens) + STATE_PAGES


def pool_size(ready_blocks, pool_tokens: int | None = None) -> int:
    """Usable blocks: the smallest stage's block count minus the null block, optionally capped by a token count."""
    n = min(ready_blocks) - 1
    if pool_tokens is not None:
        n = min(n, pool_tokens // BLOCK_TOKENS)
    if n < 1:
        raise ValueError(f"KV pool has no usable block (ready={list(ready_blocks)}, pool_tokens={pool_tokens})")
    return n


def prefix_content(token_ids, n: int) -> np.ndarray:
    """The first n token ids as int32 (what a kept context is compared with)."""
    return np.asarray(token_ids[:n], dtype=np.int32)


def session_key(token_ids, n: int | None = None) -> bytes:
    """Content key of a context: the bytes of its first SESSION_KEY_TOKENS token ids (of its first n tokens)."""
    n = len(token_ids) if n is None else n
    return prefix_content(token_ids, min(n, SESSION_KEY_TOKENS)).tobytes()


def common_prefix(content, token_ids) -> int | None:
    """Tokens a kept context and a prompt share from the start (None without token ids)."""
    if content is None or token_ids is None:
        return None
    a = np.asarray(content)
    b = np.asarray(token_ids[:len(a)], dtype=np.int32)
    n = min(len(a), len(b))
    diff = np.flatnonzero(a[:n] != b[:n])
    return int(diff[0]) if diff.size else n


def resumable_tokens(tokens: int, content, req) -> int:
    """How much of a kept context of `tokens` tokens the request resumes from: all of it when the prompt starts with it
    and goes beyond it, else 0. Compared by token ids when both sides have them, else by the declared prefix."""
    if tokens <= 0 or tokens >= req.num_tokens:
        return 0
    if req.token_ids is not None and content is not None:
        return tokens if np.array_equal(prefix_content(req.token_ids, tokens), content) else 0
    return tokens if tokens <= req.prefix_tokens else 0


class PagePool:
    """Free pages of blocks 1..num_blocks; page p is page p % 67 of block p // 67."""

    def __init__(self, num_blocks: int):
        self.num_blocks = int(num_blocks)
        n = self.num_blocks + 1
        self._bits = [_FULL] * n                 # free pages of each block, bit i = page i
        self._bits[NULL_BLOCK] = 0
        self.num_free = self.num_blocks * PAGES_PER_BLOCK
        self._tick = 0
        self._whole_at: dict[int, int] = {}      # whole free block -> when it became whole
        self._whole_heap: list[tuple[int, int]] = []
        self._part_free: dict[int, int] = {}     # partly used block -> its free pages
        self._part_heap: list[tuple[int, int]] = []
        for b in range(1, n):
            self._mark_whole(b)

    # --- block states -------------------------------------------------------------------------------------------

    def _mark_whole(self, b: int):
        self._part_free.pop(b, None)
        self._whole_at[b] = self._tick
        heapq.heappush(self._whole_heap, (self._tick, b))
        self._tick += 1
        if len(self._whole_heap) > 4 * len(self._whole_at) + 256:
            self._whole_heap = [(t, x) for x, t in self._whole_at.items()]
            heapq.heapify(self._whole_heap)

    def _refresh(self, b: int):
        """Re-file block b after its free pages changed."""
        free = self._bits[b].bit_count()
        if free == PAGES_PER_BLOCK:
            if b not in self._whole_at:
                self._mark_whole(b)
            return
        self._whole_at.pop(b, None)
        if free == 0:
            self._part_free.pop(b, None)
        elif self._part_free.get(b) != free:
            self._part_free[b] = free
            heapq.heappush(self._part_heap, (free, b))
            if len(self._part_heap) > 4 * len(self._part_free) + 256:      # drop stale entries now and then
                self._part_heap = [(f, x) for x, f in self._part_free.items()]
                heapq.heapify(self._part_heap)

    def _oldest_whole(self) -> int:
        h = self._whole_heap
        while self._whole_at.get(h[0][1]) != h[0][0]:
            heapq.heappop(h)
        return h[0][1]

    def _fullest_partial(self) -> int | None:
        h = self._part_heap
        while h and self._part_free.get(h[0][1]) != h[0][0]:
            heapq.heappop(h)
        return h[0][1] if h else None

    @property
    def num_whole(self) -> int:
        return len(self._whole_at)

    def can_take(self, pages: int, states: int) -> bool:
        """Whether `pages` KV pages and `states` state blocks can be handed out now."""
        return self.num_whole >= states and self.num_free - states * PAGES_PER_BLOCK >= pages

    # --- hand-out -----------------------------------------------------------------------------------------------

    def _take_from(self, b: int, k: int) -> list[int]:
        bits, out, base = self._bits[b], [], b * PAGES_PER_BLOCK
        for _ in range(k):
            low = bits & -bits
            out.append(base + low.bit_length() - 1)
            bits ^= low
        self._bits[b] = bits
        self._refresh(b)
        return out

    def take_pages(self, n: int) -> list[int]:
        if n > self.num_free:
            raise RuntimeError(f"page pool: {n} pages asked, {self.num_free} free")
        out: list[int] = []
        need = n
        while need:
            b = self._fullest_partial()
            if b is None:
                break
            got = self._take_from(b, min(need, self._part_free[b]))
            out += got
            need -= len(got)
        while need:
            got = self._take_from(self._oldest_whole(), min(need, PAGES_PER_BLOCK))
            out += got
            need -= len(got)
        self.num_free -= n
        return out

    def take_states(self, n: int) -> list[int]:
        if n > self.num_whole:
            raise RuntimeError(f"page pool: {n} state blocks asked, {self.num_whole} whole blocks free")
        out = []
        for _ in range(n):
            b = self._oldest_whole()
            self._bits[b] = 0
            self._refresh(b)
            out.append(b)
        self.num_free -= n * PAGES_PER_BLOCK
        return out

    def give_pages(self, pages) -> None:
        if not len(pages):
            return
        per_block: dict[int, int] = {}
        for p in pages:
            b, i = divmod(int(p), PAGES_PER_BLOCK)
            if b == NULL_BLOCK or b > self.num_blocks or (self._bits[b] >> i) & 1 or (per_block.get(b, 0) >> i) & 1:
                raise RuntimeError(f"page pool: page {p} given back twice or out of range")
            per_block[b] = per_block.get(b, 0) | (1 << i)
        for b in sorted(per_block):                      # blocks re-filed in ascending order
            self._bits[b] |= per_block[b]
            self._refresh(b)
        self.num_free += len(pages)

    def give_states(self, blocks) -> None:
        for b in blocks:
            if b == NULL_BLOCK or self._bits[b] != 0:
                raise RuntimeError(f"page pool: state block {b} is not held")
            self._bits[b] = _FULL
            self._refresh(b)
        self.num_free += len(blocks) * PAGES_PER_BLOCK

    def give(self, alloc: "Allocation") -> None:
        self.give_pages(alloc.kv_pages)
        self.give_states(alloc.state_blocks)

    def is_free(self, page: int) -> bool:
        b, i = divmod(int(page), PAGES_PER_BLOCK)
        return bool((self._bits[b] >> i) & 1)


@dataclass
class Allocation:
    kv_pages: list[int]                 # KV pages from token 0
    state_blocks: list[int]             # whole blocks

    @property
    def num_pages(self) -> int:
        return len(self.kv_pages) + len(self.state_blocks) * PAGES_PER_BLOCK


@dataclass(eq=False)
class Kept:
    """A session's kept context: its last prompt's KV pages and the KDA state at the prompt's end."""
    session: object
    tokens: int
    alloc: Allocation
    content: np.ndarray | None          # its token ids (when the requests carry them)
    token: int | None = None            # the greedy token that prompt got


class KvManager:
    """Per-request reservations over the pool plus the kept sessions; pure state, driven by the scheduler.

    `keep_sessions`: a finished prompt stays as its session's kept context. `content_keys`: kept contexts are found
    by their first token ids (`find_session`) instead of a session id."""

    def __init__(self, num_blocks: int, keep_sessions: bool = False, content_keys: bool = False):
        self.pool = PagePool(num_blocks)
        self.keep_sessions = keep_sessions
        self.content_keys = content_keys
        self.capacity = self.pool.num_blocks * PAGES_PER_BLOCK
        self.hard = 0                                  # charge of running requests
        self.kept_charge = 0
        self.kept: OrderedDict[object, Kept] = OrderedDict()    # least recently used first
        self.held: dict[str, Allocation] = {}
        self._charge: dict[str, int] = {}
        self.evicted: dict[object, int] = {}           # key -> tokens of a kept context evicted and not replaced
        self._short = Counter()                        # content keys: lengths of kept contexts under the key size
        self.lower = None                              # a DRAM tier (`tier.DramTier`) taking evicted contexts
        self.stats = dict(admitted=0, hits=0, hit_tokens=0, evicted_sessions=0, evicted_tokens=0, dropped_stale=0,
                          peak_hard=0, states_short=0, repeats=0, tier_hits=0, tier_hit_tokens=0)

    @property
    def num_blocks(self) -> int:
        return self.pool.num_blocks

    @property
    def used_tokens(self) -> int:
        return (self.hard + self.kept_charge) * PAGE_TOKENS

    def footprint(self, prompt_tokens: int) -> int:
        return pages_for(prompt_tokens)

    kept_cost = footprint

    def fits_ever(self, prompt_tokens: int) -> bool:
        return self.footprint(prompt_tokens) <= self.capacity

    # --- lookups ------------------------------------------------------------------------------------------------

    def _hit(self, k: Kept, req) -> int:
        """The exact hit of `req` on kept context `k`, remembered on the request (asked at every forming while it
        waits; comparing a long prompt's ids costs ~0.1 ms)."""
        memo = getattr(req, "hit_memo", None)
        if memo is not None and memo[0] is k:
            return memo[1]
        hit = resumable_tokens(k.tokens, k.content, req)
        req.hit_memo = (k, hit)
        return hit

    def peek_hit(self, req) -> int:
        """The hit the request would get if admitted now (from HBM, else from the DRAM tier)."""
        if req.session is None or not self.keep_sessions:
            return 0
        k = self.kept.get(req.session)
        if k is None:
            return self.lower.peek(req.session, req) if self.lower is not None else 0
        return self._hit(k, req)

    def take_ops(self) -> list:
        """The DRAM tier's copies recorded since the last call, in order (they ride the next plan)."""
        return self.lower.take_ops() if self.lower is not None else []

    def shared_prefix(self, req) -> int:
        """Tokens the prompt shares with its session's previous context when the request declares no prefix: the
        hit, else the common start with a kept context it does not extend, else its evicted context's length."""
        if req.session is None or not self.keep_sessions:
            return 0
        k = self.kept.get(req.session)
        if k is not None:
            return self._hit(k, req) or min(common_prefix(k.content, req.token_ids) or 0, req.num_tokens - 1)
        lower = self.lower.tokens(req.session) if self.lower is not None else 0
        return min(lower or self.evicted.get(req.session, 0), req.num_tokens - 1)

    def find_session(self, token_ids) -> bytes:
        """Content keys: the key of the kept context this prompt may continue (its own key if none is kept)."""
        key = session_key(token_ids)
        if key in self.kept:
            return key
        for m in sorted(m for m, c in self._short.items() if c and m < len(token_ids)):
            short = session_key(token_ids, m)
            if short in self.kept:
                return short
        return key

    def kept_key(self, req):
        return session_key(req.token_ids) if self.content_keys else req.session

    def repeat_token(self, req) -> int | None:
        """A prompt identical to its kept context: the token that prompt already got (greedy), with the context
        refreshed; else None."""
        if req.session is None or not self.keep_sessions or req.token_ids is None:
            return None
        k = self.kept.get(req.session)
        if k is None or k.token is None or k.tokens != req.num_tokens \
                or not np.array_equal(prefix_content(req.token_ids, k.tokens), k.content):
            return None
        self.kept.move_to_end(req.session)
        self.stats["repeats"] += 1
        return k.token

    # --- admission ----------------------------------------------------------------------------------------------

    def _whole_blocks_for(self, states: int, give_back: int, skip) -> bool:
        """Whether `states` whole blocks can be had: free now (with the `give_back` the admission returns first), or
        freed by evicting a kept context other than `skip`."""
        if self.pool.num_whole + give_back >= states:
            return True
        self.stats["states_short"] += 1
        return any(x != skip for x in self.kept)

    def fits(self, req) -> bool:
        """Whether the request's whole footprint can be reserved now (kept contexts evicted as needed)."""
        need = self.hard + self.footprint(req.num_tokens)
        own = self.kept.get(req.session) if req.session is not None else None
        own_cost = 0 if own is None else self.kept_cost(own.tokens)
        if need + self.kept_charge - own_cost <= self.capacity:
            if own is None:
                states, back = STATE_BLOCKS, 0
            elif self._hit(own, req):
                states, back = 0, 0                    # takes over the kept states
            else:
                states, back = STATE_BLOCKS, STATE_BLOCKS   # the superseded context's states come back first
            return self._whole_blocks_for(states, back, req.session)
        return need <= self.capacity

    def _unkeep(self, k: Kept):
        self.kept_charge -= self.kept_cost(k.tokens)
        if self.content_keys and k.tokens < SESSION_KEY_TOKENS:
            self._short[k.tokens] -= 1

    def _make_room(self, pages: int, states: int):
        """Evict kept contexts, least recently used first, until the charge fits and the pool can hand out `pages`
        KV pages and `states` state blocks."""
        while self.kept and (self.hard + self.kept_charge > self.capacity or not self.pool.can_take(pages, states)):
            key, k = self.kept.popitem(last=False)
            self._unkeep(k)
            self.evicted[key] = k.tokens
            if self.lower is not None:
                self.lower.store(key, k)               # its write-back is recorded before any reuse of the pages
            self.pool.give(k.alloc)
            self.stats["evicted_sessions"] += 1
            self.stats["evicted_tokens"] += k.tokens
        if not self.pool.can_take(pages, states):
            raise RuntimeError(f"page pool cannot hand out {pages} pages and {states} states "
                               f"({self.pool.num_free} free, {self.pool.num_whole} whole blocks)")

    def allocate(self, req) -> int:
        """Reserve the request's whole footprint (the caller checked `fits`), taking over its session's kept context
        when it resumes from it. Returns the hit: tokens already in the reserved KV."""
        if not self.fits(req):
            raise RuntimeError(f"{req.req_id}: allocate without room")
        k = self.kept.pop(req.session, None) if req.session is not None else None
        hit = 0
        info = {"hit_kind": "none_first_round", "kept_tokens": 0, "common_prefix_tokens": None}
        evicted_before = self.stats["evicted_sessions"]
        if k is not None:
            self._unkeep(k)
            hit = self._hit(k, req)
            info["kept_tokens"] = k.tokens
            if hit:
                info["hit_kind"], info["common_prefix_tokens"] = "full", hit
            else:                                      # the prompt left its context: give it back
                self.pool.give(k.alloc)
                self.stats["dropped_stale"] += 1
                info["hit_kind"] = "superseded"
                info["common_prefix_tokens"] = common_prefix(k.content, req.token_ids)
        elif req.session is not None and req.session in self.evicted:
            info["hit_kind"] = "evicted"
            info["evicted_context_tokens"] = self.evicted[req.session]
        low = None                                     # the session's context in the DRAM tier, detached for a read
        if k is None and self.lower is not None and req.session is not None:
            low = self.lower.detach(req.session)
            if low is not None and not resumable_tokens(low.tokens, low.content, req):
                self.lower.release_detached(low)
                low = None
        charge = self.footprint(req.num_tokens)
        self.hard += charge
        self.stats["peak_hard"] = max(self.stats["peak_hard"], self.hard)
        n_kv = kv_pages_for(req.num_tokens)
        if hit:
            alloc = k.alloc
            more = n_kv - len(alloc.kv_pages)
            self._make_room(more, 0)
            alloc.kv_pages += self.pool.take_pages(more)
        else:
            self._make_room(n_kv, STATE_BLOCKS)
            pages = self.pool.take_pages(n_kv)         # KV pages before the state blocks
            alloc = Allocation(pages, self.pool.take_states(STATE_BLOCKS))
            if low is not None:                        # resumes from the DRAM tier: its read fills the first pages
                self.lower.read(low, alloc)
                hit = low.tokens
                info["hit_kind"], info["common_prefix_tokens"] = "tier", hit
                self.stats["tier_hits"] += 1
                self.stats["tier_hit_tokens"] += hit
        self.held[req.req_id] = alloc
        self._charge[req.req_id] = charge
        self.stats["admitted"] += 1
        if hit:
            self.stats["hits"] += 1
            self.stats["hit_tokens"] += hit
        info["evicted_sessions_at_admit"] = self.stats["evicted_sessions"] - evicted_before
        req.admit_info = info
        return hit

    def admit(self, req) -> Allocation | None:
        """Allocate if it fits now, else None; sets `req.cached` to the hit."""
        if not self.fits(req):
            return None
        req.cached = self.allocate(req)
        return self.held[req.req_id]

    def release(self, req):
        """The request is done. With `keep_sessions` its prompt's pages and final KDA state stay as its session's
        kept context (returns the key); else they are freed."""
        alloc = self.held.pop(req.req_id)
        self.hard -= self._charge.pop(req.req_id)
        if not (self.keep_sessions and req.session is not None):
            self.pool.give(alloc)
            return None
        key = self.kept_key(req)
        old = self.kept.pop(key, None)
        if old is not None:
            self._unkeep(old)
            self.pool.give(old.alloc)
        content = prefix_content(req.token_ids, req.num_tokens) if req.token_ids is not None else None
        self.kept[key] = Kept(key, req.num_tokens, alloc, content, getattr(req, "output_token", None))
        self.evicted.pop(key, None)
        self.kept_charge += self.kept_cost(req.num_tokens)
        if self.content_keys and req.num_tokens < SESSION_KEY_TOKENS:
            self._short[req.num_tokens] += 1
        if self.lower is not None:
            self.lower.drop(key)                       # an older copy of this session's context is stale now
        self._make_room(0, 0)
        return key

    def drop(self, req):
        """Give back a reservation without keeping anything (a cancelled request)."""
        alloc = self.held.pop(req.req_id)
        self.hard -= self._charge.pop(req.req_id)
        self.pool.give(alloc)
