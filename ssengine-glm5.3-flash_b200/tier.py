"""A DRAM tier under HBM's kept contexts: where an evicted session context goes, and the copies that move it.

Roles (the reference's kvpool, ssengine/kvpool/, re-designed around stream order):
- `DramTier` (stage 0's host, beside the `KvManager`): the contexts HBM evicted, by session key, least recently used
  first, over a `PagePool` of DRAM blocks with the same page / state structure as HBM's. When HBM evicts a kept
  context it is stored here (the tier's own oldest contexts dropped for room, a write-back op recorded); when a round
  resumes from a context held here, HBM reserves a miss's footprint, a read op copies the context into its first pages
  and its state blocks, and the DRAM pages are freed (exclusive: a context lives in one tier at a time).
- `TierOp`s travel inside the next `Plan` (`Plan.tier_ops`). Every stage applies them on its stream, in the order they
  were recorded, just before that plan's forward (`TierArena.apply`). Every hazard is a page reuse, and a reuse is
  always recorded after the op that freed the page: a write-back reads evicted HBM pages before a later op or forward
  reuses them, and a read takes DRAM pages before a later write-back reuses them. In-order execution on each stage's
  stream therefore needs no completion tracking and no deferred frees.
- `TierArena` (each stage): the DRAM side of the stage's cache views, a `StageKv` in pinned host memory with the same
  rows per block; an op's copies are the runs its pages and state blocks span in each view (`StageKv.tier_ranges` on
  both sides), moved by one `ssb_copy_runs` launch per op (SM loads and stores; host memory through unified virtual
  addressing).
Not restated from the reference: the SSD tier, write-back ahead of eviction, and staged loading (reads started ahead
of admission on their own streams); here a context is copied when HBM evicts it and read when its round is admitted,
on the stage's compute stream.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

from .kvpages import PAGES_PER_BLOCK
from .pagepool import Allocation, Kept, PagePool, kv_pages_for, resumable_tokens

PIECE_BYTES = 256 * 1024            # runs are cut into pieces of at most this many bytes (one CTA each)


@dataclass
class TierOp:
    """Copy one context between HBM and DRAM: "write" HBM -> DRAM, "read" DRAM -> HBM. Page ids index each side's
    page space (page p = page p % 67 of block p // 67); state blocks pair up in order (group g = index g)."""
    kind: str
    hbm_pages: list[int]
    hbm_states: list[int]
    dram_pages: list[int]
    dram_states: list[int]
    tokens: int = 0


@dataclass
class DramTier:
    """DRAM-resident contexts over `num_blocks` DRAM blocks (see the module docstring)."""
    num_blocks: int
    pool: PagePool = field(init=False)

    def __post_init__(self):
        self.pool = PagePool(self.num_blocks)
        self.entries: OrderedDict[object, Kept] = OrderedDict()     # least recently used first
        self.ops: list[TierOp] = []
        self.stats = dict(stored=0, stored_tokens=0, dropped=0, dropped_tokens=0, read=0, read_tokens=0,
                          too_big=0, superseded=0)

    def __contains__(self, key) -> bool:
        return key in self.entries

    def peek(self, key, req) -> int:
        """The hit a request of session `key` would get from the context held here (0 if none)."""
        k = self.entries.get(key)
        return 0 if k is None else resumable_tokens(k.tokens, k.content, req)

    def tokens(self, key) -> int:
        k = self.entries.get(key)
        return 0 if k is None else k.tokens

    def _drop(self, key):
        k = self.entries.pop(key)
        self.pool.give(k.alloc)
        self.stats["dropped"] += 1
        self.stats["dropped_tokens"] += k.tokens

    def drop(self, key):
        """Forget the session's context (its round superseded it); nothing to copy."""
        if key in self.entries:
            k = self.entries.pop(key)
            self.pool.give(k.alloc)
            self.stats["superseded"] += 1

    def store(self, key, kept: Kept) -> TierOp | None:
        """HBM evicts `kept` (its pages still hold the context; the op recorded here copies them before anything
        reuses them). Returns the write op, or None when the context cannot fit the tier at all."""
        self.drop(key)
        pages, states = len(kept.alloc.kv_pages), len(kept.alloc.state_blocks)
        if pages + states * PAGES_PER_BLOCK > self.pool.num_blocks * PAGES_PER_BLOCK:
            self.stats["too_big"] += 1
            return None
        while not self.pool.can_take(pages, states):
            if not self.entries:                       # the rest is held by a context detached for a read
                self.stats["too_big"] += 1
                return None
            self._drop(next(iter(self.entries)))
        dram = Allocation(self.pool.take_pages(pages), self.pool.take_states(states))
        self.entries[key] = Kept(key, kept.tokens, dram, kept.content, kept.token)
        op = TierOp("write", list(kept.alloc.kv_pages), list(kept.alloc.state_blocks), list(dram.kv_pages),
                    list(dram.state_blocks), kept.tokens)
        self.ops.append(op)
        self.stats["stored"] += 1
        self.stats["stored_tokens"] += kept.tokens
        return op

    def detach(self, key) -> Kept | None:
        """Take the session's context out of the tier for a read, its DRAM pages still reserved (so that write-backs
        recorded before the read cannot reuse them); None if the tier holds none."""
        return self.entries.pop(key, None)

    def release_detached(self, k: Kept):
        """A detached context that the round does not resume (it superseded it): free its pages."""
        self.pool.give(k.alloc)
        self.stats["superseded"] += 1

    def read(self, k: Kept, hbm: Allocation) -> TierOp:
        """The detached context `k`'s round was admitted with `hbm` reserved: copy the context into its first pages
        and its state blocks, and free the DRAM copy."""
        n = len(k.alloc.kv_pages)
        op = TierOp("read", list(hbm.kv_pages[:n]), list(hbm.state_blocks), list(k.alloc.kv_pages),
                    list(k.alloc.state_blocks), k.tokens)
        self.ops.append(op)
        self.pool.give(k.alloc)
        self.stats["read"] += 1
        self.stats["read_tokens"] += k.tokens
        return op

    def take_ops(self) -> list[TierOp]:
        ops, self.ops = self.ops, []
        return ops


def op_runs(op: TierOp, hbm_ranges, dram_ranges, piece: int = PIECE_BYTES) -> np.ndarray:
    """int64 [n, 3] (src, dst, bytes) of one op on one stage: for every KV range the 128-token page slices of its
    pages, for every state range the rows of the state block its group names; adjacent slices contiguous on both
    sides merged; runs cut into pieces of at most `piece` bytes."""
    if [(r.name, r.kind) for r in hbm_ranges] != [(r.name, r.kind) for r in dram_ranges]:
        raise ValueError("HBM and DRAM views differ")
    write = op.kind == "write"
    if op.kind not in ("write", "read"):
        raise ValueError(f"tier op kind {op.kind!r}")
    if len(op.hbm_pages) != len(op.dram_pages) or len(op.hbm_states) != len(op.dram_states):
        raise ValueError("tier op: page or state counts differ between the two sides")
    hp = np.asarray(op.hbm_pages, np.int64)
    dp = np.asarray(op.dram_pages, np.int64)
    src, dst, size = [], [], []
    for hr, dr in zip(hbm_ranges, dram_ranges):       # every slice in view order, each view's pages in op order
        if hr.kind == "kv":
            pb = hr.nbytes // PAGES_PER_BLOCK
            h = hr.base + (hp // PAGES_PER_BLOCK) * hr.stride + (hp % PAGES_PER_BLOCK) * pb
            d = dr.base + (dp // PAGES_PER_BLOCK) * dr.stride + (dp % PAGES_PER_BLOCK) * pb
            n = np.full(len(hp), pb, np.int64)
        elif 0 <= hr.group < len(op.hbm_states):
            h = np.array([hr.base + op.hbm_states[hr.group] * hr.stride], np.int64)
            d = np.array([dr.base + op.dram_states[hr.group] * dr.stride], np.int64)
            n = np.array([hr.nbytes], np.int64)
        else:
            continue
        src.append(h if write else d)
        dst.append(d if write else h)
        size.append(n)
    if not size:
        return np.zeros((0, 3), np.int64)
    s, t, n = np.concatenate(src), np.concatenate(dst), np.concatenate(size)
    # merge slices that continue the previous one on both sides
    brk = np.ones(len(n), bool)
    brk[1:] = (s[1:] != s[:-1] + n[:-1]) | (t[1:] != t[:-1] + n[:-1])
    head = np.flatnonzero(brk)
    rs, rt = s[head], t[head]
    rn = np.add.reduceat(n, head)
    # cut runs into pieces of at most `piece` bytes
    cnt = -(-rn // piece)
    idx = np.repeat(np.arange(len(rn)), cnt)
    off = (np.arange(int(cnt.sum())) - np.repeat(np.cumsum(cnt) - cnt, cnt)) * piece
    arr = np.stack([rs[idx] + off, rt[idx] + off, np.minimum(piece, rn[idx] - off)], axis=1).astype(np.int64)
    if arr.size and ((arr & 15) != 0).any():
        raise ValueError("tier copy runs must be 16-byte aligned")
    return arr


class TierArena:
    """A stage's DRAM side: its cache views in pinned host memory for the DRAM tier's `num_blocks` blocks (ids
    1..num_blocks; row 0 is the null block, as in HBM) (see the module docstring). `copier(runs [n, 3] int64 numpy,
    stream)` moves one op's runs; by default `ssb_copy_runs` through the library."""

    def __init__(self, stage_kv, stage: int, num_blocks: int, copier=None, device=None):
        from .kvpages import StageKv

        self.stage = stage
        self.hbm = stage_kv
        self.dram = StageKv(stage_kv.layers, stage_kv.is_dsa, num_blocks + 1, stage_kv.kda_heads, "cpu",
                            pin=copier is None, pool_fp8=stage_kv.pool_fp8)
        self.hbm_ranges = stage_kv.tier_ranges(stage)
        self.dram_ranges = self.dram.tier_ranges(stage)
        self.device = stage_kv.device if device is None else device     # where the copy kernel's status word lives
        self.copier = copier if copier is not None else self._cuda_copier
        self.bytes_moved = 0

    def _cuda_copier(self, runs: np.ndarray, stream=None):
        import torch

        from . import lib

        if not hasattr(self, "_status"):
            if torch.device(self.device).type != "cuda":
                raise ValueError(f"the copy kernel needs the stage's views on a CUDA device, not {self.device}")
            self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        # the runs' upload, the kernel and the runs buffer's life all on the kernel's stream: the caching allocators
        # keep the pinned staging and the device buffer until that stream has passed them
        with torch.cuda.stream(s):
            dev = torch.from_numpy(runs).pin_memory().to(self.device, non_blocking=True)
            lib.check("ssb_copy_runs", lib.load().ssb_copy_runs(dev.data_ptr(), runs.shape[0],
                                                                self._status.data_ptr(), lib.stream_ptr(s)))

    def check(self):
        """Raise if a copy kernel rejected a run (reads the status word: synchronizes with the device)."""
        from . import lib

        if hasattr(self, "_status") and int(self._status.item()):
            raise lib.SsbError("ssb_copy_runs status", int(self._status.item()))

    def _check_ids(self, op: TierOp):
        """Every page and state block of the op inside its side's views (ids 1..num_blocks - 1): a bad id raises here
        instead of sending the copy kernel outside the views."""
        for name, pages, states, kv in (("HBM", op.hbm_pages, op.hbm_states, self.hbm),
                                        ("DRAM", op.dram_pages, op.dram_states, self.dram)):
            lo, hi = PAGES_PER_BLOCK, kv.num_blocks * PAGES_PER_BLOCK
            if any(not lo <= p < hi for p in pages) or any(not 1 <= b < kv.num_blocks for b in states):
                raise ValueError(f"tier op: a {name} page or state block outside the {kv.num_blocks} blocks")

    def apply(self, ops, stream=None):
        """Copy `ops` in order on `stream`, one launch each, before the plan's forward."""
        for op in ops:
            self._check_ids(op)
            runs = op_runs(op, self.hbm_ranges, self.dram_ranges)
            if runs.size:
                self.copier(runs, stream)
                self.bytes_moved += int(runs[:, 2].sum())


def context_bytes(tokens: int, stage_kv) -> int:
    """Bytes one context of `tokens` tokens moves on a stage: its pages' slices of every KV view plus its six state
    blocks' rows."""
    rs = stage_kv.tier_ranges(0)
    kv = sum(r.nbytes // PAGES_PER_BLOCK for r in rs if r.kind == "kv") * kv_pages_for(tokens)
    return kv + sum(r.nbytes for r in rs if r.kind == "state")
