"""Microbatches of a synthetic cold-prompt stream, formed the way the reference's scheduler hands them to the stages.

The reference's control plane (ssengine/engine/scheduler.py `next_microbatch`, ssengine/engine/kv.py `PagePool`) cuts
prompts into chunks of at most `mb_tokens` rows per microbatch and gives every request its KV pages and six state
blocks from one block-id space (block 0 is the null block). This module is the minimal host-side former the
benchmark and the tests use for BASELINE config 4's workload (cold prompts served first come first served):

- a request takes ceil(len / 8,576) whole blocks for its KV pages (all 67 pages of each, in order) and six state
  blocks when its first chunk is scheduled, and returns them to the free list after the microbatch holding its last
  chunk (every stage runs microbatches in order on one stream, so a block reused by a later microbatch is never in
  use);
- a microbatch fills up to `mb_tokens` rows with the current request's next chunk, then the following requests';
- the blocks never exceed the pool: the high-water mark sizes the stages' pools (`blocks_needed`).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .kvpages import BLOCK_TOKENS, PAGES_PER_BLOCK
from .messages import Chunk, Plan


def prompt_lengths(n: int, seed: int, median: int = 8192, sigma: float = 1.0, max_len: int = 131072) -> np.ndarray:
    """BASELINE config 4's prompt lengths: lognormal with the given median, capped at max_len, at least 1."""
    rng = np.random.default_rng(seed)
    return np.clip(rng.lognormal(np.log(median), sigma, n), 1, max_len).astype(np.int64)


@dataclass
class _Req:
    rid: int
    length: int
    done: int = 0
    pages: list | None = None
    kv_blocks: list | None = None
    state: list | None = None


class BlockPool:
    """Free list of block ids 1.. (0 is the null block); tracks the high-water mark."""

    def __init__(self):
        self.free: list[int] = []
        self.next = 1
        self.high = 0

    def take(self, n: int) -> list[int]:
        out = []
        for _ in range(n):
            if self.free:
                out.append(self.free.pop())
            else:
                out.append(self.next)
                self.next += 1
        self.high = max(self.high, self.next - 1)
        return out

    def give(self, blocks: list[int]) -> None:
        self.free.extend(sorted(blocks, reverse=True))


def microbatches(lengths, mb_tokens: int, count: int, vocab: int | None = None, seed: int = 0):
    """The first `count` microbatches of the prompt stream `lengths` (FCFS, chunked). Returns (plans, pool high-water
    mark). With `vocab`, chunks carry uniform token ids (stage 0's input)."""
    rng = np.random.default_rng(seed)
    pool = BlockPool()
    reqs = [_Req(i, int(n)) for i, n in enumerate(lengths)]
    at = 0
    plans = []
    for mb in range(count):
        chunks, room, freed = [], mb_tokens, []
        while room > 0 and at < len(reqs):
            r = reqs[at]
            if r.pages is None:
                r.kv_blocks = pool.take(-(-r.length // BLOCK_TOKENS))
                r.pages = [b * PAGES_PER_BLOCK + p for b in r.kv_blocks for p in range(PAGES_PER_BLOCK)]
                r.state = pool.take(6)
            n = min(room, r.length - r.done)
            last = r.done + n == r.length
            ids = rng.integers(0, vocab, n).tolist() if vocab is not None else None
            need = -(-(r.done + n) // 128)
            chunks.append(Chunk(f"r{r.rid}", r.done, n, r.pages[:need], list(r.state), last, ids))
            r.done += n
            room -= n
            if last:
                freed += r.kv_blocks + r.state          # reusable from the next microbatch on
                at += 1
        if not chunks:
            break
        pool.give(freed)
        plans.append(Plan(mb, chunks))
    return plans, pool.high


def blocks_needed(plans) -> int:
    """Pool size (incl. the null block) that holds every block the plans name."""
    hi = 0
    for p in plans:
        for c in p.chunks:
            hi = max(hi, max(c.state_blocks), max((q // PAGES_PER_BLOCK for q in c.kv_pages), default=0))
    return hi + 1
