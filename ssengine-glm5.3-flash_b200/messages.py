"""The reference's control messages for a stage (ssengine/runtime/transport.py:20-36): the fields a `StageModel` reads,
same names, order and meaning. Plain dataclasses here (the reference uses msgspec structs for the wire; a drop-in
stage receives whatever object carries these attributes)."""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Chunk:
    req_id: str
    start: int                      # tokens of this request already in KV (cached + computed by earlier chunks)
    num_tokens: int                 # tokens computed in this chunk
    kv_pages: list[int]             # KV pages (128 tokens each) covering [0, start + num_tokens)
    state_blocks: list[int]         # 6 KDA state blocks
    is_last: bool                   # last chunk of the prompt: the last stage returns this request's token
    token_ids: list[int] | None     # the chunk's prompt tokens; stage 0 only


@dataclass
class Plan:
    mb_id: int                      # 0, 1, 2, ... in dispatch order
    chunks: list[Chunk] = field(default_factory=list)   # hidden rows concatenated in this order
    tier_ops: list = field(default_factory=list)        # DRAM tier copies every stage applies, in order, before the
                                                        # forward (`tier.TierOp`; not in the reference's message)

    @property
    def num_tokens(self) -> int:
        return sum(c.num_tokens for c in self.chunks)
