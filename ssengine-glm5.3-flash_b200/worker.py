"""The stage worker loop: one microbatch through one pipeline stage, in the order of the reference's `run_worker`
(ssengine/runtime/worker.py:341-365: prepare -> recv (stages > 0) / gate (stage 0) -> run -> release -> send).

B200 form of the hop (the reference copies the finished [T, 4H] rows into the next stage's ring with the copy engine,
ssengine/runtime/transport.py:323-335): the stage's last kernel -- the final mHC post boundary -- stores its rows
straight into the peer's receive slot (`P2pPipe.send_slot`, an IPC-mapped address on the next GPU) and the ready
flag follows it (`send_commit`). Every wait is a bounded device kernel; nothing on this path synchronizes the host.
"""

from __future__ import annotations

import torch

from .stage import Batch, StageModel


class StageWorker:
    """Runs microbatches through `stage`; `pipe` is the stage's `edge.P2pPipe` (None for a one-stage pipeline).
    With `events`, each forward is bracketed by CUDA events (busy time) appended to `self.spans`."""

    def __init__(self, stage: StageModel, pipe=None, events: bool = False, tier=None):
        self.stage, self.pipe = stage, pipe
        self.tier = tier                # a `tier.TierArena`: a plan's DRAM tier copies run before its forward
        self.n = 0
        self.events = events
        self.spans: list[tuple] = []
        self.last_tokens = None

    def step(self, work) -> torch.Tensor | None:
        """One microbatch (a Plan, or a Batch prepared earlier). Returns the last stage's greedy tokens, else None."""
        st, pipe = self.stage, self.pipe
        batch = work if isinstance(work, Batch) else st.prepare(work)
        if batch.tier_ops:                             # carried from the plan by prepare, also for a batch made early
            if self.tier is None:
                raise RuntimeError("a microbatch carries DRAM tier copies but this stage has no tier")
            self.tier.apply(batch.tier_ops)            # on the current stream, in order, before the forward
        self.n += 1
        hidden = None
        if pipe is not None:
            if st.first:
                pipe.gate(self.n)
            else:
                hidden = pipe.recv(batch.num_tokens, st.hidden_width)
        if self.events:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        if pipe is not None and not st.last:
            st.run(batch, hidden, edge_out=pipe.send_slot)
            out = None
        else:
            out = st.run(batch, hidden)
        if self.events:
            e1.record()
            self.spans.append((e0, e1))
        if pipe is not None:
            if not st.first:
                pipe.release()
            if st.last:
                pipe.exited(self.n)
            else:
                pipe.send_commit()
        if st.last:
            self.last_tokens = out
        return out

    def busy_ms(self) -> float:
        """Device time inside the forwards recorded so far (synchronizes on the last event)."""
        if not self.spans:
            return 0.0
        self.spans[-1][1].synchronize()
        return sum(a.elapsed_time(b) for a, b in self.spans)
