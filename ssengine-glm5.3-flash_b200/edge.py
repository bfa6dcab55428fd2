"""Stage edge over NVLink: `P2pPipe`, the drop-in for the reference's `CePipe` (ssengine/runtime/transport.py:205-335).

Same interface and protocol: a ring of K slots of [max_rows, width] bf16 rows lives on the receiver; n counts
microbatches from 1 on both sides and slot = (n - 1) % K; ready[] lives on the receiver and free[] on the sender, so
each side waits on its own memory and writes the other's over NVLink; stage 0 holds the in-flight gate word `exits`,
written by the last stage. Handles are exchanged once at start-up over gloo, which also serves the barriers.

What differs (B200 design): the rows reach the peer slot by SM stores -- the stage's last kernel writes the peer slot
itself (`send_slot` / `send_commit`), or `send` runs an SM copy kernel -- instead of a copy-engine memcpy; the waits are
bounded kernels (`ssb_flag_wait`: after `wait_ns` the stream moves on and the status word holds 4, which `check`
raises), not unbounded stream memory operations. There is no fallback: without the CUDA library the pipe raises.

The device operations go through a small backend object so that the protocol (slots, flag values, ordering) can be
exercised on the CPU with a fake device (tests/test_edge_cpu.py).
"""

from __future__ import annotations

import ctypes
from datetime import timedelta

import torch
import torch.distributed as dist

from . import lib

FLAG_BYTES = 256


def ring_slots(max_in_flight: int, slot_bytes: int, ring_bytes: int) -> int:
    """K = max_in_flight + 1 slots, fewer when that exceeds ring_bytes; at least 1 (CePipe.__init__,
    transport.py:231)."""
    return max(1, min(max_in_flight + 1, ring_bytes // slot_bytes))


class CudaEdge:
    """Device operations of the pipe through the C ABI."""

    def __init__(self, device: torch.device):
        self.so = lib.load()
        self.device = device
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def alloc(self, nbytes: int) -> torch.Tensor:
        return torch.zeros(nbytes, dtype=torch.uint8, device=self.device)

    def export(self, t: torch.Tensor) -> tuple[bytes, int]:
        buf = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        lib.check("ssb_ipc_export", self.so.ssb_ipc_export(t.data_ptr(), buf, ctypes.byref(off)))
        return buf.raw, off.value

    def open(self, handle: tuple[bytes, int]) -> int:
        raw, off = handle
        p = ctypes.c_void_p()
        lib.check("ssb_ipc_open", self.so.ssb_ipc_open(ctypes.create_string_buffer(raw, 64), ctypes.byref(p)))
        return (p.value or 0) + off, p.value

    def close(self, base: int) -> None:
        lib.check("ssb_ipc_close", self.so.ssb_ipc_close(base))

    def wait(self, stream, addr: int, value: int, wait_ns: int) -> None:
        lib.check("ssb_flag_wait", self.so.ssb_flag_wait(addr, value & 0xFFFFFFFF, wait_ns, self.status.data_ptr(),
                                                         stream.cuda_stream))

    def write(self, stream, addr: int, value: int) -> None:
        lib.check("ssb_flag_write", self.so.ssb_flag_write(addr, value & 0xFFFFFFFF, stream.cuda_stream))

    def copy(self, stream, dst: int, src: torch.Tensor, nbytes: int) -> None:
        lib.check("ssb_p2p_copy", self.so.ssb_p2p_copy(dst, src.data_ptr(), nbytes, stream.cuda_stream))

    def current_stream(self):
        return torch.cuda.current_stream(self.device)

    def new_stream(self):
        return torch.cuda.Stream(self.device)

    def status_value(self) -> int:
        return int(self.status.item())

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)


class P2pPipe:
    """`CePipe` with SM stores into the peer slot and bounded waits (see the module docstring)."""

    RING_BYTES = 4 << 30

    def __init__(self, stage: int, num_stages: int, device: torch.device, init_method: str, max_in_flight: int,
                 max_rows: int, width: int, *, wait_ns: int = 10_000_000_000, backend=None,
                 init_group: bool = True, group_timeout_s: float = 120.0):
        self.stage, self.num_stages, self.device = stage, num_stages, device
        self.rows, self.width = max_rows, width
        self.slot_bytes = max_rows * width * 2
        self.K = ring_slots(max_in_flight, self.slot_bytes, self.RING_BYTES)
        self.depth = max_in_flight
        self.wait_ns = wait_ns
        self._own_group = init_group
        if init_group:
            dist.init_process_group("gloo", init_method=init_method, rank=stage, world_size=num_stages,
                                    timeout=timedelta(seconds=group_timeout_s))
        self.be = backend if backend is not None else CudaEdge(device)
        self.send_stream = self.be.new_stream()
        self._opened = []
        mine = {}
        self.ring = self.ready = self.free = self.exits = None
        if stage > 0:                                   # receiver: ring + ready[]
            self.ring_mem = self.be.alloc(self.K * self.slot_bytes)
            self.ring = self.ring_mem.view(torch.bfloat16).view(self.K, max_rows, width)
            self.ready = self.be.alloc(FLAG_BYTES)
            mine |= {"ring": self.be.export(self.ring_mem), "ready": self.be.export(self.ready)}
        if stage < num_stages - 1:                      # sender: free[]
            self.free = self.be.alloc(FLAG_BYTES)
            mine["free"] = self.be.export(self.free)
        if stage == 0 and num_stages > 1:               # the in-flight gate
            self.exits = self.be.alloc(FLAG_BYTES)
            mine["exits"] = self.be.export(self.exits)
        self.be.synchronize()
        allh = [None] * num_stages
        dist.all_gather_object(allh, mine)
        self.peer_ring = self.peer_ready = self.peer_free = self.peer_exits = None
        if stage < num_stages - 1:
            self.peer_ring = self._open(allh[stage + 1]["ring"])
            self.peer_ready = self._open(allh[stage + 1]["ready"])
        if stage > 0:
            self.peer_free = self._open(allh[stage - 1]["free"])
        if stage == num_stages - 1 and num_stages > 1:
            self.peer_exits = self._open(allh[0]["exits"])
        dist.barrier()
        self.n_recv = self.n_send = 0

    def _open(self, handle) -> int:
        ptr, base = self.be.open(handle)
        self._opened.append(base)
        return ptr

    # -- pipe (the reference's methods) --
    def recv(self, num_tokens: int, width: int) -> torch.Tensor:
        assert width == self.width and num_tokens <= self.rows, (num_tokens, width, self.rows, self.width)
        self.n_recv += 1
        slot = (self.n_recv - 1) % self.K
        self.be.wait(self.be.current_stream(), self.ready.data_ptr() + 4 * slot, self.n_recv, self.wait_ns)
        return self.ring[slot, :num_tokens]

    def release(self) -> None:
        """After the forward that read the last recv()'s rows is queued: the sender may reuse that slot."""
        slot = (self.n_recv - 1) % self.K
        self.be.write(self.be.current_stream(), self.peer_free + 4 * slot, self.n_recv)

    def gate(self, n: int) -> None:
        """Stage 0, before its n-th forward (from 1): wait until the last stage finished forward n - max_in_flight."""
        if self.exits is not None and n > self.depth:
            self.be.wait(self.be.current_stream(), self.exits.data_ptr(), n - self.depth, self.wait_ns)

    def exited(self, n: int) -> None:
        """Last stage, after its n-th forward is queued."""
        if self.peer_exits is not None:
            self.be.write(self.be.current_stream(), self.peer_exits, n)

    def send(self, hidden: torch.Tensor, after=None) -> None:
        """Rows of a finished forward into the next stage's slot by an SM copy on the send stream."""
        assert hidden.is_contiguous() and hidden.dtype == torch.bfloat16 and hidden.shape[1] == self.width
        assert hidden.shape[0] <= self.rows, (hidden.shape, self.rows)
        s = self.send_stream
        if after is not None:
            s.wait_event(after)
        dst = self._claim(s)
        self.be.copy(s, dst, hidden, hidden.numel() * 2)
        self.be.write(s, self.peer_ready + 4 * ((self.n_send - 1) % self.K), self.n_send)
        if isinstance(hidden, torch.Tensor) and hidden.is_cuda:
            hidden.record_stream(s)

    def send_slot(self, stream=None) -> int:
        """Fused send, part 1: on `stream` (default current) wait until the next slot is free and return its peer
        address; the stage's last kernel then writes its rows there ([rows, width] bf16, row pitch width)."""
        return self._claim(stream if stream is not None else self.be.current_stream())

    def send_commit(self, stream=None) -> None:
        """Fused send, part 2: after the kernel that wrote the slot, publish it (ready[slot] = n)."""
        s = stream if stream is not None else self.be.current_stream()
        self.be.write(s, self.peer_ready + 4 * ((self.n_send - 1) % self.K), self.n_send)

    def _claim(self, stream) -> int:
        self.n_send += 1
        slot = (self.n_send - 1) % self.K
        if self.n_send > self.K:
            self.be.wait(stream, self.free.data_ptr() + 4 * slot, self.n_send - self.K, self.wait_ns)
        return self.peer_ring + slot * self.slot_bytes

    def check(self) -> None:
        """Raise if a bounded wait of this pipe gave up (reads the device status word: synchronizes)."""
        v = self.be.status_value()
        if v != 0:
            raise lib.SsbError("stage edge wait", v)

    def close(self, mbs: int = 0) -> None:
        self.be.synchronize()
        dist.barrier()                                  # peers are done with our ring and flags
        for base in self._opened:
            self.be.close(base)
        self._opened.clear()
        dist.barrier()
        if self._own_group:
            dist.destroy_process_group()
