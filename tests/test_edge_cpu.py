"""The stage-edge protocol of `P2pPipe` (ssengine-glm5.3-flash_b200/edge.py) on the CPU: two gloo ranks, each stage a
process, with a fake device whose memory is shared host memory, so that the ring, the ready / free flags and the
in-flight gate run exactly as on GPUs (the reference's CePipe protocol, ssengine/runtime/transport.py:205-335): rows
arrive in order through a ring smaller than the microbatch count, the sender never overwrites a slot the receiver has
not released, stage 0 never runs more than max_in_flight ahead, and a wait that nobody satisfies ends with status 4."""

import ctypes
import multiprocessing as mp
import os
import socket
import time
from multiprocessing import shared_memory

import numpy as np
import pytest
import torch


class FakeStream:
    def wait_event(self, ev):
        pass


class FakeEdge:
    """Device operations on shared host memory: an allocation is a SharedMemory block, its handle the block name."""

    def __init__(self):
        self.blocks = []
        self.status = 0
        self.log = []

    def alloc(self, nbytes):
        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        shm.buf[:nbytes] = b"\0" * nbytes
        self.blocks.append(shm)
        return torch.frombuffer(shm.buf, dtype=torch.uint8)

    def export(self, t):
        for shm in self.blocks:
            base = ctypes.addressof(ctypes.c_char.from_buffer(shm.buf))
            if base <= t.data_ptr() < base + shm.size:
                return shm.name, t.data_ptr() - base
        raise KeyError

    def open(self, handle):
        name, off = handle
        shm = shared_memory.SharedMemory(name=name)
        self.blocks.append(shm)
        base = ctypes.addressof(ctypes.c_char.from_buffer(shm.buf))
        return base + off, base

    def close(self, base):
        pass

    def wait(self, stream, addr, value, wait_ns):
        t0 = time.monotonic_ns()
        while np.int32(np.uint32(ctypes.c_uint32.from_address(addr).value) - np.uint32(value)) < 0:
            if time.monotonic_ns() - t0 > wait_ns:
                self.status = 4
                return
            time.sleep(0.0005)
        self.log.append(("wait", value))

    def write(self, stream, addr, value):
        ctypes.c_uint32.from_address(addr).value = value
        self.log.append(("write", value))

    def copy(self, stream, dst, src, nbytes):
        ctypes.memmove(dst, src.data_ptr(), nbytes)

    def current_stream(self):
        return FakeStream()

    def new_stream(self):
        return FakeStream()

    def status_value(self):
        return self.status

    def synchronize(self):
        pass


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


ROWS, WIDTH, MBS, DEPTH = 8, 32, 6, 1


def rows_of(n, count):
    g = torch.Generator().manual_seed(1000 + n)
    return torch.randn(count, WIDTH, generator=g).to(torch.bfloat16)


def stage_main(stage, port, q):
    import sys
    sys.path.insert(0, os.environ["SSB_ROOT"])
    import __graft_entry__
    __graft_entry__.import_package()
    from ssengine_b200.edge import P2pPipe

    try:
        be = FakeEdge()
        pipe = P2pPipe(stage, 2, torch.device("cpu"), f"tcp://127.0.0.1:{port}", DEPTH, ROWS, WIDTH,
                       wait_ns=20_000_000_000, backend=be)
        assert pipe.K == DEPTH + 1
        if stage == 0:
            for n in range(1, MBS + 1):
                pipe.gate(n)
                pipe.send(rows_of(n, ROWS - n % 3))
            pipe.check()
        else:
            for n in range(1, MBS + 1):
                got = pipe.recv(ROWS - n % 3, WIDTH).clone()
                assert torch.equal(got, rows_of(n, ROWS - n % 3)), n
                time.sleep(0.01)                    # a slow consumer: the sender must wait for free slots
                pipe.release()
                pipe.exited(n)
            pipe.check()
        waits = [v for k, v in be.log if k == "wait"]
        pipe.close()
        q.put((stage, "ok", waits))
    except Exception as ex:                          # report to the parent
        q.put((stage, repr(ex), []))


def test_two_stage_protocol_over_gloo():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    os.environ["SSB_ROOT"] = root
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=stage_main, args=(s, port, q)) for s in (0, 1)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        stage, msg, waits = q.get(timeout=120)
        res[stage] = (msg, waits)
    for p in ps:
        p.join(timeout=60)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    # stage 0: free waits for n > K (value n - K) and gate waits for n > depth (value n - depth)
    assert res[1][1] == list(range(1, MBS + 1))          # stage 1 waited ready >= n, in order


def test_wait_that_nobody_satisfies_reports_status():
    be = FakeEdge()
    t = be.alloc(256)
    be.wait(None, t.data_ptr(), 1, 2_000_000)             # 2 ms, flag stays 0
    assert be.status_value() == 4


def test_ring_slots_follow_the_reference_sizing():
    import __graft_entry__
    __graft_entry__.import_package()
    from ssengine_b200.edge import ring_slots

    slot = 8192 * 16384 * 2
    assert ring_slots(4, slot, 4 << 30) == 5
    assert ring_slots(40, slot, 4 << 30) == 16
    assert ring_slots(4, 8 << 30, 4 << 30) == 1
