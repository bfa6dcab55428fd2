"""GPU checks of the stage-edge primitives (`ssb_flag_wait`, `ssb_flag_write`, `ssb_p2p_copy`, `ssb_ipc_export`) and,
on a box with 2 GPUs, of `P2pPipe` between two stage processes over NVLink (the reference's CePipe protocol,
ssengine/runtime/transport.py:205-335), including the fused path in which a compute kernel (`ssb_rmsnorm`) writes its
rows straight into the peer's ring slot. A wait that nobody satisfies is made to run out (a flag that nothing sets):
the kernel returns, the status word holds 4, the context stays usable."""

import ctypes
import multiprocessing as mp
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_flag_write_then_wait_and_copy(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    s = torch.cuda.current_stream().cuda_stream
    flags = torch.zeros(64, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    src = torch.randn(1000, 256, device=cuda).to(torch.bfloat16)
    dst = torch.zeros_like(src)
    lib.check("copy", so.ssb_p2p_copy(dst.data_ptr(), src.data_ptr(), src.numel() * 2, s))
    lib.check("write", so.ssb_flag_write(flags.data_ptr() + 8, 7, s))
    lib.check("wait", so.ssb_flag_wait(flags.data_ptr() + 8, 7, 1_000_000_000, status.data_ptr(), s))
    lib.check("wait", so.ssb_flag_wait(flags.data_ptr() + 8, 5, 1_000_000_000, status.data_ptr(), s))
    torch.cuda.synchronize()
    assert torch.equal(dst, src) and int(flags[2]) == 7 and int(status[0]) == 0
    assert so.ssb_p2p_copy(dst.data_ptr() + 8, src.data_ptr(), 64, s) == 1      # misaligned: rejected on the host


def test_wait_runs_out_and_the_context_stays_usable(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    s = torch.cuda.current_stream().cuda_stream
    flags = torch.zeros(64, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib.check("wait", so.ssb_flag_wait(flags.data_ptr(), 1, 2_000_000, status.data_ptr(), s))     # 2 ms, nobody sets
    torch.cuda.synchronize()
    assert int(status[0]) == 4
    x = torch.arange(10, device=cuda).float()
    assert float((x * 2).sum()) == 90.0


def test_ipc_export_of_a_caching_allocator_tensor(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    big = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    view = big[4096:]
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(-1)
    lib.check("export", so.ssb_ipc_export(view.data_ptr(), buf, ctypes.byref(off)))
    assert off.value >= 4096 and any(buf.raw)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


ROWS, WIDTH, MBS = 512, 4 * 1024, 5


def rows_of(n, count, device):
    g = torch.Generator(device="cpu").manual_seed(50 + n)
    return torch.randn(count, WIDTH, generator=g).to(torch.bfloat16).to(device)


def stage_main(stage, port, q):
    import sys
    sys.path.insert(0, os.environ["SSB_ROOT"])
    import __graft_entry__
    __graft_entry__.import_package()
    from ssengine_b200 import lib
    from ssengine_b200.edge import P2pPipe

    try:
        dev = torch.device("cuda", stage)
        torch.cuda.set_device(dev)
        so = lib.load()
        pipe = P2pPipe(stage, 2, dev, f"tcp://127.0.0.1:{port}", 1, ROWS, WIDTH, wait_ns=5_000_000_000)
        w = torch.ones(WIDTH, device=dev).to(torch.bfloat16)
        if stage == 0:
            for n in range(1, MBS + 1):
                pipe.gate(n)
                x = rows_of(n, ROWS - n, dev)
                if n % 2:
                    pipe.send(x, torch.cuda.current_stream(dev).record_event())
                else:                                  # fused: the norm kernel writes the peer slot
                    dst = pipe.send_slot()
                    lib.check("rmsnorm", so.ssb_rmsnorm(x.data_ptr(), WIDTH, None, ROWS - n, w.data_ptr(), 1e-6, dst,
                                                        torch.cuda.current_stream(dev).cuda_stream))
                    pipe.send_commit()
            torch.cuda.synchronize(dev)
            pipe.check()
        else:
            for n in range(1, MBS + 1):
                got = pipe.recv(ROWS - n, WIDTH).float()
                x = rows_of(n, ROWS - n, dev).float()
                want = x if n % 2 else (x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).float()
                torch.cuda.synchronize(dev)
                err = float((got - want).abs().max())
                assert err <= (0 if n % 2 else 0.02), (n, err)
                pipe.release()
                pipe.exited(n)
            torch.cuda.synchronize(dev)
            pipe.check()
        pipe.close()
        q.put((stage, "ok"))
    except Exception as ex:
        q.put((stage, repr(ex)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_stage_pipe_over_nvlink():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    os.environ["SSB_ROOT"] = root
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=stage_main, args=(s, port, q)) for s in (0, 1)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}, res
