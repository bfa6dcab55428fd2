"""The DRAM tier's copy kernel (`ssb_copy_runs`, csrc/tier.cu) through `TierArena` on the GPU: a context written
from a stage's HBM views into their pinned host mirror and read back into other pages and state blocks, on a side
stream, against the same ops applied by plain host memmove to a host copy of the same views (every byte equal)."""

import ctypes

import pytest
import torch

from ssengine_b200.kvpages import StageKv
from ssengine_b200.tier import TierArena, TierOp

pytestmark = pytest.mark.gpu


def memmove_copier(runs, stream=None):
    for s, d, n in runs.tolist():
        ctypes.memmove(d, s, n)


def _views(kv):
    return kv.pages + kv.pool + kv.tail


@pytest.mark.parametrize("pool_fp8", [False, True])
def test_copy_kernel_moves_a_context_like_memmove(cuda, pool_fp8):
    layers, is_dsa = list(range(12)), (lambda i: i % 4 == 3)
    gpu = StageKv(layers, is_dsa, 10, 4, cuda, pool_fp8=pool_fp8)
    host = StageKv(layers, is_dsa, 10, 4, "cpu", pool_fp8=pool_fp8)
    g = torch.Generator().manual_seed(7)
    for d, h in zip(_views(gpu), _views(host)):
        b = torch.randint(0, 256, h.view(torch.uint8).shape, dtype=torch.uint8, generator=g)
        h.view(torch.uint8).copy_(b)
        d.view(torch.uint8).copy_(b.to(cuda))
    arena = TierArena(gpu, 0, 9, device=cuda)                   # the default copier: ssb_copy_runs
    ref = TierArena(host, 0, 9, copier=memmove_copier)
    write = TierOp("write", [70, 71, 140, 141, 142], [3, 4, 5, 6, 7, 8], [70, 71, 72, 73, 74], [2, 3, 4, 5, 6, 7])
    read = TierOp("read", [150, 151, 152, 153, 154], [9, 8, 7, 6, 5, 3], [70, 71, 72, 73, 74], [2, 3, 4, 5, 6, 7])
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    arena.apply([write, read], stream=s)                         # the read lands on pages the write did not touch
    ref.apply([write, read])
    torch.cuda.synchronize(cuda)
    arena.check()
    for d, h in zip(_views(gpu), _views(host)):
        assert torch.equal(d.view(torch.uint8).cpu(), h.view(torch.uint8))
    for d, h in zip(_views(arena.dram), _views(ref.dram)):      # the pinned mirror holds what memmove wrote
        assert torch.equal(d.view(torch.uint8), h.view(torch.uint8))
    assert arena.bytes_moved == ref.bytes_moved > 0
