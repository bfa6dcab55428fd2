"""The routing + permutation entry point that allocates nothing (`ssb_moe_route_permute_noalloc`), for callers that
cannot call cudaMalloc (a stage whose KV pool took the free HBM at start-up, code that must not stall the GPU with an
allocation mid-microbatch, a host holding only buffers another process mapped for it).

Checked through the C ABI against the existing entry point `ssb_moe_forward`, whose routing ids / weights, permuted
rows, expert counts and offsets sit in its workspace: two calls in a row (a larger problem, then a smaller one, so
stale contents of the shared static scratch would show), then the size limit. This file is collected last so that a
run stopping at the first failure has already run every other test."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _forward_reference(cuda, T, H, F, E, k, seed):
    """ssb_moe_forward (the existing entry point) and its routing / permutation buffers."""
    from ssengine_b200 import moe, weights

    layer = moe.MoELayer.from_logical(weights.moe_logical(seed, H, F, E), k, cuda)
    layer(weights.hidden_states(seed + 1, T, H).to(cuda))
    torch.cuda.synchronize()
    layer.check_status()
    v = {n: layer.ws_view(n, T, dt, shp).clone() for n, dt, shp in [
        ("LOGITS", torch.float32, (T, E)), ("IDS", torch.int32, (T, k)), ("WEIGHTS", torch.float32, (T, k)),
        ("ROWS", torch.int32, (T, k)), ("COUNTS", torch.int32, (E + 1,)), ("OFFSETS", torch.int32, (E + 2,))]}
    return v


def _no_alloc(cuda, logits, T, E, k):
    from ssengine_b200 import lib

    so = lib.load()
    out = {"IDS": torch.full((T, k), -7, dtype=torch.int32, device=cuda),
           "WEIGHTS": torch.full((T, k), float("nan"), dtype=torch.float32, device=cuda),
           "ROWS": torch.full((T, k), -7, dtype=torch.int32, device=cuda),
           "COUNTS": torch.full((E + 1,), -7, dtype=torch.int32, device=cuda),
           "OFFSETS": torch.full((E + 2,), -7, dtype=torch.int32, device=cuda)}
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = so.ssb_moe_route_permute_noalloc(
        logits.data_ptr(), T, E, k, out["IDS"].data_ptr(), out["WEIGHTS"].data_ptr(), out["ROWS"].data_ptr(),
        out["COUNTS"].data_ptr(), out["OFFSETS"].data_ptr(), status.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    lib.check("ssb_moe_route_permute_noalloc", rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


def _same(got, ref):
    for name in ("IDS", "ROWS", "COUNTS", "OFFSETS"):
        np.testing.assert_array_equal(got[name].cpu().numpy(), ref[name].cpu().numpy(), err_msg=name)
    np.testing.assert_allclose(got["WEIGHTS"].cpu().numpy(), ref["WEIGHTS"].cpu().numpy(), rtol=2e-6, atol=1e-7)


def test_no_alloc_matches_the_existing_entry_point_on_two_calls_in_a_row(cuda):
    big = _forward_reference(cuda, 1000, 512, 256, 16, 4, seed=21)
    small = _forward_reference(cuda, 300, 256, 128, 8, 2, seed=22)
    _same(_no_alloc(cuda, big["LOGITS"], 1000, 16, 4), big)
    _same(_no_alloc(cuda, small["LOGITS"], 300, 8, 2), small)


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    t = torch.zeros(64, dtype=torch.int32, device=cuda)
    p = t.data_ptr()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert so.ssb_moe_route_permute_noalloc(p, 16385, 8, 2, p, p, p, p, p, p, s) == 7
    assert so.ssb_moe_route_permute_noalloc(p, 16, 513, 2, p, p, p, p, p, p, s) == 7
    assert so.ssb_moe_route_permute_noalloc(p, 16, 64, 32, p, p, p, p, p, p, s) == 7
