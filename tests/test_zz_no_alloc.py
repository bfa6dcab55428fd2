"""The routing + permutation entry point that allocates nothing (`ssb_moe_route_permute_noalloc`), for callers that
cannot call cudaMalloc (a stage whose KV pool took the free HBM at start-up, code that must not stall the GPU with an
allocation mid-microbatch, a host holding only buffers another process mapped for it).

Checked through the C ABI against the existing entry point `ssb_moe_forward`, whose routing ids / weights, permuted
rows, expert counts and offsets sit in its workspace: two calls in a row (a larger problem, then a smaller one, so
stale contents of the shared static scratch would show); against the CPU oracle directly at the limits of the static
scratch (T = 16384, E = 512, k = 31, where an off-by-one in its fixed layout would show) and on an empty call (zero
counts and offsets); then the size limit. This file is collected last so that a run stopping at the first failure has
already run every other test."""

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


def _oracle_route(logits_np, E, k):
    from oracle import moe as omoe

    ids, w = omoe.route_softmax_topk(logits_np, k)
    counts, offsets, rows, _ = omoe.permutation(ids, E)
    return {"IDS": ids, "WEIGHTS": w, "ROWS": rows.astype(np.int32), "COUNTS": counts,
            "OFFSETS": offsets.astype(np.int32)}


def test_no_alloc_at_its_limits_against_the_oracle(cuda):
    T, E, k = 16384, 512, 31
    logits = np.random.default_rng(31).standard_normal((T, E)).astype(np.float32)
    want = _oracle_route(logits, E, k)
    for _ in range(2):                              # twice: the second call reads the first call's leftovers
        got = _no_alloc(cuda, torch.from_numpy(logits).to(cuda), T, E, k)
        np.testing.assert_array_equal(got["IDS"].cpu().numpy(), want["IDS"])
        np.testing.assert_allclose(got["WEIGHTS"].cpu().numpy(), want["WEIGHTS"], rtol=2e-6, atol=1e-7)
        np.testing.assert_array_equal(got["ROWS"].cpu().numpy(), want["ROWS"])
        np.testing.assert_array_equal(got["COUNTS"].cpu().numpy(), want["COUNTS"])
        np.testing.assert_array_equal(got["OFFSETS"].cpu().numpy(), want["OFFSETS"])


def test_no_alloc_with_no_tokens_writes_zero_counts_and_offsets(cuda):
    from ssengine_b200 import lib

    so = lib.load()
    E = 16
    counts = torch.full((E + 1,), -7, dtype=torch.int32, device=cuda)
    offsets = torch.full((E + 2,), -7, dtype=torch.int32, device=cuda)
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda)
    p = dummy.data_ptr()
    rc = so.ssb_moe_route_permute_noalloc(p, 0, E, 4, p, p, p, counts.data_ptr(), offsets.data_ptr(), None,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    lib.check("ssb_moe_route_permute_noalloc", rc)
    torch.cuda.synchronize()
    assert (counts.cpu().numpy() == 0).all() and (offsets.cpu().numpy() == 0).all()
