"""GPU parity of the whole NVFP4 MoE layer (`ssb_moe_forward` through the C ABI) against the CPU oracle.

Bit-exact: routing indices (on the layer's own logits), expert counts, 128-aligned expert offsets, the permuted row of
every (token, slot), the GEMM tile table. Within tolerance (stated per assert): router logits, routing weights, layer
output (relative L2; BASELINE's per-layer bar is 3e-2)."""

import numpy as np
import pytest
import torch

from oracle import moe as omoe

pytestmark = pytest.mark.gpu

LAYER_TOL = 3e-2       # relative L2 of a layer's output (BASELINE: per-layer hidden states within 3e-2)


def run_layer(cuda, T, H, F, E, k, seed=0):
    from ssengine_b200 import moe, weights

    p = weights.moe_logical(seed, H, F, E)
    x = weights.hidden_states(seed + 1, T, H)
    layer = moe.MoELayer.from_logical(p, k, cuda)
    out = layer(x.to(cuda))
    torch.cuda.synchronize()
    layer.check_status()
    return layer, weights.to_numpy(p), x, out


@pytest.mark.parametrize("T,H,F,E,k", [
    (1000, 512, 256, 16, 4),      # T not a multiple of 128 / 256
    (512, 256, 128, 8, 2),        # BASELINE config 1's MoE dims (F % 256 != 0: K = 128 down GEMM)
    (16, 512, 256, 64, 2),        # most experts get no token
    (1, 256, 128, 8, 2),          # one token
])
def test_moe_layer_matches_oracle(cuda, T, H, F, E, k):
    layer, p, x, out = run_layer(cuda, T, H, F, E, k)
    xf = x.float().numpy()
    ref, parts = omoe.moe_forward(xf, p, k, return_parts=True)

    logits = layer.ws_view("LOGITS", T, torch.float32, (T, E)).cpu().numpy()
    np.testing.assert_allclose(logits, parts["logits"], rtol=1e-4, atol=1e-4 * np.abs(parts["logits"]).max())

    # routing on the layer's own logits: bit-exact indices
    ids = layer.ws_view("IDS", T, torch.int32, (T, k)).cpu().numpy()
    wts = layer.ws_view("WEIGHTS", T, torch.float32, (T, k)).cpu().numpy()
    rid, rw = omoe.route_softmax_topk(logits, k)
    np.testing.assert_array_equal(ids, rid)
    np.testing.assert_allclose(wts, rw, rtol=2e-6, atol=1e-7)

    # permutation: bit-exact
    counts, offsets, rows, _ = omoe.permutation(ids, E)
    np.testing.assert_array_equal(layer.ws_view("COUNTS", T, torch.int32, (E + 1,)).cpu().numpy(), counts)
    np.testing.assert_array_equal(layer.ws_view("OFFSETS", T, torch.int32, (E + 2,)).cpu().numpy(), offsets)
    np.testing.assert_array_equal(layer.ws_view("ROWS", T, torch.int32, (T, k)).cpu().numpy(), rows)
    n_tiles = int(layer.ws_view("NUM_MTILES", T, torch.int32, (1,)).item())
    assert n_tiles == offsets[-1] // 128
    tiles = layer.ws_view("MTILES", T, torch.int32, (n_tiles, 4)).cpu().numpy()
    want = [(e, offsets[e] + 128 * i, min(128, counts[e] - 128 * i), 0)
            for e in range(E + 1) for i in range(-(-int(counts[e]) // 128))]
    assert [tuple(r) for r in tiles.tolist()] == want
    # the CTA-pair table after the tile table (capacity rcap / 128 tiles): per expert ceil(tiles / 2) pairs
    # {expert, first row, rows of the first 128, rows of the next 128}
    cap = -(-(T * (k + 1) + (E + 1) * 127) // 128)
    n_pairs = int(layer.ws_view("NUM_MTILES", T, torch.int32, (2,)).cpu().numpy()[1])
    both = layer.ws_view("MTILES", T, torch.int32, (cap + n_pairs, 4)).cpu().numpy()
    want_pairs = [(e, offsets[e] + 256 * j, min(128, counts[e] - 256 * j), max(0, min(128, counts[e] - 256 * j - 128)))
                  for e in range(E + 1) for j in range(-(-int(counts[e]) // 256))]
    assert [tuple(r) for r in both[cap:].tolist()] == want_pairs

    # the layer output, on the layer's own routing and on the oracle's own
    o = out.float().cpu().numpy()
    ref_same = omoe.moe_forward(xf, p, k, ids=ids, weights=wts)
    rel_same = np.linalg.norm(o - ref_same) / np.linalg.norm(ref_same)
    rel = np.linalg.norm(o - ref) / np.linalg.norm(ref)
    assert rel_same < LAYER_TOL, rel_same
    assert rel < LAYER_TOL, rel


@pytest.mark.parametrize("T,H,F,E,k,n_group,topk_group", [
    (600, 512, 256, 288, 8, 1, 1),     # the reference model's routing with its 288 experts (H, F scaled down)
    (300, 256, 128, 64, 4, 8, 4),      # grouped selection
])
def test_moe_layer_sigmoid_routing(cuda, T, H, F, E, k, n_group, topk_group):
    """The whole layer with the reference model's routing (sigmoid scores + correction bias, scale 5/2): routing and
    permutation bit-exact against the oracle on the layer's own logits, the output within the per-layer bar."""
    from ssengine_b200 import moe, weights

    p = weights.moe_logical(9, H, F, E, routing="sigmoid", n_group=n_group, topk_group=topk_group)
    x = weights.hidden_states(10, T, H)
    layer = moe.MoELayer.from_logical(p, k, cuda)
    out = layer(x.to(cuda))
    torch.cuda.synchronize()
    layer.check_status()
    pn = weights.to_numpy(p)
    logits = layer.ws_view("LOGITS", T, torch.float32, (T, E)).cpu().numpy()
    ids = layer.ws_view("IDS", T, torch.int32, (T, k)).cpu().numpy()
    wts = layer.ws_view("WEIGHTS", T, torch.float32, (T, k)).cpu().numpy()
    r = pn["route"]
    rid, rw = omoe.route_sigmoid_bias(logits, k, r["bias"], n_group, topk_group, r["scale"])
    np.testing.assert_array_equal(ids, rid)
    np.testing.assert_allclose(wts, rw, rtol=1.2e-7, atol=0)
    counts, offsets, rows, _ = omoe.permutation(ids, E)
    np.testing.assert_array_equal(layer.ws_view("ROWS", T, torch.int32, (T, k)).cpu().numpy(), rows)
    np.testing.assert_array_equal(layer.ws_view("OFFSETS", T, torch.int32, (E + 2,)).cpu().numpy(), offsets)
    o = out.float().cpu().numpy()
    xf = x.float().numpy()
    ref_same = omoe.moe_forward(xf, pn, k, ids=ids, weights=wts)
    assert np.linalg.norm(o - ref_same) / np.linalg.norm(ref_same) < LAYER_TOL
    ref = omoe.moe_forward(xf, pn, k)
    assert np.linalg.norm(o - ref) / np.linalg.norm(ref) < LAYER_TOL


def test_moe_layer_is_deterministic(cuda):
    layer, p, x, out = run_layer(cuda, 777, 512, 256, 16, 4, seed=5)
    again = layer(x.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(out, again)


def test_moe_layer_zero_tokens(cuda):
    from ssengine_b200 import moe, weights

    p = weights.moe_logical(0, 256, 128, 8)
    layer = moe.MoELayer.from_logical(p, 2, cuda)
    out = layer(torch.empty(0, 256, dtype=torch.bfloat16, device=cuda))
    torch.cuda.synchronize()
    assert out.shape == (0, 256)
