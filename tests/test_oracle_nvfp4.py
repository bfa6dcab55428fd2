"""The CPU oracle's NVFP4 codec against known answers of the format (e2m1 / e4m3 grids, round-to-nearest-even ties,
saturation) and its own round trips; the product's host layouts (ssengine_b200.layout) against the oracle's."""

import numpy as np
import torch

from oracle import nvfp4


def test_e2m1_grid_and_ties():
    vals = np.array([0, 0.25, 0.26, 0.5, 0.74, 0.75, 1.0, 1.25, 1.3, 1.5, 1.75, 2.0, 2.5, 2.6, 3.0, 3.5, 4.0, 5.0,
                     5.01, 6.0, 7.0, 1e9], dtype=np.float32)
    want = [0.0, 0.0, 0.5, 0.5, 0.5, 1.0, 1.0, 1.0, 1.5, 1.5, 2.0, 2.0, 2.0, 3.0, 3.0, 4.0, 4.0, 4.0, 6.0, 6.0, 6.0,
            6.0]
    np.testing.assert_array_equal(nvfp4.e2m1_decode(nvfp4.e2m1_encode(vals)), np.array(want, dtype=np.float32))
    np.testing.assert_array_equal(nvfp4.e2m1_decode(nvfp4.e2m1_encode(-vals)), -np.array(want, dtype=np.float32))
    # every grid value maps to its own code, negative zero included; a value that rounds to zero keeps its sign (the
    # hardware conversion's and vLLM's quantizer's convention)
    codes = np.arange(16, dtype=np.uint8)
    v = nvfp4.e2m1_decode(codes)
    v[8] = -0.0
    np.testing.assert_array_equal(nvfp4.e2m1_encode(v), codes)
    assert nvfp4.e2m1_encode(np.float32(-0.1)) == 8 and nvfp4.e2m1_encode(np.float32(0.1)) == 0


def test_e4m3_every_code_and_midpoints():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F and c != 0x80], dtype=np.uint8)
    v = nvfp4.e4m3_decode(codes)
    np.testing.assert_array_equal(nvfp4.e4m3_encode(v), codes)
    pos = np.sort(nvfp4.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8)))
    mids = ((pos[1:].astype(np.float64) + pos[:-1]) / 2).astype(np.float32)
    got = nvfp4.e4m3_decode(nvfp4.e4m3_encode(mids))
    lo, hi = pos[:-1], pos[1:]
    lo_even = (nvfp4.e4m3_encode(lo) & 1) == 0
    np.testing.assert_array_equal(got, np.where(lo_even, lo, hi))        # ties to the even code
    assert nvfp4.e4m3_decode(nvfp4.e4m3_encode(np.float32(1000.0))) == 448.0  # saturating
    assert nvfp4.e4m3_decode(nvfp4.e4m3_encode(np.float32(2.0 ** -10))) == 0.0
    assert nvfp4.e4m3_decode(nvfp4.e4m3_encode(np.float32(3 * 2.0 ** -10))) == 2.0 ** -8   # tie -> even (2 * 2^-9)


def test_quantize_block_rule():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 64)).astype(np.float32) * np.float32(3.0)
    x[1, :16] = 0.0                              # an all-zero block: scale 0, codes 0
    x[2, 16:32] = 1e6                            # saturating block
    gs = 448.0 * 6 / 8
    codes, sf = nvfp4.quantize(x, gs)
    assert codes.shape == (5, 64) and sf.shape == (5, 4)
    assert sf[1, 0] == 0 and not codes[1, :16].any()
    d = nvfp4.dequantize(codes, sf, gs)
    blk = np.abs(x).reshape(5, 4, 16).max(2)
    err = np.abs(d - x).reshape(5, 4, 16).max(2)
    ok = (blk < 8) & (blk > 0)      # blocks whose scale does not saturate (amax / 6 * gs < 448)
    # e2m1's widest step (4 -> 6) at scale amax / 6, plus the e4m3 rounding of the scale, bounds the error
    assert (err[ok] <= blk[ok] * 0.25 + 1e-6).all()
    # the rule step by step for one block
    b = x[0, :16]
    amax = np.float32(np.abs(b).max())
    s = nvfp4.e4m3_encode((amax / np.float32(6)) * np.float32(gs))
    r = np.float32(gs) / nvfp4.e4m3_decode(s)
    np.testing.assert_array_equal(codes[0, :16], nvfp4.e2m1_encode(b * r))
    assert sf[0, 0] == s


def test_pack_and_atoms_round_trip():
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 16, size=(300, 320), dtype=np.uint8)
    p = nvfp4.pack(codes)
    assert p.shape == (300, 160) and p[0, 0] == (codes[0, 0] | (codes[0, 1] << 4))
    np.testing.assert_array_equal(nvfp4.unpack(p), codes)
    sf = rng.integers(0, 256, size=(300, 20), dtype=np.uint8)
    flat = nvfp4.sf_to_atoms(sf)
    ncb = nvfp4.atom_cols(320)
    assert ncb == 8 and flat.size == 3 * ncb * 512
    np.testing.assert_array_equal(nvfp4.atoms_to_sf(flat, 300, 20), sf)
    r, c = 200, 13          # the documented byte position
    assert flat[((r // 128) * ncb + c // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + c % 4] == sf[r, c]
    # padding (rows >= 300 and scale columns >= 20) is zero
    full = nvfp4.atoms_to_sf(flat, 384, 32)
    assert not full[300:].any() and not full[:, 20:].any()


def test_product_layouts_match_the_oracle():
    from ssengine_b200 import layout

    rng = np.random.default_rng(2)
    codes = rng.integers(0, 16, size=(256, 512), dtype=np.uint8)
    np.testing.assert_array_equal(layout.pack_codes(torch.from_numpy(codes)).numpy(), nvfp4.pack(codes))
    np.testing.assert_array_equal(layout.unpack_codes(torch.from_numpy(nvfp4.pack(codes))).numpy(), codes)
    sf = rng.integers(0, 256, size=(200, 24), dtype=np.uint8)
    a = layout.sf_to_atoms(torch.from_numpy(sf), 384).numpy()
    np.testing.assert_array_equal(a, nvfp4.sf_to_atoms(sf))
    np.testing.assert_array_equal(layout.atoms_to_sf(torch.from_numpy(a), 200, 384).numpy(), sf)
    assert layout.sf_atom_cols(384) == nvfp4.atom_cols(384) == 8
    w = torch.arange(512 * 3).view(512, 3)
    il = layout.gate_up_interleave(w)
    assert il[0, 0] == 0 and il[128, 0] == w[256, 0] and il[256, 0] == w[128, 0] and il[384, 0] == w[384, 0]
    assert torch.equal(layout.gate_up_deinterleave(il), w)
