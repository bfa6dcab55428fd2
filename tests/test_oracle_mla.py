"""The oracle's e4m3 codec (oracle/mla.py) pinned to torch's float8_e4m3fn cast, an independent implementation of the
same OCP format (round to nearest even) for every in-range value class: normals, subnormals, ties, the largest
finite value; and the device conversion's saturation (beyond +-448 -> +-448) as known answers."""

import numpy as np
import torch

from oracle import mla as omla


def test_e4m3_matches_torch_in_range():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000) * 4,
        rng.standard_normal(5000) * 1e-3,                            # subnormal range (< 2^-6)
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -6, 1.0625, 1.1875,
                  17.0, 19.0, 240.0, 432.0, 440.0]),                 # ties to even and the top of the range
        omla.e4m3_decode(np.arange(256, dtype=np.uint8)[np.arange(256) % 128 != 127]),   # every finite code
    ]).astype(np.float32)
    got = omla.e4m3_encode(x)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(omla.e4m3_decode(got), torch.from_numpy(got).view(torch.float8_e4m3fn).float().numpy())


def test_e4m3_saturates():
    np.testing.assert_array_equal(omla.e4m3_encode(np.array([449.0, 464.0, 1e6, -500.0, np.inf])),
                                  np.array([0x7E, 0x7E, 0x7E, 0xFE, 0x7E], np.uint8))
    assert omla.e4m3_decode(np.array([0x7E], np.uint8))[0] == 448.0


def test_quantize_scale_in_fp32():
    x = np.array([1.0, 3.0, 100.0], np.float32)
    np.testing.assert_array_equal(omla.quantize(x, 3.0), omla.e4m3_encode(x * (np.float32(1) / np.float32(3.0))))


def test_fast_e4m3_encoder_equals_the_float64_restatement():
    rng = np.random.default_rng(12)
    x = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * s for s in (1e-4, 1e-2, 1.0, 40.0, 600.0)])
    codes = np.arange(256, dtype=np.uint8)
    vals = omla.e4m3_decode(codes[(codes & 0x7F) != 0x7F]).astype(np.float32)
    x = np.concatenate([x, vals, np.nextafter(vals, np.float32(np.inf)), np.nextafter(vals, np.float32(-np.inf)),
                        np.array([0.0, -0.0, 464.0, 480.0, -1e9], np.float32)])
    np.testing.assert_array_equal(omla.e4m3_encode(x), omla.e4m3_encode_reference(x))
