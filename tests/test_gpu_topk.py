"""GPU parity of the canonical indexer top-k (`ssb_topk_canonical`): bit-exact against fixtures produced by the
reference's own `canonical_topk_torch` (ssengine/model/topk_canon.py:33-52), its known-answer test, and the oracle on
larger rows with heavy ties, empty and short rows, rows longer than the shared-memory cache, and k = 2048."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import topk as otopk
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


def gpu_topk(cuda, logits, ks, ke, k, max_keys=None):
    from ssengine_b200 import lib

    so = lib.load()
    lg = torch.from_numpy(np.ascontiguousarray(logits, dtype=np.float32)).to(cuda)
    a = torch.from_numpy(np.asarray(ks, dtype=np.int32)).to(cuda)
    b = torch.from_numpy(np.asarray(ke, dtype=np.int32)).to(cuda)
    out = torch.full((lg.shape[0], k), -7, dtype=torch.int32, device=cuda)
    mk = lg.shape[1] if max_keys is None else max_keys
    rc = so.ssb_topk_canonical(lg.data_ptr(), lg.shape[0], lg.shape[1], a.data_ptr(), b.data_ptr(), k, out.data_ptr(),
                               mk, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    lib.check("ssb_topk_canonical", rc)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("case", ["ties", "dense", "wide_ties"])
def test_matches_reference_fixture(cuda, case):
    z = np.load(GOLDEN / "topk_canon.npz")
    g = {k.split("__", 1)[1]: z[k] for k in z.files if k.startswith(case + "__")}
    np.testing.assert_array_equal(gpu_topk(cuda, g["logits"], g["ks"], g["ke"], int(g["k"])), g["out"])


def test_reference_known_answer(cuda):
    logits = np.array([[9., 2., 7., 2., 0., 2.], [5., 5., 1., 3., 8., 8.], [1., 6., 4., 0., 5., 3.]], dtype=np.float32)
    assert gpu_topk(cuda, logits, [0, 2, 0], [6, 4, 6], 3).tolist() == [[0, 1, 2], [0, 1, -1], [1, 2, 4]]


@pytest.mark.parametrize("rows,width,k,levels,max_keys", [
    (64, 5000, 512, 9, None),        # heavy ties, cached rows
    (16, 70000, 2048, 0, None),      # rows longer than the shared-memory cache: re-read per pass
    (32, 3000, 512, 2, 1000),        # max_keys hint below the row length: streamed rows
    (40, 2048, 2048, 0, None),       # k equal to the longest row
])
def test_matches_oracle(cuda, rows, width, k, levels, max_keys):
    rng = np.random.default_rng(rows * width + k)
    if levels:
        logits = rng.integers(-levels, levels, size=(rows, width)).astype(np.float32) * 0.5
    else:
        logits = rng.standard_normal((rows, width)).astype(np.float32)
    ks = rng.integers(0, width // 4, size=rows).astype(np.int32)
    ke = np.minimum(width, ks + rng.integers(0, width, size=rows)).astype(np.int32)
    ke[0] = ks[0]                              # empty row
    ke[1] = min(width, ks[1] + k - 1)           # fewer keys than k
    logits[2, :] = -np.inf                     # a row of equal values
    np.testing.assert_array_equal(gpu_topk(cuda, logits, ks, ke, k, max_keys), otopk.canonical_topk(logits, ks, ke, k))
