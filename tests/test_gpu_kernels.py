"""GPU parity of the single kernels through the C ABI against the CPU oracle: the NVFP4 quantizer (bit-exact), the
tcgen05 NVFP4 GEMM in its three epilogues, and the MoE routing (indices bit-exact on identical logits)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import nvfp4

pytestmark = pytest.mark.gpu


def _lib():
    from ssengine_b200 import lib

    return lib, lib.load()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _rand_operand(rng, rows, K):
    from ssengine_b200 import weights

    codes = rng.integers(0, 16, size=(rows, K), dtype=np.uint8)
    sf = np.asarray(weights.SCALE_CODES, dtype=np.uint8)[rng.integers(0, len(weights.SCALE_CODES), size=(rows, K // 16))]
    return codes, sf


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("rows,K", [(300, 320), (128, 4096), (1, 64)])
def test_quantize_bit_exact(cuda, rows, K):
    lib, so = _lib()
    rng = np.random.default_rng(rows + K)
    x = (rng.standard_normal((rows, K)) * 2).astype(np.float32)
    x[0, :16] = 0.0
    x[0, 16:32] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -5.0, 6.0, 7.0, 1e-3, -1e-3, 40.0, -40.0]
    if rows > 1:
        x[1, :16] = 1e4
    xb = torch.from_numpy(x).to(torch.bfloat16)
    gs = 448.0 * 6 / 8
    ncb = so.ssb_sf_atom_cols(K)
    codes = torch.zeros(rows, K // 2, dtype=torch.uint8, device=cuda)
    sf = torch.zeros(-(-rows // 128) * ncb * 512, dtype=torch.uint8, device=cuda)
    rc = so.ssb_nvfp4_quantize(xb.cuda().data_ptr(), rows, K, K, gs, codes.data_ptr(), K // 2, sf.data_ptr(),
                               _stream())
    lib.check("ssb_nvfp4_quantize", rc)
    torch.cuda.synchronize()
    oc, osf = nvfp4.quantize(xb.float().numpy(), gs)
    np.testing.assert_array_equal(codes.cpu().numpy(), nvfp4.pack(oc))
    np.testing.assert_array_equal(sf.cpu().numpy(), nvfp4.sf_to_atoms(osf))


def _gemm(epi, a, asf, M, K, b, bsf, N, alpha, out, ldo, out_sf=None, out_gs=1.0):
    lib, so = _lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = so.ssb_nvfp4_gemm(epi, a.data_ptr(), asf.data_ptr(), M, K, b.data_ptr(), bsf.data_ptr(), N, alpha,
                           out.data_ptr(), ldo, 0 if out_sf is None else out_sf.data_ptr(), out_gs,
                           status.data_ptr(), _stream())
    lib.check("ssb_nvfp4_gemm", rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0


@pytest.mark.parametrize("M,K,N", [(300, 512, 128), (129, 4096, 8), (1000, 1024, 256)])
def test_gemm_f32_epilogue(cuda, M, K, N):
    rng = np.random.default_rng(M * 7 + N)
    ac, asf = _rand_operand(rng, M, K)
    bc, bsf = _rand_operand(rng, N, K)
    nb = -(-N // 128) * 128
    bcp = np.zeros((nb, K), dtype=np.uint8)
    bcp[:N] = bc
    bsfp = np.zeros((nb, K // 16), dtype=np.uint8)
    bsfp[:N] = bsf
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    _gemm(0, _dev(nvfp4.pack(ac)), _dev(nvfp4.sf_to_atoms(asf)), M, K, _dev(nvfp4.pack(bcp)),
          _dev(nvfp4.sf_to_atoms(bsfp)), N, 0.5, out, N)
    ref = 0.5 * (nvfp4.dequantize(ac, asf, 1.0).astype(np.float64) @ nvfp4.dequantize(bc, bsf, 1.0).T)
    got = out.cpu().numpy()
    scale = np.abs(ref).max()
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5 * scale)


@pytest.mark.parametrize("M,K,N", [(300, 4096, 512), (1, 1024, 256), (129, 1024, 512), (513, 1024, 256)])
def test_gemm_bf16_epilogue(cuda, M, K, N):
    """Dense bf16 GEMMs of more than one 128-row block run on CTA pairs (row blocks 2p, 2p + 1): M = 129 gives a pair
    whose second half holds one row, M = 300 and 513 a last pair whose second half is past M, M = 1 a single CTA.
    The output rows past M and the columns past N of a wider row pitch must keep their sentinel."""
    rng = np.random.default_rng(11 + M)
    ac, asf = _rand_operand(rng, M, K)
    bc, bsf = _rand_operand(rng, N, K)
    ldo, sentinel = N + 64, 12288.0
    buf = torch.full((M + 40, ldo), sentinel, dtype=torch.bfloat16, device=cuda)
    _gemm(1, _dev(nvfp4.pack(ac)), _dev(nvfp4.sf_to_atoms(asf)), M, K, _dev(nvfp4.pack(bc)),
          _dev(nvfp4.sf_to_atoms(bsf)), N, 1e-2, buf, ldo)
    ref = 1e-2 * (nvfp4.dequantize(ac, asf, 1.0).astype(np.float64) @ nvfp4.dequantize(bc, bsf, 1.0).T)
    full = buf.float().cpu().numpy()
    np.testing.assert_allclose(full[:M, :N], ref, rtol=8e-3, atol=1e-3 * np.abs(ref).max())
    assert (full[M:] == sentinel).all() and (full[:M, N:] == sentinel).all()


def test_gemm_swiglu_requant_epilogue(cuda):
    from ssengine_b200 import layout

    M, K, F = 300, 512, 256
    rng = np.random.default_rng(12)
    ac, asf = _rand_operand(rng, M, K)
    bc, bsf = _rand_operand(rng, 2 * F, K)          # logical: gate rows [0, F), up rows [F, 2F)
    bci = layout.gate_up_interleave(torch.from_numpy(bc)).numpy()
    bsfi = layout.gate_up_interleave(torch.from_numpy(bsf)).numpy()
    alpha, gs_h = 1.0 / 60.0, 448.0 * 6 / 32
    codes = torch.zeros((M, F // 2), dtype=torch.uint8, device=cuda)
    osf = torch.zeros(-(-M // 128) * nvfp4.atom_cols(F) * 512, dtype=torch.uint8, device=cuda)
    _gemm(2, _dev(nvfp4.pack(ac)), _dev(nvfp4.sf_to_atoms(asf)), M, K, _dev(nvfp4.pack(bci)),
          _dev(nvfp4.sf_to_atoms(bsfi)), 2 * F, alpha, codes, F // 2, osf, gs_h)
    gu = alpha * (nvfp4.dequantize(ac, asf, 1.0) @ nvfp4.dequantize(bc, bsf, 1.0).T)
    h = omoe.silu(gu[:, :F].astype(np.float32)) * gu[:, F:].astype(np.float32)
    rc_, rs_ = nvfp4.quantize(h, gs_h)
    got_c = nvfp4.unpack(codes.cpu().numpy())
    got_s = nvfp4.atoms_to_sf(osf.cpu().numpy(), M, F // 16)
    # codes and scales agree except where h sits on a rounding boundary (fp32 summation order)
    assert (got_c == rc_).mean() > 0.99 and (got_s == rs_).mean() > 0.99
    d_gpu = nvfp4.dequantize(got_c, got_s, gs_h)
    d_ref = nvfp4.dequantize(rc_, rs_, gs_h)
    assert np.linalg.norm(d_gpu - d_ref) / np.linalg.norm(d_ref) < 1e-2


@pytest.mark.parametrize("T,E,k", [(1000, 128, 8), (257, 8, 2), (64, 288, 8), (33, 512, 31)])
def test_route_indices_bit_exact(cuda, T, E, k):
    lib, so = _lib()
    rng = np.random.default_rng(T + E)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[: T // 2] = np.round(logits[: T // 2] * 2) / 2        # many exact ties
    lg = _dev(logits)
    ids = torch.zeros((T, k), dtype=torch.int32, device=cuda)
    w = torch.zeros((T, k), dtype=torch.float32, device=cuda)
    lib.check("ssb_moe_route", so.ssb_moe_route(lg.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr(), _stream()))
    torch.cuda.synchronize()
    rid, rw = omoe.route_softmax_topk(logits, k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T,E,k,n_group,topk_group", [(8192, 288, 8, 1, 1), (1000, 256, 8, 8, 4), (77, 64, 6, 4, 3),
                                                      (33, 512, 31, 1, 1)])
def test_sigmoid_route_bit_exact(cuda, T, E, k, n_group, topk_group):
    """ssb_moe_route_sigmoid (the reference model's routing) against the oracle: ids bit-exact (ties to the lower
    expert / group included), weights within one fp32 ulp (the same fp32 operations; the sigmoid goes through a
    double-precision exp on both sides)."""
    lib, so = _lib()
    rng = np.random.default_rng(T + E + n_group)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[: T // 2] = np.round(logits[: T // 2] * 2) / 2        # many exact ties
    bias = (12.4 + rng.uniform(0, 0.52, E)).astype(np.float32) if n_group == 1 else \
        (np.round(rng.uniform(0, 0.1, E) * 8) / 8).astype(np.float32)
    ids = torch.zeros((T, k), dtype=torch.int32, device=cuda)
    w = torch.zeros((T, k), dtype=torch.float32, device=cuda)
    lg, bs = _dev(logits), _dev(bias)              # held until the kernel has run
    lib.check("ssb_moe_route_sigmoid", so.ssb_moe_route_sigmoid(lg.data_ptr(), T, E, k, bs.data_ptr(), n_group,
                                                                topk_group, 2.5, ids.data_ptr(), w.data_ptr(),
                                                                _stream()))
    torch.cuda.synchronize()
    rid, rw = omoe.route_sigmoid_bias(logits, k, bias, n_group, topk_group, 2.5)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1.2e-7, atol=0)


def test_sigmoid_route_reference_case(cuda):
    """The reference's own routing test case (tests/golden/routing_ref.npz, from its moe_tuning `forced_logits`):
    the kernel selects exactly the experts the reference's rule selects."""
    from pathlib import Path

    lib, so = _lib()
    f = np.load(Path(__file__).resolve().parent / "golden" / "routing_ref.npz")
    sel = np.unpackbits(f["selected"], axis=1)[:, :288].astype(bool)
    logits = np.where(sel, np.float32(30.0), np.float32(-30.0))
    T = logits.shape[0]
    ids = torch.zeros((T, 8), dtype=torch.int32, device=cuda)
    w = torch.zeros((T, 8), dtype=torch.float32, device=cuda)
    lg, bs = _dev(logits), _dev(f["bias"])        # held until the kernel has run
    lib.check("ssb_moe_route_sigmoid", so.ssb_moe_route_sigmoid(lg.data_ptr(), T, 288, 8, bs.data_ptr(), 1, 1, 2.5,
                                                                ids.data_ptr(), w.data_ptr(), _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(np.sort(ids.cpu().numpy(), axis=1), f["ids_sorted"])


@pytest.mark.parametrize("rows,heads", [(300, 8), (1, 64), (1000, 64), (129, 3)])
def test_gated_rmsnorm_nvfp4_equals_norm_then_quantize(cuda, rows, heads):
    """ssb_gated_rmsnorm_nvfp4 writes the same codes and scale atoms as ssb_gated_rmsnorm followed by
    ssb_nvfp4_quantize (heads = 3: 384 columns, the atom columns up to the 256-column padding stay zero)."""
    lib, so = _lib()
    P = heads * 128
    gen = torch.Generator(device=cuda).manual_seed(rows + heads)
    x = (torch.randn(rows, P, device=cuda, generator=gen) * 3).to(torch.bfloat16)
    gate = torch.randn(rows, P, device=cuda, generator=gen).to(torch.bfloat16)
    w = (torch.rand(128, device=cuda, generator=gen) + 0.5).to(torch.bfloat16)
    gs, eps = 448.0 * 6.0 / 12.0, 1e-5
    rp = -(-rows // 128) * 128
    nsf = rp // 128 * so.ssb_sf_atom_cols(P) * 512
    y = torch.empty_like(x)
    lib.check("ssb_gated_rmsnorm", so.ssb_gated_rmsnorm(x.data_ptr(), P, gate.data_ptr(), P, w.data_ptr(), eps,
                                                        y.data_ptr(), P, rows, heads, _stream()))
    c1 = torch.zeros(rp, P // 2, dtype=torch.uint8, device=cuda)
    s1 = torch.zeros(nsf, dtype=torch.uint8, device=cuda)
    lib.check("ssb_nvfp4_quantize", so.ssb_nvfp4_quantize(y.data_ptr(), rows, P, P, gs, c1.data_ptr(), P // 2,
                                                          s1.data_ptr(), _stream()))
    c2 = torch.zeros_like(c1)
    s2 = torch.zeros_like(s1)
    lib.check("ssb_gated_rmsnorm_nvfp4", so.ssb_gated_rmsnorm_nvfp4(x.data_ptr(), P, gate.data_ptr(), P, w.data_ptr(),
                                                                    eps, gs, c2.data_ptr(), P // 2, s2.data_ptr(),
                                                                    rows, heads, _stream()))
    torch.cuda.synchronize()
    assert torch.equal(c1, c2) and torch.equal(s1, s2)
