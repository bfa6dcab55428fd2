"""GPU parity of the KDA prefill (`ssb_kda_prefill`, `ssb_kda_conv`) against the oracle (oracle/kda.py): ragged
sequences (1 row, partial and whole 64-token chunks, several chunks), fresh and continued requests, rows outside every
sequence, states of other blocks untouched, and a request split across two calls.

Tolerances: conv outputs within one bf16 step of the oracle (the kernel's SiLU uses the fast __expf / __fdividef
intrinsics, the oracle exact exp) and >= 99% bit-equal; conv state blocks bit-exact (copies); KDA outputs and final
recurrent states within 2e-2 relative L2 of the float64 token-by-token recurrence (the chunked scan rounds its
tensor-core operands to bf16; measured on the CPU model of the same factorisation: ~3e-3)."""

import numpy as np
import pytest
import torch

from oracle import kda as ok
from oracle.mhc import bf16

pytestmark = pytest.mark.gpu

D = 128


def make(rng, T, H, blocks):
    P = H * D
    return dict(
        x=bf16(rng.standard_normal((T, 3 * P + 8))),          # wider rows: the projection's extra columns
        w=bf16(rng.uniform(-0.6, 0.6, (3 * P, 4))),
        g=bf16(rng.standard_normal((T, P))),
        beta=bf16(rng.standard_normal((T, H))),
        a_log=rng.uniform(-1, 1, H).astype(np.float32),
        dtb=(rng.standard_normal(P) * 0.5).astype(np.float32),
        cst=bf16(rng.standard_normal((blocks, 3, 3 * P))),
        rst=(rng.standard_normal((blocks, H, D, D)) * 0.05).astype(np.float32),
    )


def layer(cuda, d):
    from ssengine_b200.kda import KdaLayer

    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(cuda)
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)
    L = KdaLayer(bf(d["w"]), f32(d["a_log"]), f32(d["dtb"]), -5.0)
    dev = dict(x=bf(d["x"]), g=bf(d["g"]), beta=bf(d["beta"]), cst=bf(d["cst"]), rst=f32(d["rst"]))
    return L, dev


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_close(got, want):
    ulp = np.maximum(np.abs(want), 2.0 ** -126) * 2.0 ** -7
    diff = np.abs(got - want)
    assert (diff <= ulp).all(), float((diff / ulp).max())
    assert (diff == 0).mean() >= 0.99


def run_prefill(cuda, d, seqs, H):
    from ssengine_b200.kda import seq_table

    L, dev = layer(cuda, d)
    T = d["x"].shape[0]
    out = torch.zeros(T, H * D, dtype=torch.bfloat16, device=cuda)
    L.prefill(dev["x"], dev["g"], dev["beta"], out, seq_table(seqs, cuda), dev["cst"], dev["rst"])
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), dev["cst"].float().cpu().numpy(), dev["rst"].cpu().numpy()


SEQS = [(0, 1, 1, 1), (1, 64, 2, 0), (64, 129, 3, 1), (129, 131, 4, 1), (140, 340, 5, 0), (340, 468, 6, 1)]


@pytest.mark.parametrize("H", [2])
def test_conv_matches_oracle(cuda, H):
    from ssengine_b200.kda import seq_table

    rng = np.random.default_rng(11)
    T, P = 470, H * D
    d = make(rng, T, H, 8)
    L, dev = layer(cuda, d)
    q, k, v = L.conv_qkv(dev["x"], seq_table(SEQS, cuda), dev["cst"], dev["rst"])
    torch.cuda.synchronize()
    oq, okk, ov, ost = ok.conv(d["x"][:, :3 * P], d["w"], d["cst"], SEQS, P)
    for got, want in ((q, oq), (k, okk), (v, ov)):
        bf16_close(got.float().cpu().numpy(), want)
    np.testing.assert_array_equal(dev["cst"].float().cpu().numpy(), ost)
    assert not q[131:140].any() and not q[468:].any()       # rows outside every sequence


@pytest.mark.parametrize("H", [2, 4])
def test_prefill_matches_oracle(cuda, H):
    rng = np.random.default_rng(100 + H)
    T, P = 470, H * D
    d = make(rng, T, H, 8)
    out, cst, rst = run_prefill(cuda, d, SEQS, H)
    want, wcst, wrst = ok.prefill(d["x"][:, :3 * P], d["w"], d["cst"], d["g"], d["beta"], d["a_log"], d["dtb"], -5.0,
                                  d["rst"], SEQS, H, D)
    for s, e, blk, _ in SEQS:
        assert rel(out[s:e], want[s:e]) < 2e-2, (s, e, rel(out[s:e], want[s:e]))
        assert rel(rst[blk], wrst[blk]) < 2e-2, (blk, rel(rst[blk], wrst[blk]))
    assert not out[131:140].any() and not out[468:].any()
    np.testing.assert_array_equal(rst[0], d["rst"][0])       # blocks of no sequence untouched
    np.testing.assert_array_equal(rst[7], d["rst"][7])
    np.testing.assert_array_equal(cst, wcst)


def test_split_request_equals_whole(cuda):
    """One request computed in two calls (the second continuing from the first's state blocks) agrees with one call
    and with the oracle."""
    H = 2
    rng = np.random.default_rng(7)
    T, cut = 300, 117
    d = make(rng, T, H, 2)
    whole, wc, wr = run_prefill(cuda, d, [(0, T, 1, 1)], H)

    from ssengine_b200.kda import seq_table

    L, dev = layer(cuda, d)
    out = torch.zeros(T, H * D, dtype=torch.bfloat16, device=cuda)
    L.prefill(dev["x"], dev["g"], dev["beta"], out, seq_table([(0, cut, 1, 1)], cuda), dev["cst"], dev["rst"])
    L.prefill(dev["x"][cut:], dev["g"][cut:], dev["beta"][cut:], out[cut:], seq_table([(0, T - cut, 1, 1)], cuda),
              dev["cst"], dev["rst"])
    torch.cuda.synchronize()
    split = out.float().cpu().numpy()
    assert rel(split, whole) < 1e-2
    np.testing.assert_array_equal(dev["cst"].float().cpu().numpy(), wc)
    assert rel(dev["rst"].cpu().numpy()[1], wr[1]) < 1e-2
    want, _, _ = ok.prefill(d["x"][:, :3 * H * D], d["w"], d["cst"], d["g"], d["beta"], d["a_log"], d["dtb"], -5.0,
                            d["rst"], [(0, T, 1, 1)], H, D)
    assert rel(split, want) < 2e-2


def test_workspace_paths_agree(cuda):
    """The caller-workspace entry (exact size), the shared scratch and the self-allocating `ssb_kda_prefill` give the
    same bits; a workspace one byte short is refused (code 3) before anything runs."""
    import ctypes

    from ssengine_b200 import lib
    from ssengine_b200.kda import seq_table, workspace_bytes

    H = 2
    rng = np.random.default_rng(21)
    T = 470
    d = make(rng, T, H, 8)
    outs = []
    for mode in ("exact", "scratch", "alloc"):
        L, dev = layer(cuda, d)
        out = torch.zeros(T, H * D, dtype=torch.bfloat16, device=cuda)
        st = seq_table(SEQS, cuda)
        if mode == "alloc":
            so = lib.load()
            C = L.c_struct(dev["cst"], dev["rst"])
            rc = so.ssb_kda_prefill(ctypes.byref(C), dev["x"].data_ptr(), dev["x"].stride(0), dev["g"].data_ptr(),
                                    dev["g"].stride(0), dev["beta"].data_ptr(), dev["beta"].stride(0), T,
                                    st.data_ptr(), st.shape[0], out.data_ptr(), out.stride(0), None,
                                    lib.stream_ptr(None))
            assert rc == 0
        else:
            ws = torch.empty(workspace_bytes(H, T, len(SEQS)), dtype=torch.uint8, device=cuda) if mode == "exact" \
                else None
            L.prefill(dev["x"], dev["g"], dev["beta"], out, st, dev["cst"], dev["rst"], workspace=ws)
        torch.cuda.synchronize()
        outs.append((out.cpu(), dev["rst"].cpu(), dev["cst"].cpu()))
    for o, r, c in outs[1:]:
        assert torch.equal(o, outs[0][0]) and torch.equal(r, outs[0][1]) and torch.equal(c, outs[0][2])

    L, dev = layer(cuda, d)
    st = seq_table(SEQS, cuda)
    short = torch.empty(workspace_bytes(H, T, len(SEQS)) - 1, dtype=torch.uint8, device=cuda)
    so = lib.load()
    C = L.c_struct(dev["cst"], dev["rst"])
    out = torch.zeros(T, H * D, dtype=torch.bfloat16, device=cuda)
    rc = so.ssb_kda_prefill_ws(ctypes.byref(C), dev["x"].data_ptr(), dev["x"].stride(0), dev["g"].data_ptr(),
                               dev["g"].stride(0), dev["beta"].data_ptr(), dev["beta"].stride(0), T, st.data_ptr(),
                               st.shape[0], out.data_ptr(), out.stride(0), short.data_ptr(), short.numel(), None,
                               lib.stream_ptr(None))
    assert rc == 3


def test_rejected_sequences_leave_state(cuda):
    """Sequences whose chunks exceed the workspace (rows summing above T) raise status 6, a sequence reaching past T
    raises 1; their state blocks stay as they were while the valid sequence is computed as usual."""
    from ssengine_b200.kda import seq_table

    H = 2
    rng = np.random.default_rng(23)
    T = 130
    d = make(rng, T, H, 4)
    for seqs, code in (([(0, 130, 1, 1), (0, 130, 2, 1)], 6), ([(0, 130, 1, 1), (100, 140, 2, 1)], 1)):
        L, dev = layer(cuda, d)
        out = torch.zeros(T, H * D, dtype=torch.bfloat16, device=cuda)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        L.prefill(dev["x"], dev["g"], dev["beta"], out, seq_table(seqs, cuda), dev["cst"], dev["rst"], status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == code
        rst, cst = dev["rst"].cpu().numpy(), dev["cst"].float().cpu().numpy()
        np.testing.assert_array_equal(rst[2], d["rst"][2])
        np.testing.assert_array_equal(cst[2], d["cst"][2])
        want, _, wrst = ok.prefill(d["x"][:, :3 * H * D], d["w"], d["cst"], d["g"], d["beta"], d["a_log"], d["dtb"],
                                   -5.0, d["rst"], [(0, 130, 1, 1)], H, D)
        assert rel(out.float().cpu().numpy(), want) < 2e-2
        assert rel(rst[1], wrst[1]) < 2e-2
