"""The oracle against the library implementations the reference's mHC, KDA and NVFP4 steps come from: upstream vLLM
0.22.0's `mhc_pre_torch` / `mhc_post_torch`, `rms_norm` and the KDA gated norm, `fp8_mqa_logits_torch` (DeepGEMM's
reference of the indexer score), `reference_mla_sparse_prefill` (FlashMLA's reference of sparse MLA prefill),
FLA `chunk_kda` (and flash-linear-attention 0.5.1's own fp32 references `naive_recurrent_kda` /
`naive_kda_lowerbound_gate`), `causal_conv1d_fn`, `scaled_fp4_quant` and the CUTLASS NVFP4 MoE (`run_cutlass_moe_fp4`), whose outputs on
seeded inputs are
committed under tests/golden/ (made by tests/golden/make_vllm_golden.py; the inputs are regenerated here from the
same seeds). Tolerances are stated per assert, each with the margin over the measured difference."""

import sys
from pathlib import Path

import numpy as np

from oracle import kda, mhc, nvfp4

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_vllm_golden as gen  # noqa: E402

BF16_STEP = 2.0 ** -7          # one bf16 step relative to the value, at most


def test_mhc_pre_matches_vllm():
    f = np.load(GOLDEN / "mhc_vllm.npz")
    i, e = gen.mhc_inputs(), gen.MHC_EPS
    post_mix, comb, li = mhc.pre_mixes(i["res"], i["fn"], i["scale"], i["base"], e["rms_eps"], e["pre_eps"],
                                       e["sinkhorn_eps"], e["post_mult"], e["repeat"])
    # fp32 (vLLM) against float64 (oracle): measured 2.7e-7 of the largest value
    np.testing.assert_allclose(post_mix, f["pre_post_mix"], rtol=0, atol=2e-6 * np.abs(f["pre_post_mix"]).max())
    np.testing.assert_allclose(comb, f["pre_comb"], rtol=0, atol=2e-6 * np.abs(f["pre_comb"]).max())
    # the bf16 layer input: measured identical
    np.testing.assert_array_equal(li, f["pre_layer_input"])


def test_mhc_post_matches_vllm():
    f = np.load(GOLDEN / "mhc_vllm.npz")
    i = gen.mhc_inputs()
    got, want = mhc.post(i["x"], i["res"], i["post_mix"], i["comb"]), f["post_new_res"]
    diff = got != want
    # fp32 and float64 sums round to bf16 alike but where they straddle a rounding boundary: measured 1 of 6,144
    assert diff.mean() <= 1e-3, diff.sum()
    assert (np.abs(got - want)[diff] <= BF16_STEP * np.abs(want)[diff]).all()


def test_kda_recurrence_matches_vllm_chunk_kda():
    f = np.load(GOLDEN / "kda_vllm.npz")
    i = gen.kda_inputs()
    H, D = i["H"], i["D"]
    out, state = kda.recurrent(i["q"], i["k"], i["v"], i["g"], i["beta"], i["a_log"], i["dt_bias"],
                               gen.KDA_LOWER_BOUND, D ** -0.5, i["state"], gen.KDA_SEQS, H, D)

    def rel(a, b):
        return np.linalg.norm(a - b) / np.linalg.norm(b)

    # chunk_kda keeps q, k, v and the solved triangular block in bf16: measured 4.0e-3 (output), 3.2e-3 (states)
    assert rel(out, f["chunk_o"]) < 1e-2
    for n, (s, e, blk, _) in enumerate(gen.KDA_SEQS):
        assert rel(out[s:e], f["chunk_o"][s:e]) < 1e-2, n
        assert rel(state[blk], f["chunk_state"][n]) < 1e-2, n


def test_nvfp4_quantizer_matches_vllm_scaled_fp4_quant():
    f = np.load(GOLDEN / "nvfp4_vllm.npz")
    i = gen.nvfp4_inputs()
    x, gs = i["x"], i["gs"]
    codes, sf = nvfp4.quantize(x, gs)
    # the swizzled scale layout vLLM writes is the 128x4-atom layout of the GEMM operands
    np.testing.assert_array_equal(nvfp4.sf_to_atoms(f["sf"]), f["sf_swizzled"])
    # scales: identical except where (amax / 6) * gs sits on an e4m3 rounding midpoint (measured 4 of 6,400 blocks):
    # there vLLM's amax * (1/6) lands on the other side, one scale step away
    differ = sf != f["sf"]
    assert differ.sum() <= 8, differ.sum()
    amax = np.abs(x).reshape(x.shape[0], -1, 16).max(axis=2)
    for r, b in np.argwhere(differ):
        lo, hi = sorted(nvfp4.e4m3_decode(np.array([sf[r, b], f["sf"][r, b]])))
        assert abs(int(sf[r, b]) - int(f["sf"][r, b])) == 1
        sf_f = np.float32(amax[r, b] / np.float32(6.0)) * np.float32(gs)
        assert abs(sf_f - (lo + hi) / 2) <= 4 * np.spacing(np.float32(sf_f)), (r, b)
    # codes: byte-identical, signed zeros included, in every block whose scale agrees
    same = np.repeat(~differ, 16, axis=1)
    vcodes = nvfp4.unpack(f["codes"])
    np.testing.assert_array_equal(codes[same], vcodes[same])
    assert (vcodes == 8).any()          # the fixture holds negative zeros


def test_moe_experts_match_vllm_cutlass_nvfp4_moe():
    from ssengine_b200 import weights

    from oracle import moe as omoe

    f = np.load(GOLDEN / "moe_vllm.npz")
    c = gen.MOE_CASE
    p = weights.to_numpy(weights.moe_logical(c["seed"], c["H"], c["F"], c["E"]))
    x = weights.hidden_states(c["seed"] + 1, c["T"], c["H"]).float().numpy()
    ref, parts = omoe.moe_forward(x, p, c["k"], return_parts=True)
    # the routing the fixture was made with is the oracle's own
    np.testing.assert_array_equal(parts["ids"], f["ids"])
    np.testing.assert_array_equal(parts["weights"], f["weights"])
    got = (f["out_bf16"].astype(np.uint32) << 16).view(np.float32)

    def rel(a, b):
        return np.linalg.norm(a - b) / np.linalg.norm(b)

    # with vLLM's bf16 intermediates restated, the same algorithm: measured 1.2e-4 (fp32 summation order)
    same = omoe.moe_forward(x, p, c["k"], ids=f["ids"], weights=f["weights"], intermediates="bf16")
    assert rel(got, same) < 1e-3
    # the layer's own fp32 intermediates: measured 2.4e-2, inside the per-layer bar of 3e-2
    assert rel(got, ref) < 3e-2


def test_indexer_logits_match_deepgemm_reference():
    from oracle import indexer

    f = np.load(GOLDEN / "indexer_vllm.npz")["logits"]
    i = gen.indexer_inputs()
    pages = np.arange(i["k"].shape[0] // indexer.POOLS_PER_PAGE)     # pool p at cache row p
    rows = indexer.logits(i["q"], i["w"], i["k"], pages, i["positions"])
    assert any(len(r) == 0 for r in rows) and max(len(r) for r in rows) > 50
    for r, row in enumerate(rows):
        n = len(row)
        # the same visibility: pools < (pos + 1) / 4 are scored, the rest masked to -inf
        assert np.isfinite(f[r, :n]).all() and np.isneginf(f[r, n:]).all(), r
        # the reference rounds each head's score to bf16 before the ReLU: measured 3.2e-3 of the row's largest logit
        if n:
            assert np.abs(row - f[r, :n]).max() <= 1e-2 * np.abs(row).max(), r


def test_norms_match_vllm():
    from oracle import stage
    from oracle.mhc import bf16

    f = np.load(GOLDEN / "norms_vllm.npz")
    i = gen.norm_inputs()
    # the KDA output norm (sigmoid gate, per head): identical after the bf16 rounding of the output
    np.testing.assert_array_equal(bf16(kda.gated_rmsnorm(i["o"], i["gate"], i["gw"], i["eps"], D=i["D"])), f["gated"])
    # RMSNorm: vLLM rounds the normalized row to bf16 before the weight multiply; with that order restated the bytes
    # are identical, and this build's single rounding stays within one bf16 step (measured: 1,045 of 4,096 values)
    x = i["x"].astype(np.float32)
    inv = (1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + i["eps"])).astype(np.float32)
    np.testing.assert_array_equal(bf16(bf16(x * inv) * i["w"]), f["rms"])
    ours = bf16(stage.rmsnorm(i["x"], i["w"], i["eps"]))
    assert (np.abs(ours - f["rms"]) <= BF16_STEP * np.abs(f["rms"])).all()


def test_sparse_mla_matches_flashmla_reference():
    from oracle import mla

    f = np.load(GOLDEN / "mla_vllm.npz")
    i = gen.mla_inputs()
    pages = np.arange(3)                           # position p at cache row p (three 128-token pages)
    got = mla.sparse_mla(i["q8"], i["kv8"], i["indices"], pages, i["bmm1"], 1.0)
    # -1 fills skipped, repeated tokens counted twice, rows shorter than the selection: fp32 reference against the
    # float64 oracle, measured 2.0e-7 relative L2 (5.1e-7 absolute on values up to 2)
    np.testing.assert_allclose(got, f["out"], rtol=0, atol=5e-6)


def test_kda_gate_and_recurrence_match_fla_naive_reference():
    f = np.load(GOLDEN / "kda_fla.npz")
    i = gen.kda_inputs()
    H, D, T = i["H"], i["D"], i["q"].shape[0]
    # the lower-bound gate: measured 6.5e-7 absolute (fp32 against float64) on decays in [-5, 0]
    g = kda.gate(i["g"], i["a_log"], i["dt_bias"], gen.KDA_LOWER_BOUND, H, D).reshape(T, H * D)
    np.testing.assert_allclose(g, f["gate"], rtol=0, atol=5e-6)
    out, state = kda.recurrent(i["q"], i["k"], i["v"], i["g"], i["beta"], i["a_log"], i["dt_bias"],
                               gen.KDA_LOWER_BOUND, D ** -0.5, i["state"], gen.KDA_SEQS, H, D)

    def rel(a, b):
        return np.linalg.norm(a - b) / np.linalg.norm(b)

    # FLA's fp32 token-by-token reference: measured 1.4e-7 (outputs) and 9e-8 (final states) relative L2
    assert rel(out, f["o"]) < 1e-5
    for n, (_, _, blk, _) in enumerate(gen.KDA_SEQS):
        assert rel(state[blk], f["state"][n]) < 1e-5, n


def test_kda_conv_matches_vllm_causal_conv1d():
    f = np.load(GOLDEN / "conv_vllm.npz")
    i = gen.conv_inputs()
    # the window, the conv-state read for a continuing sequence, zeros for a fresh one, the write-back of the last three
    # rows: with vLLM's rounding of each product to bf16 restated, identical bytes and states
    q, k, v, st = kda.conv(i["x"], i["w"], i["state"], gen.KDA_SEQS, i["P"], bf16_products=True)
    np.testing.assert_array_equal(np.concatenate([q, k, v], axis=1), f["out"])
    for n, (_, _, blk, _) in enumerate(gen.KDA_SEQS):
        np.testing.assert_array_equal(st[blk], f["state"][n])
    # exact fp32 products (Dao's channel-last arithmetic, which the reference's conv reproduces bitwise): measured
    # 0.031 absolute on outputs up to 4.1
    q, k, v, _ = kda.conv(i["x"], i["w"], i["state"], gen.KDA_SEQS, i["P"])
    assert np.abs(np.concatenate([q, k, v], axis=1) - f["out"]).max() <= 0.02 * np.abs(f["out"]).max()


def test_mla_rope_matches_vllm_rotary_embedding():
    """oracle.dsa.rope against vLLM's MLA rotary embedding (interleaved pairs, theta 10000, fp32 cos / sin cache).
    vLLM forms each angle as fp32 position x fp32 inverse frequency, off the exact angle by up to ~2^-23 x position
    radians; the oracle uses exact angles, so the bound grows with the position (measured: 1.9e-4 below position
    2,048, 1.0e-2 near 131,072); the other pairing convention (NeoX halves) would be off by ~8."""
    from oracle import dsa

    f = np.load(GOLDEN / "rope_vllm.npz")
    i = gen.rope_inputs()
    q = dsa.rope(i["q"], i["pos"], gen.ROPE_THETA)
    k = dsa.rope(i["k"][:, None, :], i["pos"], gen.ROPE_THETA)[:, 0]
    for ours, ref, x in ((q, f["q"], i["q"]), (k, f["k"], i["k"][:, None, :])):
        amax = np.abs(x).reshape(len(x), -1).max(axis=1)
        bound = 2.0 * (i["pos"] * 2.0 ** -23 + 2.0 ** -20) * amax
        err = np.abs(ours - ref).reshape(len(x), -1).max(axis=1)
        assert (err <= bound).all(), float((err / bound).max())
    short = i["pos"] < 2048
    assert np.abs(q[short] - f["q"][short]).max() < 5e-4


def test_dsa_latent_rmsnorm_matches_vllm():
    """oracle.dsa.rmsnorm (the q_a / kv latent norms) against vLLM's `rms_norm`: within one bf16 step."""
    from oracle import dsa
    from oracle.mhc import bf16

    f = np.load(GOLDEN / "norms_vllm.npz")
    i = gen.norm_inputs()
    ours = bf16(dsa.rmsnorm(i["x"], i["w"], i["eps"]))
    assert (np.abs(ours - f["rms"]) <= BF16_STEP * np.abs(f["rms"])).all()


def test_fp8_indexer_format_and_logits_match_vllm():
    """The FP8 indexer (the reference's 132-byte pool entries) against vLLM's own kernels run on the CPU: query codes
    and ue8m0 scales bit-exact, the paged cache (32 entries a page: codes, then fp32 scales) byte-exact, and the
    logits within the reference's per-head bf16 score rounding (measured 3.2e-3 of a row's largest logit on the bf16
    fixture; bound 1e-2)."""
    from oracle import indexer

    f = np.load(GOLDEN / "indexer_fp8_vllm.npz")
    i = gen.indexer_inputs()
    qc, qs = indexer.quant_query_heads(i["q"])
    np.testing.assert_array_equal(qc, f["q_codes"])
    np.testing.assert_array_equal(qs, f["q_scale"])
    pages = np.asarray(gen.INDEXER_FP8_PAGES)
    n = i["k"].shape[0]
    rows = indexer.pool_rows(pages, n)
    kc, ks = indexer.quant_pool_rows(i["k"])
    cache = indexer.write_pool_pages(np.zeros_like(f["cache"]), rows, kc, ks)
    np.testing.assert_array_equal(cache, f["cache"])
    out = indexer.logits_fp8(qc, qs, i["w"], cache, pages, i["positions"])
    for r, row in enumerate(out):
        m = len(row)
        assert np.isneginf(f["logits"][r, m:]).all()
        if m:
            assert np.abs(row - f["logits"][r, :m]).max() <= 1e-2 * np.abs(row).max(), r
