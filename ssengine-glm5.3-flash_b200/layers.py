"""Layer blocks of a Glm5Next stage built from the library's kernels: the NVFP4 dense projection and the KDA attention
block (in_proj -> gate projections -> conv + chunked delta-rule scan -> gated RMSNorm -> o_proj).

Mirrors the fork's `Glm5NextLinearAttention` forward as the reference's manifest orders it (ssengine/kernels.py
configs 2-6: in_proj k 4096 n 24896, f_b / g_b k 128 n 8192 on column views of in_proj, short conv, chunk prefill,
o_proj k 8192 n 4096; `kda_prefill_forward` ssengine/model/pp_patch.py:215-244), with the projections as NVFP4 GEMMs
(the north star's choice; the reference runs them in BF16). in_proj output columns: q | k | v (3P) | f_a (128) |
g_a (128) | beta (H heads), padded to a multiple of 256. No fallback: without the CUDA library these calls raise.
"""

from __future__ import annotations

import torch

from . import layout, lib, weights
from .kda import HEAD_DIM, KdaLayer

LOW_RANK = 128


def _round(n: int, m: int) -> int:
    return -(-n // m) * m


class Nvfp4Linear:
    """y bf16 [T, N] = x bf16 [T, K] @ W^T with W NVFP4 (e2m1 codes, e4m3 per-16 scales, fp32 global scale); the
    activation is quantized with the static global scale `gs_in` (unit-variance inputs)."""

    def __init__(self, codes: torch.Tensor, sf: torch.Tensor, gs_w: float, device, gs_in: float = weights.GS_X):
        N, K = codes.shape
        self.N, self.K = N, K
        self.N_pad = _round(N, 256)
        dev = torch.device(device)
        c = torch.zeros(self.N_pad, K, dtype=torch.uint8, device=dev)
        c[:N] = codes.to(dev)
        s = torch.zeros(self.N_pad, K // 16, dtype=torch.uint8, device=dev)
        s[:N] = sf.to(dev)
        self.codes = layout.pack_codes(c).contiguous()
        self.sf = layout.sf_to_atoms(s, K)
        self.gs_in = gs_in
        self.alpha = float(1.0 / (gs_in * gs_w))
        self.device = dev
        self._lib = lib.load()

    @classmethod
    def random(cls, gen: torch.Generator, N: int, K: int, device, gs_in: float = weights.GS_X, in_sq_mean: float = 1.0):
        """Random-init NVFP4 weights (BASELINE recipe) scaled for unit-variance outputs."""
        codes = torch.randint(0, 16, (N, K), generator=gen, device=device, dtype=torch.uint8)
        table = torch.tensor(weights.SCALE_CODES, dtype=torch.uint8, device=device)
        sf = table[torch.randint(0, len(weights.SCALE_CODES), (N, K // 16), generator=gen, device=device)]
        return cls(codes, sf, weights.unit_gs(K, in_sq_mean), device, gs_in)

    def logical(self):
        """(codes [N, K], sf [N, K / 16], gs_w) as stored (for the checker)."""
        codes = layout.unpack_codes(self.codes)[:self.N]
        sf = layout.atoms_to_sf(self.sf, self.N_pad, self.K)[:self.N]
        return codes, sf, 1.0 / (self.alpha * self.gs_in)

    def __call__(self, x: torch.Tensor, out: torch.Tensor, status: torch.Tensor, stream=None) -> torch.Tensor:
        """x bf16 [T, >= K] (row pitch x.stride(0)), out bf16 [T, >= N_pad] (row pitch out.stride(0))."""
        T = x.shape[0]
        s = lib.stream_ptr(stream)
        rows = _round(max(T, 1), 128)
        codes = torch.empty(rows, self.K // 2, dtype=torch.uint8, device=self.device)
        sf = torch.zeros(rows // 128 * layout.sf_atom_cols(self.K) * 512, dtype=torch.uint8, device=self.device)
        lib.check("ssb_nvfp4_quantize", self._lib.ssb_nvfp4_quantize(x.data_ptr(), T, self.K, x.stride(0), self.gs_in,
                                                                     codes.data_ptr(), self.K // 2, sf.data_ptr(), s))
        lib.check("ssb_nvfp4_gemm", self._lib.ssb_nvfp4_gemm(lib.EPI_BF16, codes.data_ptr(), sf.data_ptr(), T, self.K,
                                                             self.codes.data_ptr(), self.sf.data_ptr(), self.N_pad,
                                                             self.alpha, out.data_ptr(), out.stride(0), None, 1.0,
                                                             status.data_ptr(), s))
        return out


class KdaAttention:
    """The KDA attention block of one layer: hidden H, `heads` heads of 128 (P = heads * 128)."""

    def __init__(self, seed: int, hidden: int, heads: int, device, lower_bound: float = -5.0, norm_eps: float = 1e-5):
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, P = hidden, heads * HEAD_DIM
        self.H, self.heads, self.P = H, heads, P
        self.in_cols = 3 * P + 2 * LOW_RANK + heads
        self.in_proj = Nvfp4Linear.random(g, self.in_cols, H, dev)
        self.f_b = Nvfp4Linear.random(g, P, LOW_RANK, dev)
        self.g_b = Nvfp4Linear.random(g, P, LOW_RANK, dev)
        self.o_proj = Nvfp4Linear.random(g, H, P, dev)
        conv_w = ((torch.rand(3 * P, 4, generator=g, device=dev) - 0.5) * 1.2).to(torch.bfloat16)
        a_log = torch.rand(heads, generator=g, device=dev) * 2 - 1
        dt_bias = torch.randn(P, generator=g, device=dev) * 0.5
        self.kda = KdaLayer(conv_w.contiguous(), a_log, dt_bias, lower_bound)
        self.norm_w = (torch.rand(HEAD_DIM, generator=g, device=dev) + 0.5).to(torch.bfloat16)
        self.norm_eps = norm_eps
        self.device = dev
        self._lib = lib.load()

    def forward(self, y: torch.Tensor, seqs: torch.Tensor, conv_state: torch.Tensor, rec_state: torch.Tensor,
                status: torch.Tensor, out: torch.Tensor | None = None, stream=None, keep: bool = False) -> torch.Tensor:
        """y bf16 [T, H] (the layer input after the boundary's RMSNorm) -> attention output bf16 [T, H]; the KDA state
        blocks of `seqs` (int32 [R, 4] on the device) are updated in place. keep: the intermediates stay in
        `self.parts` (for checks)."""
        T, P, dev = y.shape[0], self.P, self.device
        s = lib.stream_ptr(stream)
        proj = torch.empty(T, self.in_proj.N_pad, dtype=torch.bfloat16, device=dev)
        self.in_proj(y, proj, status, stream)
        f_a = proj[:, 3 * P:3 * P + LOW_RANK]
        g_a = proj[:, 3 * P + LOW_RANK:3 * P + 2 * LOW_RANK]
        beta = proj[:, 3 * P + 2 * LOW_RANK:]
        gate = torch.empty(T, P, dtype=torch.bfloat16, device=dev)
        self.f_b(f_a, gate, status, stream)
        ogate = torch.empty(T, P, dtype=torch.bfloat16, device=dev)
        self.g_b(g_a, ogate, status, stream)
        o = torch.empty(T, P, dtype=torch.bfloat16, device=dev)
        self.kda.prefill(proj, gate, beta, o, seqs, conv_state, rec_state, stream=stream, status=status)
        if keep:
            self.parts = dict(proj=proj, gate=gate, ogate=ogate, o=o.clone())
        lib.check("ssb_gated_rmsnorm", self._lib.ssb_gated_rmsnorm(o.data_ptr(), P, ogate.data_ptr(), P,
                                                                   self.norm_w.data_ptr(), self.norm_eps, o.data_ptr(),
                                                                   P, T, self.heads, s))
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=dev)
        self.o_proj(o, out, status, stream)
        if keep:
            self.parts["normed"] = o
        return out


class MhcBoundary:
    """One mHC layer boundary (4 streams): the previous sub-block's post and the next sub-block's pre + RMSNorm, in one
    `ssb_mhc` launch (the reference's `MegaMhcPostPre`, ssengine/model/pp_patch.py:125-153)."""

    def __init__(self, gen: torch.Generator, hidden: int, device, repeat: int = 20):
        H = hidden
        self.H = H
        self.fn = (torch.randn(24, 4 * H, generator=gen, device=device) / (4 * H) ** 0.5).contiguous()
        self.scale = torch.tensor([0.8, 0.6, 1.5], device=device)
        self.base = torch.randn(24, generator=gen, device=device) * 0.3
        self.norm_w = (torch.rand(H, generator=gen, device=device) + 0.5).to(torch.bfloat16)
        self.eps = dict(rms_eps=1e-6, pre_eps=1e-2, sinkhorn_eps=1e-6, post_mult=2.0, norm_eps=1e-6)
        self.repeat = repeat
        self._c = lib.MhcParamsC(H, 4, self.fn.data_ptr(), self.scale.data_ptr(), self.base.data_ptr(),
                                 self.norm_w.data_ptr(), self.eps["rms_eps"], self.eps["pre_eps"],
                                 self.eps["sinkhorn_eps"], self.eps["post_mult"], self.eps["norm_eps"], repeat)
        self._lib = lib.load()

    def __call__(self, x, res, post_in, comb_in, new_res, post_out, comb_out, y, stream=None) -> None:
        """x = None: pre only (the stage-edge receive) on res; else post of x into new_res, then pre of new_res."""
        import ctypes

        T = res.shape[0]
        rc = self._lib.ssb_mhc(ctypes.byref(self._c), None if x is None else x.data_ptr(), res.data_ptr(),
                               None if post_in is None else post_in.data_ptr(),
                               None if comb_in is None else comb_in.data_ptr(),
                               None if new_res is None else new_res.data_ptr(), post_out.data_ptr(),
                               comb_out.data_ptr(), y.data_ptr(), T, lib.stream_ptr(stream))
        lib.check("ssb_mhc", rc)


class KdaDecoderLayer:
    """One Glm5Next KDA + MoE decoder layer on the 4-stream residual: boundary A (post of the previous sub-block,
    pre of attention) -> KDA attention -> boundary B (post of attention, pre of the FFN) -> NVFP4 MoE (routed top-k +
    shared expert). The layer's output sub-block (the MoE rows, with their post / comb mixes) is folded into the
    residual by the next boundary."""

    def __init__(self, seed: int, hidden: int, heads: int, inter: int, experts: int, top_k: int, device):
        from . import moe

        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.H = hidden
        self.bound_a = MhcBoundary(g, hidden, dev)
        self.attn = KdaAttention(seed + 1, hidden, heads, dev)
        self.bound_b = MhcBoundary(g, hidden, dev)
        self.moe = moe.MoELayer.from_logical(weights.moe_logical(seed + 2, hidden, inter, experts, device=dev), top_k,
                                             dev)
        self.device = dev

    def forward(self, res, x_prev, post_prev, comb_prev, seqs, conv_state, rec_state, status, stream=None):
        """res bf16 [T, 4, H]; x_prev bf16 [T, H] with post_prev fp32 [T, 4] / comb_prev [T, 4, 4] (x_prev None: the
        first layer of the stage, pre only). Returns (res after attention, MoE rows, post, comb) for the next
        boundary."""
        T, H, dev = res.shape[0], self.H, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        res_a = torch.empty_like(res) if x_prev is not None else res
        post_a, comb_a = torch.empty(T, 4, **f32), torch.empty(T, 4, 4, **f32)
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        self.bound_a(x_prev, res, post_prev, comb_prev, res_a if x_prev is not None else None, post_a, comb_a, y,
                     stream)
        x_a = self.attn.forward(y, seqs, conv_state, rec_state, status, stream=stream)
        res_b = torch.empty_like(res)
        post_b, comb_b = torch.empty(T, 4, **f32), torch.empty(T, 4, 4, **f32)
        self.bound_b(x_a, res_a, post_a, comb_a, res_b, post_b, comb_b, y, stream)
        x_b = self.moe.forward(y, stream=stream)
        return res_b, x_b, post_b, comb_b
