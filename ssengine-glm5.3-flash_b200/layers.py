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
