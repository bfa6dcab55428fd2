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
    def random(cls, gen: torch.Generator, N: int, K: int, device, gs_in: float = weights.GS_X, in_sq_mean: float = 1.0,
               init: str = "uniform", std: float = 0.02):
        """Random-init NVFP4 weights: BASELINE's recipe scaled for unit-variance outputs ("uniform"), or N(0, std)
        values quantized ("normal")."""
        codes, sf, gs = weights.nvfp4_tensor(gen, N, K, device, init, in_sq_mean, std)
        return cls(codes, sf, gs, device, gs_in)

    def logical(self):
        """(codes [N, K], sf [N, K / 16], gs_w) as stored (for the checker)."""
        codes = layout.unpack_codes(self.codes)[:self.N]
        sf = layout.atoms_to_sf(self.sf, self.N_pad, self.K)[:self.N]
        return codes, sf, 1.0 / (self.alpha * self.gs_in)

    def input_buffers(self, T: int) -> tuple:
        """Empty NVFP4 input buffers for T rows: codes uint8 [T padded to 128, K / 2], zeroed scale atoms."""
        rows = _round(max(T, 1), 128)
        codes = torch.empty(rows, self.K // 2, dtype=torch.uint8, device=self.device)
        sf = torch.zeros(rows // 128 * layout.sf_atom_cols(self.K) * 512, dtype=torch.uint8, device=self.device)
        return codes, sf

    def gemm(self, codes: torch.Tensor, sf: torch.Tensor, T: int, out: torch.Tensor, status: torch.Tensor,
             stream=None) -> torch.Tensor:
        """out bf16 [T, >= N_pad] from an input already quantized with `gs_in` (codes and scale atoms as
        `input_buffers` lays them out)."""
        lib.check("ssb_nvfp4_gemm", self._lib.ssb_nvfp4_gemm(lib.EPI_BF16, codes.data_ptr(), sf.data_ptr(), T, self.K,
                                                             self.codes.data_ptr(), self.sf.data_ptr(), self.N_pad,
                                                             self.alpha, out.data_ptr(), out.stride(0), None, 1.0,
                                                             status.data_ptr(), lib.stream_ptr(stream)))
        return out

    def quantize(self, x: torch.Tensor, stream=None) -> tuple:
        """x bf16 [T, >= K] -> (codes, scale atoms) of its NVFP4 form with `gs_in`, reusable by every projection of
        the same K and global scale."""
        T = x.shape[0]
        codes, sf = self.input_buffers(T)
        lib.check("ssb_nvfp4_quantize", self._lib.ssb_nvfp4_quantize(x.data_ptr(), T, self.K, x.stride(0), self.gs_in,
                                                                     codes.data_ptr(), self.K // 2, sf.data_ptr(),
                                                                     lib.stream_ptr(stream)))
        return codes, sf

    def __call__(self, x: torch.Tensor, out: torch.Tensor, status: torch.Tensor, stream=None) -> torch.Tensor:
        """x bf16 [T, >= K] (row pitch x.stride(0)), out bf16 [T, >= N_pad] (row pitch out.stride(0))."""
        codes, sf = self.quantize(x, stream)
        return self.gemm(codes, sf, x.shape[0], out, status, stream)


class DenseFfn:
    """The dense SwiGLU FFN of the reference model's leading layers (`first_kda_dense`, `kda_dense`: layers 0-2,
    ssengine/kernels.py:283-289): gate_up k H n 2F and down k F n H, NVFP4 with the activation quantized on the way
    in (configs 8-11: `scaled_fp4_quant` -> `mm_fp4` gate_up -> `scaled_fp4_quant` -> `mm_fp4` down, 4096 -> 24576 ->
    4096 in the reference). Here: input quant -> gate_up GEMM whose epilogue applies SwiGLU and writes the down GEMM's
    NVFP4 input (codes + scale atoms, global scale GS_H) -> down GEMM with a bf16 epilogue: three launches."""

    def __init__(self, seed: int, hidden: int, inter: int, device, init: str = "uniform", std: float = 0.02):
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, F = hidden, inter
        if F % 128 != 0 or H % 256 != 0:
            raise ValueError(f"dense FFN dims H={H} (% 256), F={F} (% 128)")
        self.H, self.F = H, F
        c1, s1, self.gs_w1 = weights.nvfp4_tensor(g, 2 * F, H, dev, init, std=std)
        c2, s2, self.gs_w2 = weights.nvfp4_tensor(g, H, F, dev, init, weights.SILU_U_SQ_MEAN, std=std)
        self.w1_codes = layout.pack_codes(layout.gate_up_interleave(c1)).contiguous()
        self.w1_sf = layout.sf_to_atoms(layout.gate_up_interleave(s1), H)
        self.w2 = Nvfp4Linear(c2, s2, self.gs_w2, dev, gs_in=weights.GS_H)
        self.alpha1 = float(1.0 / (weights.GS_X * self.gs_w1))
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.device = dev
        self._lib = lib.load()

    def logical(self):
        """(w1 codes [2F, H] gate rows then up rows, w1 sf, gs_w1, w2 codes [H, F], w2 sf, gs_w2) for the checker."""
        c1 = layout.gate_up_deinterleave(layout.unpack_codes(self.w1_codes))
        s1 = layout.gate_up_deinterleave(layout.atoms_to_sf(self.w1_sf, 2 * self.F, self.H))
        c2, s2, g2 = self.w2.logical()
        return c1, s1, self.gs_w1, c2, s2, g2

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """x bf16 [T, H] -> bf16 [T, H]."""
        T, H, F, dev = x.shape[0], self.H, self.F, self.device
        s = lib.stream_ptr(stream)
        rows = _round(max(T, 1), 128)
        xc = torch.empty(rows, H // 2, dtype=torch.uint8, device=dev)
        xs = torch.zeros(rows // 128 * layout.sf_atom_cols(H) * 512, dtype=torch.uint8, device=dev)
        lib.check("ssb_nvfp4_quantize", self._lib.ssb_nvfp4_quantize(x.data_ptr(), T, H, x.stride(0), weights.GS_X,
                                                                     xc.data_ptr(), H // 2, xs.data_ptr(), s))
        hc, hs = self.w2.input_buffers(T)
        lib.check("ssb_nvfp4_gemm", self._lib.ssb_nvfp4_gemm(lib.EPI_SWIGLU, xc.data_ptr(), xs.data_ptr(), T, H,
                                                             self.w1_codes.data_ptr(), self.w1_sf.data_ptr(), 2 * F,
                                                             self.alpha1, hc.data_ptr(), F // 2, hs.data_ptr(),
                                                             weights.GS_H, self.status.data_ptr(), s))
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        return self.w2.gemm(hc, hs, T, out, self.status, stream)

    __call__ = forward


class KdaAttention:
    """The KDA attention block of one layer: hidden H, `heads` heads of 128 (P = heads * 128)."""

    def __init__(self, seed: int, hidden: int, heads: int, device, lower_bound: float = -5.0, norm_eps: float = 1e-5,
                 init: str = "uniform", std: float = 0.02):
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, P = hidden, heads * HEAD_DIM
        self.H, self.heads, self.P = H, heads, P
        self.in_cols = 3 * P + 2 * LOW_RANK + heads
        w = dict(init=init, std=std)
        self.in_proj = Nvfp4Linear.random(g, self.in_cols, H, dev, **w)
        self.f_b = Nvfp4Linear.random(g, P, LOW_RANK, dev, **w)
        self.g_b = Nvfp4Linear.random(g, P, LOW_RANK, dev, **w)
        self.o_proj = Nvfp4Linear.random(g, H, P, dev, **w)
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
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=dev)
        if keep:
            # the bf16 normed rows are kept for checks, then quantized as the o_proj's input
            lib.check("ssb_gated_rmsnorm", self._lib.ssb_gated_rmsnorm(o.data_ptr(), P, ogate.data_ptr(), P,
                                                                       self.norm_w.data_ptr(), self.norm_eps,
                                                                       o.data_ptr(), P, T, self.heads, s))
            self.o_proj(o, out, status, stream)
            self.parts["normed"] = o
        else:
            # the norm writes the o_proj's NVFP4 input directly (same bytes as norm + quantize)
            codes, sf = self.o_proj.input_buffers(T)
            lib.check("ssb_gated_rmsnorm_nvfp4",
                      self._lib.ssb_gated_rmsnorm_nvfp4(o.data_ptr(), P, ogate.data_ptr(), P, self.norm_w.data_ptr(),
                                                        self.norm_eps, self.o_proj.gs_in, codes.data_ptr(), P // 2,
                                                        sf.data_ptr(), T, self.heads, s))
            self.o_proj.gemm(codes, sf, T, out, status, stream)
        return out


class MhcBoundary:
    """One mHC layer boundary (4 streams): the previous sub-block's post and the next sub-block's pre + RMSNorm
    (`ssb_mhc_ws`: the reference's `MegaMhcPostPre`, ssengine/model/pp_patch.py:125-153)."""

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

    def __call__(self, x, res, post_in, comb_in, new_res, post_out, comb_out, y, stream=None, status=None) -> None:
        """x = None: pre only (the stage-edge receive) on res; else post of x into new_res, then pre of new_res.
        `status` (int32 [1] on the device) receives 4 if a bounded wait of the pre step expired."""
        import ctypes

        T = res.shape[0]
        self._c.status = None if status is None else status.data_ptr()
        ws = lib.scratch(res.device, int(self._lib.ssb_mhc_workspace_bytes(T)))
        rc = self._lib.ssb_mhc_ws(ctypes.byref(self._c), None if x is None else x.data_ptr(), res.data_ptr(),
                                  None if post_in is None else post_in.data_ptr(),
                                  None if comb_in is None else comb_in.data_ptr(),
                                  None if new_res is None else new_res.data_ptr(), post_out.data_ptr(),
                                  comb_out.data_ptr(), y.data_ptr(), T, ws.data_ptr(), ws.numel(),
                                  lib.stream_ptr(stream))
        lib.check("ssb_mhc_ws", rc)


class KdaDecoderLayer:
    """One Glm5Next KDA + MoE decoder layer on the 4-stream residual: boundary A (post of the previous sub-block,
    pre of attention) -> KDA attention -> boundary B (post of attention, pre of the FFN) -> NVFP4 MoE (routed top-k +
    shared expert). The layer's output sub-block (the MoE rows, with their post / comb mixes) is folded into the
    residual by the next boundary."""

    def __init__(self, seed: int, hidden: int, heads: int, inter: int, experts: int, top_k: int, device,
                 ffn: str = "moe", routing: dict | None = None, init: str = "uniform", std: float = 0.02):
        """ffn "moe" (F = inter, `experts` routed top-`top_k` + shared; `routing`: moe_logical's routing keywords) or
        "dense" (the reference's leading layers: a dense SwiGLU FFN of intermediate `inter`); init / std: the NVFP4
        weights' recipe (weights.nvfp4_tensor)."""
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.H = hidden
        self.bound_a = MhcBoundary(g, hidden, dev)
        self.attn = KdaAttention(seed + 1, hidden, heads, dev, init=init, std=std)
        self.bound_b = MhcBoundary(g, hidden, dev)
        self.ffn = _make_ffn(seed + 2, hidden, inter, experts, top_k, dev, ffn, routing, init, std)
        self.moe = self.ffn                  # the FFN sub-block (MoELayer or DenseFfn)
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
                     stream, status=status)
        x_a = self.attn.forward(y, seqs, conv_state, rec_state, status, stream=stream)
        res_b = torch.empty_like(res)
        post_b, comb_b = torch.empty(T, 4, **f32), torch.empty(T, 4, 4, **f32)
        self.bound_b(x_a, res_a, post_a, comb_a, res_b, post_b, comb_b, y, stream, status=status)
        x_b = _ffn_forward(self, y, stream)
        return res_b, x_b, post_b, comb_b


def _ffn_forward(layer, y, stream):
    """The decoder layer's FFN; with `layer.moe_profile` a list, a MoE layer runs its per-step profiled form and
    appends its events (len(lib.MOE_STEPS) + 1, recorded around each launch step)."""
    from . import moe

    prof = getattr(layer, "moe_profile", None)
    if prof is None or not isinstance(layer.moe, moe.MoELayer):
        return layer.moe.forward(y, stream=stream)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(lib.MOE_STEPS) + 1)]
    for e in evs:
        e.record()                                      # creates the events the library records into
    out = torch.empty_like(y)
    layer.moe.forward_profiled(y, out, evs, stream=stream)
    prof.append(evs)
    return out


def _make_ffn(seed: int, hidden: int, inter: int, experts: int, top_k: int, device, ffn: str, routing: dict | None,
              init: str = "uniform", std: float = 0.02):
    from . import moe

    if ffn == "dense":
        return DenseFfn(seed, hidden, inter, device, init, std)
    if ffn != "moe":
        raise ValueError(f"ffn {ffn!r}")
    p = weights.moe_logical(seed, hidden, inter, experts, device=device, init=init, std=std, **(routing or {}))
    return moe.MoELayer.from_logical(p, top_k, device)


class Bf16Grouped:
    """Per-head BF16 weights [heads, N, K] for the MLA absorb / v_up batched GEMMs, kept in BF16 as the reference
    keeps them (ssengine/kernels.py configs 22 and 26: torch.bmm over 64 heads); a plain batched library GEMM (cuBLAS
    through torch.bmm) with bf16 output."""

    def __init__(self, gen: torch.Generator, heads: int, N: int, K: int, device, init: str = "uniform",
                 std: float = 0.02):
        dev = torch.device(device)
        w = torch.randn(heads, N, K, generator=gen, device=dev)
        self.w = (w * (std if init == "normal" else K ** -0.5)).to(torch.bfloat16)
        self.wt = self.w.transpose(1, 2)                 # [heads, K, N] view
        self.heads, self.N, self.K = heads, N, K
        self.device = dev

    def logical(self):
        """The bf16 weights [heads, N, K] (for the checker)."""
        return (self.w,)

    def __call__(self, x_heads: torch.Tensor, rows_pad: int, out: torch.Tensor, status=None, stream=None):
        """x_heads bf16 [heads * rows_pad, K] (head-major) -> out bf16 [heads * rows_pad, N]."""
        return self.bmm(x_heads.view(self.heads, rows_pad, self.K), out.view(self.heads, rows_pad, self.N), stream)

    def bmm(self, x: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """x bf16 [heads, rows, K], out bf16 [heads, rows, N], each with unit column stride and any row / head
        strides (e.g. a head's slice of token-major rows, x[h] = rows[:, h, :K]): the batched GEMM reads and writes
        them in place (cuBLAS strided batched, leading dimension = the row stride, batch stride = the head stride),
        so no head transposes run around it."""
        assert x.dtype == torch.bfloat16 and x.stride(2) == 1 and out.stride(2) == 1
        with torch.cuda.stream(stream) if stream is not None else _null():
            torch.bmm(x, self.wt, out=out)
        return out


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


class Nvfp4Grouped:
    """Per-head NVFP4 weights [heads, N, K] for the grouped GEMM (the MLA absorb / v_up bmm)."""

    def __init__(self, gen: torch.Generator, heads: int, N: int, K: int, device, gs_in: float = weights.GS_X,
                 init: str = "uniform", std: float = 0.02):
        dev = torch.device(device)
        codes, sf, self.gs_w = weights.nvfp4_tensor(gen, heads * N, K, dev, init, std=std)
        self.heads, self.N, self.K = heads, N, K
        self.gs_in = gs_in
        self.codes = layout.pack_codes(codes).contiguous()
        self.sf = layout.sf_to_atoms(sf, K)
        self.alpha = torch.full((heads,), 1.0 / (gs_in * self.gs_w), dtype=torch.float32, device=dev)
        self.device = dev
        self._lib = lib.load()
        self._tiles = None                  # int32 [cap, 4] tile table + [1] count, rebuilt on the device per call

    def logical(self):
        codes = layout.unpack_codes(self.codes).view(self.heads, self.N, self.K)
        sf = layout.atoms_to_sf(self.sf, self.heads * self.N, self.K).view(self.heads, self.N, self.K // 16)
        return codes, sf, self.gs_w

    def _tile_table(self, rows_pad: int, stream=None):
        """The grouped GEMM's tile table for `rows_pad` rows a head, written on the device (`ssb_head_tiles`, no host
        copy); the buffer grows only when a larger microbatch arrives."""
        n = self.heads * rows_pad // 128
        if self._tiles is None or self._tiles[0].shape[0] < n:
            self._tiles = (torch.empty(max(n, 1), 4, dtype=torch.int32, device=self.device),
                           torch.empty(1, dtype=torch.int32, device=self.device))
        tiles, num = self._tiles
        lib.check("ssb_head_tiles", self._lib.ssb_head_tiles(self.heads, rows_pad, tiles.data_ptr(), tiles.shape[0],
                                                             num.data_ptr(), lib.stream_ptr(stream)))
        return tiles, num, n

    def __call__(self, x_heads: torch.Tensor, rows_pad: int, out: torch.Tensor, status: torch.Tensor, stream=None):
        """x_heads bf16 [heads * rows_pad, K] (head-major) -> out bf16 [heads * rows_pad, N]."""
        s = lib.stream_ptr(stream)
        rows = self.heads * rows_pad
        codes = torch.empty(rows, self.K // 2, dtype=torch.uint8, device=self.device)
        sf = torch.zeros(rows // 128 * layout.sf_atom_cols(self.K) * 512, dtype=torch.uint8, device=self.device)
        lib.check("ssb_nvfp4_quantize", self._lib.ssb_nvfp4_quantize(x_heads.data_ptr(), rows, self.K, self.K,
                                                                     self.gs_in, codes.data_ptr(), self.K // 2,
                                                                     sf.data_ptr(), s))
        tiles, num, n = self._tile_table(rows_pad, stream)
        lib.check("ssb_nvfp4_gemm_grouped", self._lib.ssb_nvfp4_gemm_grouped(
            lib.EPI_BF16, codes.data_ptr(), sf.data_ptr(), rows, self.K, self.codes.data_ptr(), self.sf.data_ptr(),
            self.N, self.heads, self.alpha.data_ptr(), tiles.data_ptr(), num.data_ptr(), n, out.data_ptr(),
            self.N, status.data_ptr(), s))
        return out


class DsaAttention:
    """The DSA (sparse MLA + lightning indexer) attention block of one layer. Fixed by the kernels: 64 heads, latent
    512 + rope 64, indexer 32 heads x 128 over pools of 4 tokens, top-512 pools (2,051 tokens with the tail).

    y -> a = [q_a | kv latent | k rope] (NVFP4) -> RMSNorm(q_a), RMSNorm(kv) -> q = q_b(q_a) [64 x (nope | rope)],
    rope on the q and k rope slices -> latent cache rows e4m3([kv | k rope] / k_scale) at the rows' slots; q absorb
    (per-head NVFP4 GEMM nope -> 512) -> q8 = e4m3([absorbed | rope] / q_scale) [T, 64, 576]; indexer: q_idx = wq_idx(q_a) [32 x 128], [k_idx | weights | gate] =
    idx_proj(y), pools of 4 into the pool-key cache, logits -> top-512 pools -> tokens; sparse MLA -> [T, 64, 512];
    v_up (per-head NVFP4 GEMM 512 -> v_dim) -> o_proj. The reference's configs 12-27 (ssengine/kernels.py), with every
    projection NVFP4."""

    HEADS, LATENT, ROPE, IDX_HEADS, IDX_DIM, TOPK = 64, 512, 64, 32, 128, 512
    POOLS_PER_PAGE = 32                # pools of 4 tokens in a 128-token KV page

    def __init__(self, seed: int, hidden: int, device, q_lora: int = 1536, nope: int = 192, v_dim: int = 256,
                 theta: float = 10000.0, eps: float = 1e-6, init: str = "uniform", std: float = 0.02,
                 indexer_fp8: bool = False):
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H = hidden
        self.H, self.q_lora, self.nope, self.v_dim, self.theta, self.eps = H, q_lora, nope, v_dim, theta, eps
        # the FP8 indexer: e4m3 queries with per-(token, head) scales, pool keys in the reference's 132-byte entries
        # (the pool cache is then uint8 [pages * 33, 128]); off by default: its kernels are validated one by one, the
        # whole stage on this form not yet
        self.indexer_fp8 = indexer_fp8
        self.qh = nope + self.ROPE
        w = dict(init=init, std=std)
        self.a_proj = Nvfp4Linear.random(g, q_lora + self.LATENT + self.ROPE, H, dev, **w)
        self.q_b = Nvfp4Linear.random(g, self.HEADS * self.qh, q_lora, dev, **w)
        self.w_uk = Bf16Grouped(g, self.HEADS, self.LATENT, nope, dev, **w)
        self.w_uv = Bf16Grouped(g, self.HEADS, v_dim, self.LATENT, dev, **w)
        self.o_proj = Nvfp4Linear.random(g, H, self.HEADS * v_dim, dev, **w)
        self.wq_idx = Nvfp4Linear.random(g, self.IDX_HEADS * self.IDX_DIM, q_lora, dev, **w)
        self.idx_proj = Nvfp4Linear.random(g, self.IDX_DIM + self.IDX_HEADS + self.IDX_DIM, H, dev, **w)
        self.q_norm = (torch.rand(q_lora, generator=g, device=dev) + 0.5).to(torch.bfloat16)
        self.kv_norm = (torch.rand(self.LATENT, generator=g, device=dev) + 0.5).to(torch.bfloat16)
        self.ape = torch.randn(4, self.IDX_DIM, generator=g, device=dev) * 0.5
        self.scale = self.qh ** -0.5
        self.q_scale, self.k_scale = 1.0, 1.0          # per-tensor FP8 scales of the query and the latent cache
        self.logits_ws = None          # optional fp32 buffer the logits rows are cut from (a stage's shared one)
        self._side = None              # the indexer branch's stream (created on first use)
        self.device = dev
        self._lib = lib.load()

    def _side_stream(self) -> torch.cuda.Stream:
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def forward(self, y, positions, slots, qsl, page_table, kpool_reqs, max_rows, groups, kv_cache, pool_cache,
                tail_ring, status, stream=None, keep: bool = False):
        """y bf16 [T, H]; positions / slots int64 [T]; qsl int32 [R + 1]; page_table int32 [R, width] (KV pages);
        kpool_reqs int32 [R, 4] {first row, rows, start position, tail block}; groups: the indexer's work groups
        (int32 [G, 4]); kv_cache e4m3 bytes uint8 [pages * 128, 576], pool_cache bf16 [pages * 32, 128], tail_ring bf16
        [blocks, 2, 4, 128] updated in place -> bf16 [T, H]."""
        from . import indexer, mla

        T, dev, s = y.shape[0], self.device, lib.stream_ptr(stream)
        so, QL, L, RP, NH = self._lib, self.q_lora, self.LATENT, self.ROPE, self.HEADS
        bf = dict(dtype=torch.bfloat16, device=dev)
        a = torch.empty(T, self.a_proj.N_pad, **bf)
        # y feeds a_proj and idx_proj, qa feeds q_b and wq_idx: each quantized once (same K, same static scale)
        assert self.a_proj.gs_in == self.idx_proj.gs_in and self.q_b.gs_in == self.wq_idx.gs_in
        y_q = self.a_proj.quantize(y, stream)
        self.a_proj.gemm(*y_q, T, a, status, stream)
        qa = torch.empty(T, QL, **bf)
        kv_rows = torch.empty(T, L + RP, **bf)
        lib.check("ssb_rmsnorm_cols", so.ssb_rmsnorm_cols(a.data_ptr(), a.stride(0), QL, T, self.q_norm.data_ptr(),
                                                          self.eps, qa.data_ptr(), QL, s))
        kvn = torch.empty(T, L, **bf)
        lib.check("ssb_rmsnorm_cols", so.ssb_rmsnorm_cols(a[:, QL:].data_ptr(), a.stride(0), L, T,
                                                          self.kv_norm.data_ptr(), self.eps, kvn.data_ptr(), L, s))
        k_rope = a[:, QL + L:QL + L + RP]
        lib.check("ssb_rope", so.ssb_rope(k_rope.data_ptr(), a.stride(0), 1, 0, positions.data_ptr(), T, self.theta, s))
        lib.check("ssb_concat_cols", so.ssb_concat_cols(kvn.data_ptr(), L, L, k_rope.data_ptr(), a.stride(0), RP,
                                                        kv_rows.data_ptr(), L + RP, T, s))
        mla.cache_append(kv_rows, slots, kv_cache, self.k_scale, stream)
        # buffers of both branches, allocated on the layer's stream before the fork
        q = torch.empty(T, NH * self.qh, **bf)
        q_lat = torch.empty(NH * T, L, **bf)
        q8 = torch.empty(T, NH, L + RP, dtype=torch.uint8, device=dev)
        q_idx = torch.empty(T, self.IDX_HEADS * self.IDX_DIM, **bf)
        idx = torch.empty(T, self.idx_proj.N_pad, **bf)
        ldl = _round(int(page_table.shape[1]) * self.POOLS_PER_PAGE, 128)
        ws = self.logits_ws
        if ws is not None and ws.numel() >= T * ldl:
            logits = ws[:T * ldl].view(T, ldl)
        else:
            logits = torch.empty(T, ldl, dtype=torch.float32, device=dev)
        ids = torch.empty(T, self.TOPK, dtype=torch.int32, device=dev)
        tok = torch.empty(T, 4 * self.TOPK + 3 + 5, dtype=torch.int32, device=dev)
        if self.indexer_fp8:
            q8_idx = torch.empty(T, self.IDX_HEADS, self.IDX_DIM, dtype=torch.uint8, device=dev)
            qs_idx = torch.empty(T, self.IDX_HEADS, dtype=torch.float32, device=dev)
        qa_q = self.q_b.quantize(qa, stream)
        # the indexer branch (projections, pool insert, logits, top-k, expansion) on a side stream, beside the query
        # branch; the layer's stream waits for it before the sparse MLA, so everything after stays ordered. Nothing
        # on the side stream allocates or runs a torch op: its inputs and outputs are made here, on the layer's
        # stream, and live until the join (the top-k's key ranges included)
        main = stream if stream is not None else torch.cuda.current_stream(dev)
        with torch.cuda.stream(main):
            ranges = indexer.key_ranges(positions)
        side = self._side_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        side.wait_event(fork)
        self.wq_idx.gemm(*qa_q, T, q_idx, status, side)
        self.idx_proj.gemm(*y_q, T, idx, status, side)
        k_idx, gate = idx[:, :self.IDX_DIM], idx[:, self.IDX_DIM + self.IDX_HEADS:2 * self.IDX_DIM + self.IDX_HEADS]
        w = idx[:, self.IDX_DIM:self.IDX_DIM + self.IDX_HEADS]          # bf16 head weights, read in place
        if self.indexer_fp8:
            # the logits' common factor (softmax scale x heads^-1/2 = 2^-6) is left out: a power of two, it changes
            # neither the top-k set nor its ties
            indexer.q_quant(q_idx.view(T, self.IDX_HEADS, self.IDX_DIM), q8_idx, qs_idx, side)
            indexer.kpool_insert_fp8(k_idx, gate, self.ape, kpool_reqs, max_rows, page_table, pool_cache, tail_ring,
                                     side)
            indexer.logits_fp8(q8_idx, qs_idx, w, pool_cache, page_table, groups, logits, status, side)
        else:
            indexer.kpool_insert(k_idx, gate, self.ape, kpool_reqs, max_rows, page_table, pool_cache, tail_ring, side)
            indexer.logits(q_idx.view(T, self.IDX_HEADS, self.IDX_DIM), w, pool_cache, page_table, groups, logits,
                           status, side)
        indexer.topk(logits, positions, self.TOPK, ids, side, ranges=ranges)
        indexer.expand(ids, positions, tok, side)
        join = torch.cuda.Event()
        join.record(side)
        # queries: q_b, rope on each head's rope slice, absorb of each head's nope part into the latent
        self.q_b.gemm(*qa_q, T, q, status, stream)
        lib.check("ssb_rope", so.ssb_rope(q[:, self.nope:].data_ptr(), q.stride(0), NH, self.qh, positions.data_ptr(),
                                          T, self.theta, s))
        # absorb: each head's nope slice read in place from the token-major q rows, head-major latent out
        self.w_uk.bmm(q.view(T, NH, self.qh)[:, :, :self.nope].permute(1, 0, 2), q_lat.view(NH, T, L), stream)
        mla.q_pack(q_lat, T, q[:, self.nope:], self.qh, T, q8, self.q_scale, stream)
        main.wait_event(join)
        # sparse MLA over the selected tokens, then v_up and o_proj
        o_lat = torch.empty(T, NH, L, **bf)
        mla.sparse_mla(q8, kv_cache, tok, qsl, page_table, self.scale * self.q_scale * self.k_scale, o_lat,
                       bmm2=self.k_scale, n_idx=4 * self.TOPK + 3, stream=stream, status=status)
        # v_up: each head's latent rows read in place from the token-major attention output, written straight into
        # the token-major o_proj input
        o_in = torch.empty(T, NH * self.v_dim, **bf)
        v = o_in.view(T, NH, self.v_dim).permute(1, 0, 2)
        self.w_uv.bmm(o_lat.permute(1, 0, 2), v, stream)
        out = torch.empty(T, self.H, **bf)
        self.o_proj(o_in, out, status, stream)
        if keep:
            self.parts = dict(a=a, qa=qa, kvn=kvn, kv_rows=kv_rows, q=q, q_lat=q_lat, q8=q8, q_idx=q_idx,
                              idx=idx, w=w, logits=logits, ids=ids, tok=tok, o_lat=o_lat, v=v, o_in=o_in)
        return out


class DsaDecoderLayer:
    """One Glm5Next DSA + MoE decoder layer on the 4-stream residual: boundary A -> DSA attention -> boundary B ->
    NVFP4 MoE (the same shape as `KdaDecoderLayer` with the sparse-attention block)."""

    def __init__(self, seed: int, hidden: int, inter: int, experts: int, top_k: int, device, q_lora: int = 1536,
                 nope: int = 192, v_dim: int = 256, ffn: str = "moe", routing: dict | None = None,
                 init: str = "uniform", std: float = 0.02, indexer_fp8: bool = False):
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.H = hidden
        self.bound_a = MhcBoundary(g, hidden, dev)
        self.attn = DsaAttention(seed + 1, hidden, dev, q_lora=q_lora, nope=nope, v_dim=v_dim, init=init, std=std,
                                 indexer_fp8=indexer_fp8)
        self.bound_b = MhcBoundary(g, hidden, dev)
        self.ffn = _make_ffn(seed + 2, hidden, inter, experts, top_k, dev, ffn, routing, init, std)
        self.moe = self.ffn                  # the FFN sub-block (MoELayer or DenseFfn)
        self.device = dev

    def forward(self, res, x_prev, post_prev, comb_prev, meta: dict, caches: tuple, status, stream=None):
        """meta: positions, slots, qsl, page_table, kpool_reqs, max_rows, groups (device tensors / ints); caches:
        (latent cache, pool-key cache, tail ring). Returns (res after attention, MoE rows, post, comb)."""
        T, H, dev = res.shape[0], self.H, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        res_a = torch.empty_like(res) if x_prev is not None else res
        post_a, comb_a = torch.empty(T, 4, **f32), torch.empty(T, 4, 4, **f32)
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        self.bound_a(x_prev, res, post_prev, comb_prev, res_a if x_prev is not None else None, post_a, comb_a, y,
                     stream, status=status)
        x_a = self.attn.forward(y, meta["positions"], meta["slots"], meta["qsl"], meta["page_table"],
                                meta["kpool_reqs"], meta["max_rows"], meta["groups"], *caches, status, stream=stream)
        res_b = torch.empty_like(res)
        post_b, comb_b = torch.empty(T, 4, **f32), torch.empty(T, 4, 4, **f32)
        self.bound_b(x_a, res_a, post_a, comb_a, res_b, post_b, comb_b, y, stream, status=status)
        x_b = _ffn_forward(self, y, stream)
        return res_b, x_b, post_b, comb_b
