"""One NVFP4 MoE layer on the CUDA library (the host mirror of the reference's MoE block).

Replaces, per MoE layer of a reference stage, the router GEMM + input quant + FlashInfer `trtllm_fp4_block_scale_moe`
+ shared expert (ssengine/kernels.py:174-193, configs 28-32) with one call of `ssb_moe_forward`. The caller owns every
buffer: the layer keeps its device weights, a workspace grown on demand and an int32 device status word.
"""

from __future__ import annotations

import ctypes

import torch

from . import layout, lib


class MoELayer:
    def __init__(self, H: int, F: int, E: int, k: int, gs_x: float, gs_h: float, router: tuple, w1: tuple,
                 w2: tuple, device, add_input: bool = False, route: dict | None = None):
        """route: None for softmax top-k routing, else the sigmoid + correction-bias rule
        {"bias": fp32 [E] device tensor, "n_group", "topk_group", "scale"} (the reference model's)."""
        self.H, self.F, self.E, self.k = H, F, E, k
        self.gs_x, self.gs_h = float(gs_x), float(gs_h)
        self.device = torch.device(device)
        self.router_codes, self.router_sf, self.router_alpha, self.router_rows = router
        self.w1_codes, self.w1_sf, self.w1_alpha = w1
        self.w2_codes, self.w2_sf, self.w2_alpha = w2
        self._lib = lib.load()
        self._c = lib.MoeLayerC(H, F, E, k, self.gs_x, self.gs_h, self.router_codes.data_ptr(),
                                self.router_sf.data_ptr(), self.router_rows, self.router_alpha,
                                self.w1_codes.data_ptr(), self.w1_sf.data_ptr(), self.w1_alpha.data_ptr(),
                                self.w2_codes.data_ptr(), self.w2_sf.data_ptr(), self.w2_alpha.data_ptr(),
                                1 if add_input else 0)
        self.route = route
        if route is not None:
            self.route_bias = route["bias"].to(self.device, torch.float32).contiguous()
            self._c.routing = lib.ROUTE_SIGMOID_BIAS
            self._c.n_group, self._c.topk_group = int(route["n_group"]), int(route["topk_group"])
            self._c.routed_scale = float(route["scale"])
            self._c.route_bias = self.route_bias.data_ptr()
        self.add_input = add_input
        self._ws = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_logical(cls, p: dict, k: int, device, add_input: bool = False) -> "MoELayer":
        """From `weights.moe_logical` parameters (torch tensors on any device); `add_input`: out = x + MoE(x)."""
        dev = torch.device(device)
        H, F, E = p["H"], p["F"], p["E"]
        rc, rs, rg = (t.to(dev) if isinstance(t, torch.Tensor) else t for t in p["router"])
        rows = -(-E // 128) * 128
        rc_pad = torch.zeros(rows, H, dtype=torch.uint8, device=dev)
        rc_pad[:E] = rc
        rs_pad = torch.zeros(rows, H // 16, dtype=torch.uint8, device=dev)
        rs_pad[:E] = rs
        router = (layout.pack_codes(rc_pad).contiguous(), layout.sf_to_atoms(rs_pad, H), float(1.0 / (p["gs_x"] * rg)),
                  rows)
        w1c, w1s, w2c, w2s, a1, a2 = [], [], [], [], [], []
        for (c1, s1, g1, c2, s2, g2) in p["experts"]:
            c1, s1, c2, s2 = (t.to(dev) for t in (c1, s1, c2, s2))
            w1c.append(layout.pack_codes(layout.gate_up_interleave(c1)))
            w1s.append(layout.sf_to_atoms(layout.gate_up_interleave(s1), H))
            w2c.append(layout.pack_codes(c2))
            w2s.append(layout.sf_to_atoms(s2, F))
            a1.append(1.0 / (p["gs_x"] * g1))
            a2.append(1.0 / (p["gs_h"] * g2))
        w1 = (torch.cat(w1c).contiguous(), torch.cat(w1s).contiguous(),
              torch.tensor(a1, dtype=torch.float32, device=dev))
        w2 = (torch.cat(w2c).contiguous(), torch.cat(w2s).contiguous(),
              torch.tensor(a2, dtype=torch.float32, device=dev))
        route = None
        if p.get("route") is not None:
            r = p["route"]
            bias = r["bias"] if isinstance(r["bias"], torch.Tensor) else torch.as_tensor(r["bias"])
            route = {**r, "bias": bias.to(dev, torch.float32)}
        return cls(H, F, E, k, p["gs_x"], p["gs_h"], router, w1, w2, dev, add_input, route)

    # ---------------------------------------------------------------- forward
    def workspace_bytes(self, T: int) -> int:
        n = self._lib.ssb_moe_workspace_bytes(ctypes.byref(self._c), T)
        if n < 0:
            raise lib.SsbError("ssb_moe_workspace_bytes", 1)
        return int(n)

    def workspace(self, T: int) -> torch.Tensor:
        n = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """x bf16 [T, H] on the layer's device -> bf16 [T, H]. Enqueues work only (no host sync)."""
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[1] == self.H and x.device == self.device
        T = x.shape[0]
        ws = self.workspace(T)
        if out is None:
            out = torch.empty_like(x)
        rc = self._lib.ssb_moe_forward(ctypes.byref(self._c), x.data_ptr(), T, out.data_ptr(), ws.data_ptr(),
                                       ws.numel(), self.status.data_ptr(), lib.stream_ptr(stream))
        lib.check("ssb_moe_forward", rc)
        return out

    __call__ = forward

    def forward_profiled(self, x: torch.Tensor, out: torch.Tensor, events: list, stream=None) -> torch.Tensor:
        """`forward` with `events` (len(lib.MOE_STEPS) + 1 torch.cuda.Event, each recorded once before) recorded on
        the stream around each launch step, for per-kernel device timing."""
        T = x.shape[0]
        ws = self.workspace(T)
        arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        rc = self._lib.ssb_moe_forward_profiled(ctypes.byref(self._c), x.data_ptr(), T, out.data_ptr(),
                                                ws.data_ptr(), ws.numel(), self.status.data_ptr(),
                                                lib.stream_ptr(stream), arr)
        lib.check("ssb_moe_forward_profiled", rc)
        return out

    def check_status(self) -> None:
        """Synchronize and raise if a kernel reported a device-side error (then clear the word)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            raise lib.SsbError("device status", code)

    def ws_offsets(self, T: int) -> list[int]:
        arr = (ctypes.c_int64 * (lib.WS["END"] + 1))()
        lib.check("ssb_moe_workspace_offsets",
                  self._lib.ssb_moe_workspace_offsets(ctypes.byref(self._c), T, arr, lib.WS["END"] + 1))
        return list(arr)

    def ws_view(self, name: str, T: int, dtype: torch.dtype, shape: tuple) -> torch.Tensor:
        """A typed view of one workspace buffer of the last forward over T tokens (tests, debugging)."""
        off = self.ws_offsets(T)
        i = lib.WS[name]
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        assert off[i] + nbytes <= off[i + 1]
        return self._ws[off[i]: off[i] + nbytes].view(dtype).view(shape)

    def logical(self) -> dict:
        """The layer's parameters in the checker's logical layout (numpy; device -> host copies)."""
        import numpy as np

        H, F, E = self.H, self.F, self.E
        rc = layout.unpack_codes(self.router_codes)[:E].cpu().numpy()
        rs = layout.atoms_to_sf(self.router_sf, self.router_rows, H)[:E].cpu().numpy()
        experts = []
        s1 = self.w1_sf.numel() // (E + 1)
        s2 = self.w2_sf.numel() // (E + 1)
        a1 = self.w1_alpha.cpu().numpy().astype(np.float64)
        a2 = self.w2_alpha.cpu().numpy().astype(np.float64)
        c1_all = self.w1_codes.view(E + 1, 2 * F, H // 2)
        c2_all = self.w2_codes.view(E + 1, H, F // 2)
        for e in range(E + 1):
            c1 = layout.gate_up_deinterleave(layout.unpack_codes(c1_all[e]))
            sc1 = layout.gate_up_deinterleave(layout.atoms_to_sf(self.w1_sf[e * s1:(e + 1) * s1], 2 * F, H))
            c2 = layout.unpack_codes(c2_all[e])
            sc2 = layout.atoms_to_sf(self.w2_sf[e * s2:(e + 1) * s2], H, F)
            experts.append((c1.cpu().numpy(), sc1.cpu().numpy(), float(1.0 / (a1[e] * self.gs_x)), c2.cpu().numpy(),
                            sc2.cpu().numpy(), float(1.0 / (a2[e] * self.gs_h))))
        out = {"H": H, "F": F, "E": E, "gs_x": self.gs_x, "gs_h": self.gs_h,
               "router": (rc, rs, float(1.0 / (self.router_alpha * self.gs_x))), "experts": experts}
        if self.route is not None:
            out["route"] = {"bias": self.route_bias.cpu().numpy(), "n_group": self.route["n_group"],
                            "topk_group": self.route["topk_group"], "scale": self.route["scale"]}
        return out
