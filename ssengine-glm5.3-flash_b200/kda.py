"""KDA prefill of one layer through the C ABI: the host side of `ssb_kda_prefill` / `ssb_kda_conv`.

Mirrors the reference's interface for this path: `kda_prefill_forward(self, qkv_proj_states, g1, beta,
core_attn_out)` (ssengine/model/pp_patch.py:215-244) with the layer's conv weight, `A_log`, `dt_bias` and lower bound
(`route_kda`, :247-256), the per-microbatch sequence table (first row, end row, state block, has initial state) of
`KdaPrefillMeta` (:189-197), and the layer's state pages (conv state [blocks, 3, 3P] bf16, recurrent state [blocks, H,
128, 128] fp32; pp_patch.py:223). `conv_qkv` mirrors `kda_conv.conv_qkv` (ssengine/model/kda_conv.py:146-164).
There is no fallback: without the CUDA library these calls raise.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import lib

HEAD_DIM = 128

def workspace_bytes(heads: int, T: int, R: int) -> int:
    """Device bytes of the chunk workspace of one prefill call (`ssb_kda_workspace_bytes`)."""
    n = lib.load().ssb_kda_workspace_bytes(heads, T, R)
    if n < 0:
        raise ValueError(f"bad KDA workspace query: heads={heads}, T={T}, R={R}")
    return int(n)




def seq_table(seqs, device) -> torch.Tensor:
    """[(first row, end row, state block, has initial state)] -> int32 [R, 4] on `device` (the reference's
    `KdaPrefillMeta.seqs`, kda_conv.tables' per-sequence rows)."""
    rows = [(int(s), int(e), int(b), int(bool(i))) for s, e, b, i in seqs]
    t = torch.tensor(rows, dtype=torch.int32).reshape(-1, 4)
    return t.to(device)


@dataclass
class KdaLayer:
    """One KDA layer's parameters on the device."""
    conv_weight: torch.Tensor     # bf16 [3 * H * 128, 4]
    a_log: torch.Tensor           # fp32 [H]
    dt_bias: torch.Tensor         # fp32 [H * 128]
    lower_bound: float = -5.0

    @property
    def heads(self) -> int:
        return self.a_log.numel()

    def c_struct(self, conv_state: torch.Tensor, rec_state: torch.Tensor) -> lib.KdaLayerC:
        H = self.heads
        assert self.conv_weight.dtype == torch.bfloat16 and self.conv_weight.shape == (3 * H * HEAD_DIM, 4)
        assert self.conv_weight.is_contiguous() and self.a_log.dtype == torch.float32
        assert self.dt_bias.dtype == torch.float32 and self.dt_bias.numel() == H * HEAD_DIM
        assert conv_state.dtype == torch.bfloat16 and conv_state.shape[1:] == (3, 3 * H * HEAD_DIM)
        assert conv_state[0].is_contiguous()
        assert rec_state.dtype == torch.float32 and rec_state.shape[1:] == (H, HEAD_DIM, HEAD_DIM)
        assert rec_state[0].is_contiguous()
        return lib.KdaLayerC(H, HEAD_DIM, self.conv_weight.data_ptr(), self.a_log.data_ptr(), self.dt_bias.data_ptr(),
                             self.lower_bound, HEAD_DIM ** -0.5, conv_state.data_ptr(), conv_state.stride(0),
                             rec_state.data_ptr(), rec_state.stride(0))

    def prefill(self, qkv: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, out: torch.Tensor, seqs: torch.Tensor,
                conv_state: torch.Tensor, rec_state: torch.Tensor, stream=None, status: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> None:
        """qkv bf16 [T, >= 3P] (q | k | v first), g bf16 [T, >= P] raw gate, beta bf16 [T, >= H] raw; writes out bf16
        [T, >= P] for the rows of `seqs` (int32 [R, 4] on the device) and updates both state pages in place. `status`
        (int32 [1] on the device) receives 4 if a bounded copy wait gave up. `workspace`: uint8 device tensor of at
        least `workspace_bytes(heads, T, R)` (default: the device's shared scratch)."""
        so = lib.load()
        T = qkv.shape[0]
        for t in (qkv, g, beta, out):
            assert t.dtype == torch.bfloat16 and t.stride(1) == 1 and t.shape[0] >= T
        assert seqs.dtype == torch.int32 and seqs.is_contiguous()
        need = workspace_bytes(self.heads, T, seqs.shape[0])
        if workspace is None:
            workspace = lib.scratch(qkv.device, need)
        assert workspace.dtype == torch.uint8 and workspace.is_contiguous() and workspace.numel() >= need
        L = self.c_struct(conv_state, rec_state)
        rc = so.ssb_kda_prefill_ws(ctypes.byref(L), qkv.data_ptr(), qkv.stride(0), g.data_ptr(), g.stride(0),
                                   beta.data_ptr(), beta.stride(0), T, seqs.data_ptr(), seqs.shape[0], out.data_ptr(),
                                   out.stride(0), workspace.data_ptr(), workspace.numel(),
                                   None if status is None else status.data_ptr(), lib.stream_ptr(stream))
        lib.check("ssb_kda_prefill_ws", rc)

    def conv_qkv(self, qkv: torch.Tensor, seqs: torch.Tensor, conv_state: torch.Tensor, rec_state: torch.Tensor,
                 stream=None):
        """The short conv alone -> q, k, v bf16 [T, P] each; the conv state blocks of `seqs` updated."""
        so = lib.load()
        T, P = qkv.shape[0], self.heads * HEAD_DIM
        out = torch.empty(3, T, P, dtype=torch.bfloat16, device=qkv.device)
        L = self.c_struct(conv_state, rec_state)
        rc = so.ssb_kda_conv(ctypes.byref(L), qkv.data_ptr(), qkv.stride(0), T, seqs.data_ptr(), seqs.shape[0],
                             out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), lib.stream_ptr(stream))
        lib.check("ssb_kda_conv", rc)
        return out[0], out[1], out[2]
