"""Host-side NVFP4 operand layouts (torch ops; CPU or CUDA tensors), the layouts include/ssengine_b200.h specifies.

- codes: e2m1 codes packed two per byte, the even element in the low nibble, rows K/2 bytes apart;
- scales: e4m3 bytes in the 128x4-atom layout the tcgen05 block-scaled MMA reads (rows padded to 128, K padded to
  256; atom (row block, atom column) = 512 contiguous bytes; scale (r, c) at (r % 32) * 16 + ((r // 32) % 4) * 4 + c % 4);
- expert gate_up weights: rows regrouped in 256-row tiles of 128 gate rows then the 128 matching up rows, so one
  256-wide GEMM tile holds both halves of SwiGLU for 128 output columns.
"""

from __future__ import annotations

import torch

ATOM_ROWS = 128


def sf_atom_cols(K: int) -> int:
    return -(-K // 256) * 4


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """uint8 codes [R, K] (values 0..15) -> [R, K // 2]."""
    c = codes.to(torch.uint8)
    return c[:, 0::2] | (c[:, 1::2] << 4)


def unpack_codes(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.uint8)
    out = torch.empty(p.shape[0], p.shape[1] * 2, dtype=torch.uint8, device=p.device)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = p >> 4
    return out


def sf_to_atoms(sf: torch.Tensor, K: int) -> torch.Tensor:
    """uint8 scales [R, K // 16] -> flat uint8 atoms (zero padding)."""
    R, C = sf.shape
    assert C == K // 16, (C, K)
    nrb, ncb = -(-R // ATOM_ROWS), sf_atom_cols(K)
    pad = torch.zeros(nrb * ATOM_ROWS, ncb * 4, dtype=torch.uint8, device=sf.device)
    pad[:R, :C] = sf
    return pad.view(nrb, 4, 32, ncb, 4).permute(0, 3, 2, 1, 4).contiguous().view(-1)


def atoms_to_sf(flat: torch.Tensor, R: int, K: int) -> torch.Tensor:
    nrb, ncb = -(-R // ATOM_ROWS), sf_atom_cols(K)
    a = flat[: nrb * ncb * 512].view(nrb, ncb, 32, 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return a.view(nrb * ATOM_ROWS, ncb * 4)[:R, : K // 16]


def gate_up_interleave(w: torch.Tensor) -> torch.Tensor:
    """[2F, X] (gate rows, then up rows) -> tiles of 128 gate + 128 up rows; F % 128 == 0."""
    F = w.shape[0] // 2
    assert F % 128 == 0, F
    g = w[:F].reshape(F // 128, 128, *w.shape[1:])
    u = w[F:].reshape(F // 128, 128, *w.shape[1:])
    return torch.stack([g, u], dim=1).reshape(2 * F, *w.shape[1:])


def gate_up_deinterleave(w: torch.Tensor) -> torch.Tensor:
    F = w.shape[0] // 2
    t = w.reshape(F // 128, 2, 128, *w.shape[1:])
    return torch.cat([t[:, 0].reshape(F, *w.shape[1:]), t[:, 1].reshape(F, *w.shape[1:])], dim=0)
