"""Seeded random-init NVFP4 parameters (there is no checkpoint in this setting; the CUDA path and the CPU checker are
fed from the same generator so that parity is judged on identical quantized weights).

MoE layer: e2m1 codes uniform over the 16 codes; e4m3 block scales uniform over the e4m3 codes
whose value lies in [2^-8, 2^0] (55 codes: evenly spaced in log2 within each binade, a log-uniform draw on the
e4m3 grid); one fp32 global scale per tensor, chosen so that router logits, gate and up pre-activations and expert
outputs have unit variance for unit-variance inputs, times a per-expert factor 1, 1.25 or 1.5 (so every expert has
its own output scale). Activation global scales are static, as a calibrated checkpoint's: gs_x = 448 * 6 / 8 (inputs
of unit variance) and gs_h = 448 * 6 / 32 (SwiGLU outputs).

The logical layout here is the checker's: codes one per byte [rows, K], scales [rows, K / 16], gate rows [0, F) then
up rows [F, 2F); `ssengine_b200.moe.MoELayer` converts it to the device layouts of include/ssengine_b200.h.
"""

from __future__ import annotations

import math

import torch

E2M1_MAG = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_SQ_MEAN = sum(v * v for v in E2M1_MAG) / len(E2M1_MAG)     # codes uniform over 16 (+-)


def e4m3_value(code: int) -> float:
    e, m = (code >> 3) & 0xF, code & 7
    return m * 2.0 ** -9 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)


SCALE_CODES = tuple(c for c in range(0x7F) if 2.0 ** -8 <= e4m3_value(c) <= 1.0)
SCALE_SQ_MEAN = sum(e4m3_value(c) ** 2 for c in SCALE_CODES) / len(SCALE_CODES)
SILU_U_SQ_MEAN = 0.3557          # E[(silu(g) u)^2] for independent g, u ~ N(0, 1)

GS_X = 448.0 * 6.0 / 8.0
GS_H = 448.0 * 6.0 / 32.0


def unit_gs(K: int, in_sq_mean: float = 1.0) -> float:
    """Global scale that gives a K-long dot product of random codes/scales with inputs of mean square
    `in_sq_mean` unit variance."""
    return math.sqrt(K * in_sq_mean * E2M1_SQ_MEAN * SCALE_SQ_MEAN)


def _codes(gen, shape, device):
    return torch.randint(0, 16, shape, generator=gen, device=device, dtype=torch.uint8)


def _scales(gen, shape, device):
    table = torch.tensor(SCALE_CODES, dtype=torch.uint8, device=device)
    return table[torch.randint(0, len(SCALE_CODES), shape, generator=gen, device=device)]


def moe_logical(seed: int, H: int, F: int, E: int, device="cpu") -> dict:
    """Logical parameters of one MoE layer: E routed experts + the shared expert (index E)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    g_r = unit_gs(H)
    router = (_codes(gen, (E, H), device), _scales(gen, (E, H // 16), device), g_r)
    experts = []
    for e in range(E + 1):
        f = 1.0 + 0.25 * (e % 3)
        w1 = (_codes(gen, (2 * F, H), device), _scales(gen, (2 * F, H // 16), device), unit_gs(H) * f)
        w2 = (_codes(gen, (H, F), device), _scales(gen, (H, F // 16), device), unit_gs(F, SILU_U_SQ_MEAN) * f)
        experts.append(w1 + w2)
    return {"H": H, "F": F, "E": E, "gs_x": GS_X, "gs_h": GS_H, "router": router, "experts": experts}


def hidden_states(seed: int, T: int, H: int, device="cpu") -> torch.Tensor:
    """BASELINE config 2's input: bf16 hidden states N(0, 1)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return torch.randn(T, H, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def to_numpy(p: dict) -> dict:
    """The same parameters as numpy arrays (the checker's input)."""
    def n(t):
        return t.cpu().numpy() if isinstance(t, torch.Tensor) else t

    return {**p, "router": tuple(n(v) for v in p["router"]), "experts": [tuple(n(v) for v in e) for e in p["experts"]]}
