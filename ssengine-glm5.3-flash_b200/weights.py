"""Seeded random-init NVFP4 parameters (there is no checkpoint in this setting; the CUDA path and the CPU checker are
fed from the same generator so that parity is checked on identical quantized weights).

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


E2M1_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """A real-valued weight [N, K] -> NVFP4 (codes [N, K] one per byte, e4m3 scales [N, K / 16], global scale gs) with
    gs = 448 * 6 / max|w| (the largest block scale at the top of the e4m3 range), sf = e4m3((amax16 / 6) * gs) and
    each code the nearest e2m1 magnitude of |w| * gs / sf (midpoints to the smaller one) with w's sign. Weights are
    data: the checker reads these codes back, so the rounding rule only needs to be deterministic."""
    N, K = w.shape
    w = w.float()
    gs = float(448.0 * 6.0 / max(float(w.abs().max()), 1e-30))
    blocks = w.view(N, K // 16, 16)
    sf = (blocks.abs().amax(-1) / 6.0 * gs).to(torch.float8_e4m3fn)
    sfv = sf.float()
    r = torch.where(sfv > 0, gs / sfv.clamp_min(1e-30), torch.zeros_like(sfv))
    mag = blocks.abs() * r[..., None]
    idx = torch.bucketize(mag, torch.tensor(E2M1_MIDPOINTS, device=w.device))
    codes = (idx + 8 * (blocks < 0).to(idx.dtype)).to(torch.uint8).view(N, K)
    return codes, sf.view(torch.uint8), gs


def nvfp4_tensor(gen, N: int, K: int, device, init: str = "uniform", in_sq_mean: float = 1.0, std: float = 0.02,
                 factor: float = 1.0):
    """(codes [N, K], sf [N, K / 16], gs) of one random-init NVFP4 weight. init "uniform": BASELINE's recipe (codes
    uniform over the 16 e2m1 codes, scales log-uniform over the e4m3 codes in [2^-8, 1], gs for unit-variance outputs
    on inputs of mean square `in_sq_mean`, divided by `factor`); "normal": BASELINE config 1's recipe (N(0, std)
    values quantized by `quantize_weight`)."""
    if init == "uniform":
        return _codes(gen, (N, K), device), _scales(gen, (N, K // 16), device), unit_gs(K, in_sq_mean) * factor
    if init == "normal":
        return quantize_weight(torch.randn(N, K, generator=gen, device=device) * std)
    raise ValueError(f"init {init!r}")


def _codes(gen, shape, device):
    return torch.randint(0, 16, shape, generator=gen, device=device, dtype=torch.uint8)


def _scales(gen, shape, device):
    table = torch.tensor(SCALE_CODES, dtype=torch.uint8, device=device)
    return table[torch.randint(0, len(SCALE_CODES), shape, generator=gen, device=device)]


# the reference model's routing (ssengine/kernels.py:182-187): sigmoid scores + a per-expert correction bias, top-8,
# routed scaling factor 5/2; the bias is drawn like the reference's routing test draws it (12.4 + U[0, 0.52),
# tests/test_moe_tuning_cpu.py:62: "the checkpoint's widest spread is 0.58")
SIGMOID_ROUTE = dict(n_group=1, topk_group=1, scale=2.5, bias_base=12.4, bias_spread=0.52)


def moe_logical(seed: int, H: int, F: int, E: int, device="cpu", routing: str = "softmax",
                n_group: int = 1, topk_group: int = 1, init: str = "uniform", std: float = 0.02) -> dict:
    """Logical parameters of one MoE layer: E routed experts + the shared expert (index E). routing "softmax"
    or "sigmoid" (the reference model's rule; adds p["route"]); init: see `nvfp4_tensor`."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    router = nvfp4_tensor(gen, E, H, device, init, std=std)
    experts = []
    for e in range(E + 1):
        f = 1.0 + 0.25 * (e % 3)
        w1 = nvfp4_tensor(gen, 2 * F, H, device, init, std=std, factor=f)
        w2 = nvfp4_tensor(gen, H, F, device, init, SILU_U_SQ_MEAN, std=std, factor=f)
        experts.append(w1 + w2)
    p = {"H": H, "F": F, "E": E, "gs_x": GS_X, "gs_h": GS_H, "router": router, "experts": experts}
    if routing == "sigmoid":
        r = SIGMOID_ROUTE
        bias = r["bias_base"] + torch.rand(E, generator=gen, device=device) * r["bias_spread"]
        p["route"] = {"bias": bias.float(), "n_group": n_group, "topk_group": topk_group, "scale": r["scale"]}
    elif routing != "softmax":
        raise ValueError(f"routing {routing!r}")
    return p


def hidden_states(seed: int, T: int, H: int, device="cpu") -> torch.Tensor:
    """BASELINE config 2's input: bf16 hidden states N(0, 1)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return torch.randn(T, H, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def to_numpy(p: dict) -> dict:
    """The same parameters as numpy arrays (the checker's input)."""
    def n(t):
        return t.cpu().numpy() if isinstance(t, torch.Tensor) else t

    out = {**p, "router": tuple(n(v) for v in p["router"]), "experts": [tuple(n(v) for v in e) for e in p["experts"]]}
    if "route" in p:
        out["route"] = {k: n(v) for k, v in p["route"].items()}
    return out
