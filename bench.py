#!/usr/bin/env python
"""Prefill benchmark on B200s: the Glm5Next NVFP4 model as a pipeline of stages, one process per
GPU; or one NVFP4 MoE layer (`--workload moe-layer`).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|vllm-cutlass] [--workload ...]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...      (N > 1)

Pipeline workload (the default; the metric "prefill tok/s, 1 stage + PP2/4/8"): the 45-layer random-init Glm5Next
(hidden 4096; KDA layers with 64 heads of 128; DSA layers 3, 7, ..., 43 with 64 MLA heads, latent 512 + rope 64 in
e4m3, indexer 32 x 128 top-512 pools; layers 0-2 with the dense SwiGLU FFN 4096 -> 2 x 12288 -> 4096; the others 128
experts top-8 + 1 shared, F 1024, with the model's sigmoid + correction-bias routing; vocab 151,552) split into N
pipeline stages -- N = 1: the whole model as one stage; 2: 23/22; 4: 12/11/11/11; 8: 6/6/6/6/6/5/5/5 -- one stage per
GPU, joined by the P2P stage edge (each stage's last kernel stores its [T, 16384] rows into the next GPU's receive
slot; bounded flag waits; no NCCL on the activation path; gloo only for start-up and the timing reductions). The
input stream: 256 cold prompts with lognormal lengths (median 8,192, capped at 131,072), uniform token ids, cut
first-come-first-served into 8,192-token microbatches with KV pages and state blocks from one block pool
(`ssengine_b200.schedule`). A step feeds `--mb-per-step` microbatches (default 4) into the pipeline; K steps (the
same K x 4 microbatches of the stream at every N) are timed after W warm-up steps, the time being each rank's
CUDA-event span from its first timed microbatch to its last, the maximum over ranks, with the pipeline's fill and
drain inside it; `value` = the timed microbatches' tokens / that time (strong scaling: the model and the timed
tokens are fixed, N stages share them). The line also
carries the pipeline-bubble fraction, stage 0's 12-layer slice (the PP4 stage-0 layers, timed inside the N = 1 run),
the MoE gate_up GEMM's roofline and the model's algorithmic FLOP rate. `e2e`: the same timed microbatches through the
public path with each microbatch's plan metadata and token ids packed on the host and copied in (`prepare`) and the
last stage's greedy tokens copied back to pinned host memory, inside the timed region.

`--workload sessions` (not the default line): the same stages serving BASELINE config 5's closed-loop session load
(`ssengine_b200.controller`): stage 0's host forms microbatches with the SRPT scheduler over the page pool with the
exact prefix cache (optionally a DRAM tier under it, `--dram-gb`), by the dispatch rule's projection (`--forming`),
and the line reports TTFT p50 / p90 / p99, rounds a second, computed and new tokens a second and the prefix-hit share
over the rounds arriving after `--session-warm-s`.

`--impl reference` times the reference's path on the host cores: the reference has no CPU implementation (its GPU path
needs a vLLM fork and FlashInfer builds absent here), so it times this repository's CPU restatement (oracle/) of each
layer kind on a bounded sample of a microbatch (rank 0 only), with weights built on the host without the CUDA library.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, F, E, K_TOP = 4096, 1024, 128, 8
SEED = 20261201
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch at T = 8192, from the ncu capture summarised in
# profiles/gemm_nvfp4_moe_T8192_full.md (796.9 MB + 39.6 MB); None for other token counts
GATE_UP_TRAFFIC_T8192 = 836.4e6
BASELINE_PP4_TOK_S = 138_400.0        # the reference's published saturated 8k prefill at PP4 on 4 x B200
                                      # (its docs/results/fp8.md:59)
N_LAYERS, MB_TOKENS, N_PROMPTS = 45, 8192, 256
MB_PER_STEP = 4                       # pipeline: a step = 4 microbatches, so K = 20 steps time 80 microbatches
MODEL = dict(hidden=4096, inter=1024, experts=128, top_k=8, vocab=151_552, kda_heads=64, q_lora=1536, mla_nope=192,
             mla_v_dim=256, dense_layers=3, dense_inter=12288, routing="sigmoid", layer_kind="hybrid")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference", "vllm-cutlass"], default="ours")
    ap.add_argument("--workload", choices=["pipeline", "moe-layer", "components", "sessions"], default="pipeline",
                    help="components: the attention-pair kernels and the mHC boundary alone (profiling runs); "
                         "sessions: the pipeline serving BASELINE config 5's closed-loop session load (TTFT)")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="pipeline: model layers (45 = BASELINE config 4)")
    ap.add_argument("--tokens", type=int, default=MB_TOKENS, help="tokens per microbatch")
    ap.add_argument("--mb-per-step", type=int, default=MB_PER_STEP,
                    help="pipeline: microbatches a step feeds the pipeline (the same timed set at every N)")
    ap.add_argument("--cpu-tokens", type=int, default=16, help="CPU baseline sample (tokens)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-clocks", action="store_true", help="skip the nvidia-smi window (profiling runs)")
    ap.add_argument("--no-components", action="store_true", help="skip the per-component timings")
    ap.add_argument("--sessions", type=int, default=400, help="sessions: concurrent closed-loop sessions")
    ap.add_argument("--session-s", type=float, default=60.0, help="sessions: seconds of arrivals")
    ap.add_argument("--session-warm-s", type=float, default=20.0,
                    help="sessions: rounds arriving in the first seconds are served but not measured")
    ap.add_argument("--think-s", type=float, default=5.0, help="sessions: mean think time")
    ap.add_argument("--start-ctx", type=int, default=16_384,
                    help="sessions: a session's first round brings a context uniform in [0, start-ctx)")
    ap.add_argument("--pool-gb", type=float, default=100.0,
                    help="sessions: device memory per stage for KV and state blocks (the pool size follows)")
    ap.add_argument("--force-after-ms", type=float, default=60_000.0, help="sessions: force-schedule bound")
    ap.add_argument("--forming", choices=["rule", "limits"], default="rule",
                    help="sessions: form each microbatch when the dispatch rule's projection says so (the reference "
                         "controller's way), or whenever the in-flight limits allow")
    ap.add_argument("--dram-gb", type=float, default=0.0,
                    help="sessions: pinned host memory per stage for the DRAM tier under HBM (0: no tier)")
    return ap.parse_args()


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def workload(T: int) -> str:
    return (f"BASELINE config 2: one NVFP4 MoE layer, {T} tokens, hidden {H}, {E} experts top-{K_TOP} + 1 shared, "
            f"expert FFN {H}->2x{F} SwiGLU->{H}")


def layer_flops(T: int) -> float:
    rows = T * K_TOP + T
    return 2.0 * T * H * E + rows * (2.0 * H * 2 * F + 2.0 * F * H)


# ---------------------------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampler over a time window (every 100 ms)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 7]
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx.append(float(r[1]))
            except ValueError:
                continue
            for n, v in zip(names, r[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------- CPU side
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def dense_on_host(layer) -> tuple[dict, dict]:
    """The layer's logical NVFP4 parameters and their fp32 dequantization (done on the device: exact products and
    one IEEE division, the same values as the checker's numpy dequantization), copied to host memory."""
    import numpy as np
    import torch

    from ssengine_b200 import layout

    dev = layer.device
    e2m1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], device=dev)
    e4m3 = torch.tensor([float(v) for v in _e4m3_table()], device=dev)

    def deq(codes, sf, gs):
        v = e2m1[codes.long()].view(codes.shape[0], -1, 16) * e4m3[sf.long()][:, :, None]
        return (v / torch.tensor(gs, dtype=torch.float32, device=dev)).reshape(codes.shape[0], -1)

    Hh, Ff, Ee = layer.H, layer.F, layer.E
    rc = layout.unpack_codes(layer.router_codes)[:Ee]
    rs = layout.atoms_to_sf(layer.router_sf, layer.router_rows, Hh)[:Ee]
    g_r = float(1.0 / (layer.router_alpha * layer.gs_x))
    experts, logical = [], []
    a1 = layer.w1_alpha.cpu().numpy().astype(np.float64)
    a2 = layer.w2_alpha.cpu().numpy().astype(np.float64)
    s1n, s2n = layer.w1_sf.numel() // (Ee + 1), layer.w2_sf.numel() // (Ee + 1)
    c1a = layer.w1_codes.view(Ee + 1, 2 * Ff, Hh // 2)
    c2a = layer.w2_codes.view(Ee + 1, Hh, Ff // 2)
    for e in range(Ee + 1):
        c1 = layout.gate_up_deinterleave(layout.unpack_codes(c1a[e]))
        s1 = layout.gate_up_deinterleave(layout.atoms_to_sf(layer.w1_sf[e * s1n:(e + 1) * s1n], 2 * Ff, Hh))
        c2 = layout.unpack_codes(c2a[e])
        s2 = layout.atoms_to_sf(layer.w2_sf[e * s2n:(e + 1) * s2n], Hh, Ff)
        g1, g2 = float(1.0 / (a1[e] * layer.gs_x)), float(1.0 / (a2[e] * layer.gs_h))
        experts.append((deq(c1, s1, g1).cpu().numpy(), deq(c2, s2, g2).cpu().numpy()))
        logical.append((None, None, g1, None, None, g2))
        del c1, s1, c2, s2
    dense = {"router": deq(rc, rs, g_r).cpu().numpy(), "experts": experts}
    p = {"H": Hh, "F": Ff, "E": Ee, "gs_x": layer.gs_x, "gs_h": layer.gs_h, "router": (None, None, g_r),
         "experts": [(np.empty((2 * Ff, 0), dtype=np.uint8),) + tuple(l[1:]) for l in logical]}
    return p, dense


def _e4m3_table():
    out = []
    for c in range(256):
        s, e, m = c >> 7, (c >> 3) & 0xF, c & 7
        v = float("nan") if (e == 15 and m == 7) else (m * 2.0 ** -9 if e == 0 else (1 + m / 8) * 2.0 ** (e - 7))
        out.append(-v if s else v)
    return out


def time_oracle(p: dict, dense: dict, x_np, reps: int = 1) -> float:
    """Seconds per forward of the CPU restatement over x_np (weights already fp32)."""
    from oracle import moe as omoe

    t0 = time.perf_counter()
    for _ in range(reps):
        omoe.moe_forward(x_np, p, K_TOP, dense=dense)
    return (time.perf_counter() - t0) / reps




# ---------------------------------------------------------------------------------------------- pipeline workload
def split_for(n_stages: int, layers: int = N_LAYERS) -> tuple:
    """Layers per stage: even splits with the remainder on the first stages -- the reference's 12/11/11/11 at PP4
    (ssengine/kernels.py:277), 23/22 at PP2, 6/6/6/6/6/5/5/5 at PP8, all 45 layers as one stage at N = 1."""
    base, extra = divmod(layers, n_stages)
    return tuple(base + (1 if s < extra else 0) for s in range(n_stages))


def pipeline_plans(n_mb: int, mb_tokens: int, vocab):
    """The first n_mb microbatches of BASELINE config 4's prompt stream and the block pool they need."""
    from ssengine_b200 import schedule

    lengths = schedule.prompt_lengths(N_PROMPTS, SEED)
    plans, high = schedule.microbatches(lengths, mb_tokens, n_mb, vocab=vocab, seed=SEED)
    return plans, high + 2                              # the null block and one spare


def pipeline_workload(args, world: int) -> str:
    return (f"BASELINE config 4: random-init Glm5Next NVFP4, {args.layers} layers (KDA 64 x 128; DSA at 3, 7, ...: "
            f"64 MLA heads, e4m3 latent 512 + rope 64, indexer 32 x 128 top-512 pools; dense SwiGLU FFN in layers 0-2; "
            f"128 experts top-8 + shared, F {F}, sigmoid + bias routing; vocab {MODEL['vocab']}), PP{world} split "
            f"{'/'.join(map(str, split_for(world, args.layers)))}, {args.tokens}-token microbatches of {N_PROMPTS} cold "
            f"prompts (lognormal lengths, median 8,192, max 131,072)")


def microbatch_flops(plan, cfg, layers: int) -> float:
    """Algorithmic FLOPs of one microbatch through `layers` layers and the head: 2 K N per token for every
    projection, expert and FFN GEMM (router, 8 routed experts + the shared one, absorb / v_up, indexer projections),
    the mHC mixes, the KDA chunked recurrence at ~4 products of 128 x 128 per token and head, the indexer score
    32 x 128 x 2 per visible pool ((pos + 1) // 4) and the sparse MLA 64 heads x (576 + 512) x 2 per selected token
    (min(2,051, pos + 1)), and the head on the finished rows."""
    import numpy as np

    Hd, P, nh = cfg.hidden, cfg.kda_heads * 128, cfg.kda_heads
    pos = np.concatenate([np.arange(c.start, c.start + c.num_tokens) for c in plan.chunks]).astype(np.float64)
    T = float(len(pos))
    sel = float(np.minimum(2051, pos + 1).sum())
    pools = float(((pos + 1) // 4).sum())
    kda = 2 * Hd * (3 * P + 256 + nh) + 2 * 2 * 128 * P + 2 * P * Hd + 2 * 4 * 128 * 128 * nh
    qh = cfg.mla_nope + 64
    dsa = (2 * Hd * (cfg.q_lora + 576) + 2 * cfg.q_lora * 64 * qh + 2 * 64 * cfg.mla_nope * 512
           + 2 * 64 * 512 * cfg.mla_v_dim + 2 * 64 * cfg.mla_v_dim * Hd + 2 * cfg.q_lora * 4096 + 2 * Hd * 288)
    moe = 2 * Hd * cfg.experts + (cfg.top_k + 1) * (2 * Hd * 2 * cfg.inter + 2 * cfg.inter * Hd)
    dense = 2 * Hd * 2 * cfg.dense_inter + 2 * cfg.dense_inter * Hd
    mhc = 2 * 2 * 24 * 4 * Hd
    total = 0.0
    for i in range(layers):
        is_dsa = i % 4 == 3
        total += T * (mhc + (dsa if is_dsa else kda) + (dense if i < cfg.dense_layers else moe))
        if is_dsa:
            total += sel * 64 * (576 + 512) * 2 + pools * 32 * 128 * 2
    n_last = sum(1 for c in plan.chunks if c.is_last)
    return total + n_last * 2 * Hd * cfg.vocab


def run_pipeline(args, rank: int, world: int, local: int) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from ssengine_b200 import lib
    from ssengine_b200.edge import P2pPipe
    from ssengine_b200.stage import StageConfig, StageModel
    from ssengine_b200.worker import StageWorker

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    split = split_for(world, args.layers)
    W, K, M = max(3, args.warmup), args.steps, max(1, args.mb_per_step)
    n_warm, n_timed = W * M, K * M
    plans, nb = pipeline_plans(n_warm + n_timed, args.tokens, MODEL["vocab"] if rank == 0 else None)
    if len(plans) < n_warm + n_timed:
        raise SystemExit(f"the prompt stream gives only {len(plans)} microbatches")
    cfg = StageConfig(layer_split=split, mb_tokens=args.tokens, num_blocks=nb, seed=SEED % 997, **MODEL)
    stage = StageModel(cfg, rank, device)
    pipe = None
    if world > 1:
        # up to world + 2 microbatches in flight: every stage busy, with slack for the edge hop and uneven stages
        pipe = P2pPipe(rank, world, device, None, max_in_flight=world + 2, max_rows=args.tokens,
                       width=stage.hidden_width, init_group=False, wait_ns=60_000_000_000)
    worker = StageWorker(stage, pipe, events=True)
    batches = [stage.prepare(p) for p in plans]
    pack_bytes = [int(b.keep[0].numel()) for b in batches[n_warm:]]
    for b in batches[:n_warm]:
        worker.step(b)
    torch.cuda.synchronize()
    if pipe is not None:
        pipe.check()
    if int(stage.status.item()):
        raise lib.SsbError("stage device status", int(stage.status.item()))

    # N = 1: stage 0 of the PP4 split (layers 0-11) timed inside the forward by an event after layer 11
    slice_ev = []
    if world == 1 and len(stage.layers) >= 12:
        eleventh = stage.layers[11]

        def hook(layer, *_):
            if layer is eleventh:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                slice_ev.append(ev)

        stage.layer_hook = hook
    marks = []
    if rank == 0:
        stage.moe_profile = []
    clocks = Clocks(_gpu_id(device)) if rank == 0 and not args.no_clocks else None
    if clocks is not None:
        clocks.start()
        time.sleep(0.3)
    worker.spans.clear()
    so = lib.load()
    so.launches = 0
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    so.on = True
    t0.record()
    for b in batches[n_warm:]:
        if rank == 0:
            marks.append(len(stage.moe_profile))
        worker.step(b)
    t1.record()
    so.on = False
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    if pipe is not None:
        pipe.check()
    if int(stage.status.item()):
        raise lib.SsbError("stage device status", int(stage.status.item()))
    elapsed = t0.elapsed_time(t1)
    busy = worker.busy_ms()
    launches = so.launches
    slice_ms = sum(a.elapsed_time(e) for (a, _), e in zip(worker.spans, slice_ev)) if slice_ev else None
    gate = None
    if rank == 0:
        marks.append(len(stage.moe_profile))
        g_ms = g_fl = 0.0
        for i in range(n_timed):
            T = batches[n_warm + i].num_tokens
            for evs in stage.moe_profile[marks[i]:marks[i + 1]]:
                g_ms += evs[6].elapsed_time(evs[7])
                g_fl += 2.0 * T * (K_TOP + 1) * 2 * F * H
        gate = (g_ms, g_fl, marks[-1] - marks[0])
        stage.moe_profile = None
    stage.layer_hook = None

    e2e_ms, d2h = None, 0
    if not args.no_e2e:
        worker.events = False
        host_tok = torch.empty(4096, dtype=torch.int64, pin_memory=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for p in plans[n_warm:]:
            out = worker.step(p)                       # plan -> pinned pack -> one H2D copy -> forward
            if out is not None and out.numel():
                host_tok[:out.numel()].copy_(out, non_blocking=True)
                d2h += out.numel() * 8
        e1.record()
        torch.cuda.synchronize()
        if pipe is not None:
            pipe.check()
        e2e_ms = e0.elapsed_time(e1)

    mine = {"rank": rank, "elapsed": elapsed, "busy": busy, "e2e": e2e_ms, "launches": launches, "d2h": d2h}
    allr = [mine]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine)
    if rank == 0:
        pk, src = peaks()
        tokens = sum(b.num_tokens for b in batches[n_warm:])
        t_max = max(r["elapsed"] for r in allr)
        value = tokens / (t_max / 1e3)
        flops = sum(microbatch_flops(p, cfg, args.layers) for p in plans[n_warm:])
        sus = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        fp4_sus = 4.0 * sus
        g_ms, g_fl, n_g = gate
        achieved = g_fl / (g_ms / 1e3) / 1e12 if g_ms else None
        line = {
            "metric": "prefill tok/s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": t_max / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": value / BASELINE_PP4_TOK_S if world == 4 else None,
            "dtype": "nvfp4 (e2m1 x e2m1, ue4m3 per-16 scales) GEMMs; e4m3 attention; bf16 residual; fp32 KDA state",
            "data": "synthetic: uniform token ids, lognormal prompt lengths, seeded random-init weights",
            "config": {"workload": pipeline_workload(args, world), "global_batch": args.tokens * M,
                       "step": f"{M} microbatches of {args.tokens} tokens fed into the pipeline (the same "
                               f"{n_timed} timed microbatches at every N; fill and drain inside the timed region)",
                       "seq_len": "lognormal median 8192, max 131072", "parallelism": f"pp{world}",
                       "layer_split": list(split), "tokens_timed": tokens,
                       "l2": "inputs larger than L2 (each stage streams >= 10 GB of weights per microbatch)"},
            "pipeline": {"max_rank_ms": t_max, "per_rank_ms": [r["elapsed"] for r in allr],
                         "per_rank_busy_ms": [r["busy"] for r in allr], "microbatches_timed": n_timed,
                         "busiest_stage_tok_s": tokens / (max(r["busy"] for r in allr) / 1e3),
                         "bubble_fraction": 1.0 - sum(r["busy"] for r in allr) / (world * t_max),
                         "edge": "last boundary kernel stores into the next GPU's slot (P2P over NVLink), bounded "
                                 "flag waits, no NCCL"},
            "roofline": {"kernel": "MoE gate_up grouped NVFP4 GEMM (SwiGLU + requant epilogue), rank 0's MoE layers",
                         "bound": "tensor", "achieved": achieved, "peak": fp4_sus, "unit": "TFLOP/s",
                         "frac": achieved / fp4_sus if achieved else None,
                         "traffic": GATE_UP_TRAFFIC_T8192 if args.tokens == 8192 else None,
                         "traffic_unit": "bytes per launch at T = 8192 (ncu capture)", "launches": n_g,
                         "peak_source": f"4 x {src} sustained dense bf16 {sus} TFLOP/s (timed inside a long step; "
                                        f"B200's dense NVFP4 rate is 4x bf16)"},
            "model_flop_rate": {"tflops": flops / (t_max / 1e3) / 1e12,
                                "frac_of_nvfp4_sustained": flops / (t_max / 1e3) / 1e12 / (world * fp4_sus),
                                "algorithmic_flop": flops},
            "gpu_launches": sum(r["launches"] for r in allr),
            "clocks": clk,
        }
        if slice_ms:
            line["stage0_slice"] = {"layers": "0-11 (PP4 stage 0: 3 dense-FFN layers, 6 KDA + MoE, 3 DSA + MoE)",
                                    "tok_per_s": tokens / (slice_ms / 1e3), "ms_per_microbatch": slice_ms / n_timed,
                                    "reference_stage0_target_ms": 57.0}
        if e2e_ms is not None:
            e2e_max = max(r["e2e"] for r in allr)
            line["e2e"] = {"value": tokens / (e2e_max / 1e3), "unit": "tok/s",
                           "h2d_bytes_per_step": sum(pack_bytes) / K * world,
                           "d2h_bytes_per_step": sum(r["d2h"] for r in allr) / K,
                           "path": "StageWorker.step(plan): host pack of the plan's metadata and token ids, one "
                                   "pinned H2D copy per stage, forward, greedy tokens read back to pinned memory"}
        if world == 1 and not args.no_components:
            del worker, batches, stage
            torch.cuda.empty_cache()
            line["components"] = time_components(device, pk)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_model_baseline(args.cpu_tokens, steps=2, warm=1, layers=args.layers)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        if pipe is not None:
            pipe.close()
        dist.barrier()
        dist.destroy_process_group()


def session_pool_blocks(split, pool_bytes: float, kda_heads: int = MODEL["kda_heads"], cap: int = 7143) -> int:
    """Usable blocks of the session run's pool: what `pool_bytes` holds on the stage whose blocks cost the most (one
    block-id space serves every stage), at most the reference's 7,143 (7,144 with the null block)."""
    from ssengine_b200.kvpages import block_bytes

    start, worst = 0, 0
    for n in split:
        worst = max(worst, block_bytes(list(range(start, start + n)), lambda i: i % 4 == 3, kda_heads))
        start += n
    return max(1, min(cap, int(pool_bytes // worst)))


def run_sessions(args, rank: int, world: int, local: int) -> None:
    """The pipeline serving a closed-loop session load (BASELINE config 5's shape): stage 0's host runs the scheduler
    (SRPT, `--tokens` microbatches, force-schedule) over the page pool with the exact prefix cache and sends each plan
    to the other stages; TTFT = the round's greedy token on stage 0's host minus its arrival."""
    import datetime

    import torch
    import torch.distributed as dist

    from ssengine_b200 import lib
    from ssengine_b200.controller import Controller, Reporter, SessionLoad, StoreChannel, cuda_step, serve_stage
    from ssengine_b200.dispatch import DispatchRule
    from ssengine_b200.edge import P2pPipe
    from ssengine_b200.pagepool import KvManager
    from ssengine_b200.scheduler import Scheduler, SchedulerConfig
    from ssengine_b200.stage import StageConfig, StageModel
    from ssengine_b200.tier import DramTier, TierArena
    from ssengine_b200.worker import StageWorker

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    split = split_for(world, args.layers)
    blocks = session_pool_blocks(split, args.pool_gb * 1e9)
    cfg = StageConfig(layer_split=split, mb_tokens=args.tokens, num_blocks=blocks + 1, seed=SEED % 997, **MODEL)
    stage = StageModel(cfg, rank, device)
    gate = world + 2
    pipe = None
    if world > 1:
        pipe = P2pPipe(rank, world, device, None, max_in_flight=gate, max_rows=args.tokens,
                       width=stage.hidden_width, init_group=False, wait_ns=60_000_000_000)
    dram_blocks = session_pool_blocks(split, args.dram_gb * 1e9, cap=1 << 30) if args.dram_gb > 0 else 0
    arena = TierArena(stage.kv, rank, dram_blocks, device=device) if dram_blocks else None
    worker = StageWorker(stage, pipe, events=True, tier=arena)
    step = cuda_step(worker, device)
    chan = None
    if world > 1:
        chan = StoreChannel(dist.PrefixStore("ctl/", dist.distributed_c10d._get_default_store()))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    so = lib.load()
    so.launches, so.on = 0, True
    init = (lambda: torch.cuda.set_device(local))
    summary = None
    if rank == 0:
        kv = KvManager(blocks, keep_sessions=True)
        if dram_blocks:
            kv.lower = DramTier(dram_blocks)
        rule = DispatchRule(max_in_flight=gate, lead_ms=3.0, num_stages=world) if args.forming == "rule" else None
        sched = Scheduler(kv, SchedulerConfig(order="srpt", mb_tokens=args.tokens, force_after_ms=args.force_after_ms),
                          None, *(rule.sched_limits if rule is not None else (gate + 1, 1)))
        load = SessionLoad(sessions=args.sessions, seed=SEED, vocab=MODEL["vocab"], think_s=args.think_s,
                           start_ctx_max=args.start_ctx, stagger_s=min(5.0, args.session_warm_s))
        ctl = Controller(sched, load, world, rule=rule)
        rep = Reporter(0, ctl.local.put, init=init)
        summary = ctl.run(step, rep, chan, duration_s=args.session_s, warm_s=args.session_warm_s)
        rep.close()
        summary["kv"] = {k: int(v) for k, v in kv.stats.items()}
        if kv.lower is not None:
            summary["dram_tier"] = {k: int(v) for k, v in kv.lower.stats.items()}
        busy = [m.get("busy0", 0) for m in ctl.microbatches]
        summary["stage0_busy_s"] = sum(busy) / 1e9
    else:
        serve_stage(step, chan, Reporter(rank, chan.put_report, init=init))
    so.on = False
    torch.cuda.synchronize()
    if pipe is not None:
        pipe.check()
    if arena is not None:
        arena.check()
    if int(stage.status.item()):
        raise lib.SsbError("stage device status", int(stage.status.item()))
    mine = {"rank": rank, "launches": so.launches, "tier_bytes": arena.bytes_moved if arena is not None else 0}
    allr = [mine]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine)
    if rank == 0:
        line = {
            "metric": "TTFT p50 under the synthetic session load", "value": summary["ttft_s"]["p50"], "unit": "s",
            "higher_is_better": False, "n_gpus": world, "ttft_s": summary["ttft_s"],
            "rounds_per_s": summary["rounds_per_s"], "computed_tok_s": summary["computed_tok_s"],
            "new_tok_s": summary["new_tok_s"], "prefix_hit_share": summary["prefix_hit_share"],
            "dtype": "nvfp4 GEMMs; e4m3 attention; bf16 residual; fp32 KDA state",
            "data": "synthetic: closed-loop sessions, uniform token ids from a seeded hash stream, random-init weights",
            "config": {"workload": f"config 5 shape: {args.sessions} sessions, appends lognormal median 600 max 8192, "
                                   f"context cap 131072, think Exp({args.think_s} s), first contexts U[0, "
                                   f"{args.start_ctx}), {args.session_s:.0f} s of arrivals, rounds arriving after "
                                   f"{args.session_warm_s:.0f} s measured",
                       "parallelism": f"pp{world}", "layer_split": list(split),
                       "scheduler": f"srpt, {args.tokens}-token microbatches, force after {args.force_after_ms} ms, "
                                    f"in-flight gate {gate} on the GPU, formed "
                                    + ("by the dispatch rule's projection" if args.forming == "rule"
                                       else "whenever the in-flight limits allow"),
                       "pool": f"{blocks} blocks per stage, kept sessions LRU; "
                               + (f"DRAM tier of {dram_blocks} blocks per stage ({args.dram_gb:.0f} GB pinned), "
                                  f"exclusive, copies in stream order" if dram_blocks else "no DRAM tier")},
            "dram_tier": summary.get("dram_tier"), "tier_bytes_per_rank": [r["tier_bytes"] for r in allr],
            "rounds": summary["rounds"], "unfinished": summary["unfinished"], "microbatches": summary["microbatches"],
            "kv": summary["kv"], "stage0_busy_s": summary["stage0_busy_s"], "decisions": summary["decisions"],
            "gpu_launches": sum(r["launches"] for r in allr),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if pipe is not None:
            pipe.close()
        dist.barrier()
        dist.destroy_process_group()


def _gpu_id(device) -> str:
    import torch

    props = torch.cuda.get_device_properties(device)
    gid = str(getattr(props, "uuid", device.index))
    return gid if gid.startswith("GPU-") or not gid.count("-") else "GPU-" + gid


# ---------------------------------------------------------------------------------------------- CPU baseline
def cpu_model_baseline(sample: int, steps: int, warm: int, layers: int = N_LAYERS) -> dict:
    """CPU time of the model per token through the oracle (oracle/), each piece timed on `sample` rows of a
    microbatch and summed over the model's layers: an mHC boundary (two per layer), a KDA attention block continuing a
    request (random recurrent and conv state), a DSA attention block on rows at the end of an 8,192-token prompt
    (random e4m3 latent cache and pool keys for the prefix: the indexer over ~2,044 pools, top-512, sparse MLA over
    2,051 tokens), the MoE (128 experts top-8 + shared), the dense FFN. Weights are built on the host with torch's
    CPU generator (no CUDA library involved) and dequantized once, in the warm-up (oracle/nvfp4.WEIGHT_MEMO); numpy
    uses every host thread."""
    import numpy as np
    import torch

    from oracle import kda as ok
    from oracle import mhc as omhc
    from oracle import model as omodel
    from oracle import moe as omoe
    from oracle import nvfp4
    from oracle.mhc import bf16
    from ssengine_b200 import weights

    torch.set_num_threads(cpu_threads())
    g = torch.Generator().manual_seed(SEED)
    rng = np.random.default_rng(SEED)
    n, Hd, nh = sample, H, MODEL["kda_heads"]
    P = nh * 128

    def lin(N, K):
        c, s, gs = weights.nvfp4_tensor(g, N, K, "cpu")
        return c.numpy(), s.numpy(), gs

    kda_p = dict(in_proj=lin(3 * P + 256 + nh, Hd), f_b=lin(P, 128), g_b=lin(P, 128), o_proj=lin(Hd, P),
                 conv_w=bf16(rng.uniform(-0.6, 0.6, (3 * P, 4))), a_log=rng.uniform(-1, 1, nh),
                 dt_bias=rng.standard_normal(P) * 0.5, norm_w=np.ones(128), heads=nh, eps=1e-5)
    ql, nope, vd = MODEL["q_lora"], MODEL["mla_nope"], MODEL["mla_v_dim"]
    dsa_p = dict(a_proj=lin(ql + 576, Hd), q_b=lin(64 * (nope + 64), ql), wq_idx=lin(4096, ql), idx_proj=lin(288, Hd),
                 o_proj=lin(Hd, 64 * vd), w_uk=(bf16(rng.standard_normal((64, 512, nope)) / nope ** 0.5),),
                 w_uv=(bf16(rng.standard_normal((64, vd, 512)) / 512 ** 0.5),), q_norm=np.ones(ql),
                 kv_norm=np.ones(512), ape=rng.standard_normal((4, 128)) * 0.5, q_lora=ql, nope=nope, v_dim=vd,
                 theta=10000.0, eps=1e-6, scale=(nope + 64) ** -0.5, q_scale=1.0, k_scale=1.0)
    moe_p = weights.to_numpy(weights.moe_logical(SEED, Hd, F, E, routing="sigmoid"))
    dense_w = lin(2 * MODEL["dense_inter"], Hd) + lin(Hd, MODEL["dense_inter"])
    bound = (rng.standard_normal((24, 4 * Hd)) / (4 * Hd) ** 0.5, np.array([0.8, 0.6, 1.5]),
             rng.standard_normal(24) * 0.3, 1e-6, 1e-2, 1e-6, 2.0, 20, np.ones(Hd), 1e-6)
    y = bf16(rng.standard_normal((n, Hd)))
    res = bf16(rng.standard_normal((n, 4, Hd)))
    post = rng.uniform(0.5, 1.5, (n, 4)).astype(np.float32)
    comb = np.full((n, 4, 4), 0.25, np.float32)
    cst = bf16(rng.standard_normal((2, 3, 3 * P)))
    rst = (rng.standard_normal((2, nh, 128, 128)) * 0.05).astype(np.float32)
    L = 8192
    pages = np.arange(1, L // 128 + 1)
    kv = rng.integers(0, 0x7E, ((int(pages.max()) + 1) * 128, 576)).astype(np.uint8)
    kv |= (rng.integers(0, 2, kv.shape) << 7).astype(np.uint8)
    pool = bf16(rng.standard_normal(((int(pages.max()) + 1) * 32, 128)))
    tail = bf16(rng.standard_normal((2, 2, 4, 128)))
    positions = np.arange(L - n, L)
    counts = {"mhc": 2 * layers, "kda": sum(1 for i in range(layers) if i % 4 != 3),
              "dsa": sum(1 for i in range(layers) if i % 4 == 3), "dense": min(3, layers),
              "moe": layers - min(3, layers)}
    pieces = {
        "mhc": lambda: omhc.post_pre(y, res, post, comb, *bound),
        "kda": lambda: ok.attention_block(y, kda_p, cst, rst, [(0, n, 1, 1)], nh, weights.GS_X, 1e-5),
        "dsa": lambda: omodel.dsa_block(y, dsa_p, positions, [(0, n, L - n, pages, 1)], kv, pool, tail.copy(),
                                        weights.GS_X),
        "moe": lambda: omoe.moe_forward(y, moe_p, K_TOP, dense="lazy"),
        "dense": lambda: omodel.dense_ffn(y, dense_w, weights.GS_X, weights.GS_H),
    }
    nvfp4.WEIGHT_MEMO = {}
    try:
        for _ in range(warm):
            for fn in pieces.values():
                fn()
        per = {k: [] for k in pieces}
        for _ in range(steps):
            for k, fn in pieces.items():
                t = time.perf_counter()
                fn()
                per[k].append(time.perf_counter() - t)
    finally:
        nvfp4.WEIGHT_MEMO = None
    sec = {k: statistics.mean(v) for k, v in per.items()}
    per_token = sum(counts[k] * sec[k] for k in sec) / n
    return {"value": 1.0 / per_token, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"{n} rows of a microbatch through each layer piece of oracle/ (numpy, weights dequantized "
                      f"before timing), summed over the {layers}-layer model: "
                      + ", ".join(f"{k} {sec[k] * 1e3:.0f} ms x {counts[k]}" for k in sec),
            "step_seconds": sum(sec.values())}


# ---------------------------------------------------------------------------------------------- moe-layer workload
def build_layer(device, T: int, rank: int):
    import __graft_entry__

    __graft_entry__.import_package()
    from ssengine_b200 import moe, weights

    p = weights.moe_logical(SEED, H, F, E, device=device)
    layer = moe.MoELayer.from_logical(p, K_TOP, device)
    del p
    x = weights.hidden_states(SEED + 1 + rank, T, H, device=device)
    return layer, x


def run_reference(args, rank: int) -> None:
    """The reference arm: the CPU restatement of the path on the host cores (rank 0 only), weights built on the host
    with torch's CPU generator (no CUDA library), dequantized before timing."""
    if rank != 0:
        return
    if args.workload == "pipeline":
        W, K = max(1, args.warmup), args.steps
        cb = cpu_model_baseline(args.cpu_tokens, steps=K, warm=W, layers=args.layers)
        v = cb["value"]
        line = {"impl": "reference", "metric": "prefill tok/s", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
                "steps": K, "warmup": W, "ms_per_step": cb["step_seconds"] * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f64 / f32 (dequantized NVFP4 weights)",
                "data": "synthetic: uniform token ids, seeded random-init weights",
                "config": {"workload": pipeline_workload(args, args.gpus), "sample_tokens": args.cpu_tokens},
                "cpu_baseline": cb,
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    import torch

    from oracle import moe as omoe
    from ssengine_b200 import weights

    torch.set_num_threads(cpu_threads())
    layer_T = args.tokens
    sample = min(max(args.cpu_tokens, 256), layer_T)
    p = weights.to_numpy(weights.moe_logical(SEED, H, F, E))
    dense = omoe.dequantize_params(p)
    x_np = weights.hidden_states(SEED + 1, sample, H).float().numpy()
    for _ in range(args.warmup):
        time_oracle(p, dense, x_np)
    t = [time_oracle(p, dense, x_np) for _ in range(args.steps)]
    sec = sum(t) / len(t)
    v = sample / sec
    line = {"impl": "reference", "metric": "prefill tok/s", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantized NVFP4 weights)",
            "data": "synthetic: hidden N(0,1) bf16, seeded random-init NVFP4 weights",
            "config": {"workload": workload(layer_T), "sample_tokens": sample},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
                             "sample": f"{sample} of the {layer_T} tokens per step through oracle.moe.moe_forward "
                                       f"(numpy fp32, weights built on the host and dequantized before timing)"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_vllm_cutlass(args, rank: int) -> None:
    """Library comparison: the layer's experts through vLLM 0.22.0's `run_cutlass_moe_fp4` (row shuffle, activation
    NVFP4 quant, CUTLASS grouped GEMM, fused SiLU-and-mul + requant, grouped GEMM, unshuffle, weighted combine in
    torch), on the same weights and on the routing our router chose, the shared expert as expert E with weight 1.
    Timed like ours (CUDA events over K steps after W warm-up steps, weights and workspaces larger than L2); the line
    carries our own expert-path time (every step but the router GEMM and the routing) of the same run beside it."""
    if rank != 0:
        return
    import torch
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation
    from vllm.model_executor.layers.fused_moe.experts.cutlass_moe import run_cutlass_moe_fp4
    from vllm.model_executor.layers.quantization.utils.nvfp4_utils import swizzle_blockscale

    from ssengine_b200 import lib, moe, weights

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    T, steps, warm = args.tokens, args.steps, max(3, args.warmup)
    p = weights.moe_logical(SEED, H, F, E, device=device)
    layer = moe.MoELayer.from_logical(p, K_TOP, device)
    x = weights.hidden_states(SEED + 1, T, H, device=device)
    out = torch.empty_like(x)
    for _ in range(warm):
        layer.forward(x, out)
    nst = len(lib.MOE_STEPS)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nst + 1)] for _ in range(steps)]
    for row in evs:
        for e in row:
            e.record()                              # creates the CUDA event the library records into
    for i in range(steps):
        layer.forward_profiled(x, out, evs[i])
    torch.cuda.synchronize()
    layer.check_status()
    ours = {name: sum(evs[i][s].elapsed_time(evs[i][s + 1]) for i in range(steps)) / steps
            for s, name in enumerate(lib.MOE_STEPS)}
    ours_experts = sum(v for n, v in ours.items() if n not in ("router_gemm", "route"))
    ids = layer.ws_view("IDS", T, torch.int32, (T, K_TOP)).clone()
    wts = layer.ws_view("WEIGHTS", T, torch.float32, (T, K_TOP)).clone()
    del layer
    torch.cuda.empty_cache()

    def pack(c):                                   # one code per byte -> two per byte, the even element low
        return (c[:, 0::2] | (c[:, 1::2] << 4)).contiguous()

    ex = p["experts"]
    w1 = torch.stack([pack(e[0]) for e in ex])
    s1 = swizzle_blockscale(torch.stack([e[1] for e in ex]).view(torch.float8_e4m3fn))
    w2 = torch.stack([pack(e[3]) for e in ex])
    s2 = swizzle_blockscale(torch.stack([e[4] for e in ex]).view(torch.float8_e4m3fn))
    gs1 = torch.tensor([e[2] for e in ex], dtype=torch.float32, device=device)
    gs2 = torch.tensor([e[5] for e in ex], dtype=torch.float32, device=device)
    del p, ex
    ne, kk = E + 1, K_TOP + 1
    a1 = torch.full((ne,), weights.GS_X, dtype=torch.float32, device=device)
    a2 = torch.full((ne,), weights.GS_H, dtype=torch.float32, device=device)
    al1, al2 = 1.0 / (a1 * gs1), 1.0 / (a2 * gs2)
    topk_ids = torch.cat([ids, torch.full((T, 1), E, dtype=torch.int32, device=device)], dim=1).contiguous()
    topk_w = torch.cat([wts, torch.ones((T, 1), dtype=torch.float32, device=device)], dim=1).contiguous()
    vout = torch.empty_like(x)
    ws13 = torch.empty(T * kk * max(2 * F, H), dtype=torch.bfloat16, device=device)
    ws2 = torch.empty(T * kk * F, dtype=torch.bfloat16, device=device)

    def step():
        run_cutlass_moe_fp4(vout, x, a1, w1, s1, al1, a2, w2, s2, al2, topk_w, topk_ids, MoEActivation.SILU, ws13,
                            ws2, T, F, H, ne, device)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    rel = float((vout.float() - out.float()).norm() / out.float().norm())
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    eager_ms = start.elapsed_time(end) / steps
    # the same step replayed from a CUDA graph, so that host-side launch and allocation costs do not count
    graph_ms, graph_err = None, None
    try:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(g):
            step()
        for _ in range(warm):
            g.replay()
        start.record()
        for _ in range(steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
        graph_ms = start.elapsed_time(end) / steps
    except Exception as exc:                        # noqa: BLE001 -- reported in the line
        graph_err = f"{type(exc).__name__}: {str(exc)[:160]}"
    ms = min(eager_ms, graph_ms) if graph_ms else eager_ms
    line = {"impl": "vllm-cutlass", "metric": "prefill tok/s", "value": T / ms * 1e3, "unit": "tok/s", "n_gpus": 1,
            "steps": steps, "warmup": warm, "ms_per_step": ms, "eager_ms_per_step": eager_ms,
            "graph_ms_per_step": graph_ms, "graph_error": graph_err, "higher_is_better": True,
            "dtype": "nvfp4 x nvfp4",
            "scope": "experts only: routing given (our router's), shared expert as expert E; vLLM 0.22.0 "
                     "run_cutlass_moe_fp4",
            "ours_experts_ms_per_step": ours_experts, "ours_layer_ms_per_step": sum(ours.values()),
            "rel_l2_vs_ours": rel, "data": "synthetic: hidden N(0,1) bf16, seeded random-init NVFP4 weights",
            "config": {"workload": workload(T),
                       "l2": "inputs larger than L2 (0.9 GB of expert weights + workspaces per step)"}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------- components
def _event_ms(fn, reps: int = 5, warm: int = 2) -> float:
    """Median device time of fn() over reps launches (CUDA events on the current stream, L2 flushed between)."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def attention_pair_requests(T: int = 32768, R: int = 8, seed: int = SEED):
    """BASELINE config 3's microbatch: R requests whose new-token counts are lognormal (median 2k) summing to T,
    appended to cached prefixes of 0-64k tokens."""
    import numpy as np

    rng = np.random.default_rng(seed)
    lens = rng.lognormal(np.log(2048), 1.0, R)
    lens = np.maximum(1, (lens / lens.sum() * T).astype(np.int64))
    lens[-1] += T - lens.sum()
    prefix = rng.integers(0, 65536, R)
    return lens, prefix


def time_components(device, pk: dict) -> dict:
    """Device time of the other hot-path kernels on BASELINE config 3 (KDA 32 x 128; DSA indexer 32 x 128 with
    top-2048 tokens = top-512 pools of 4, sparse MLA 64 heads, latent 512 + rope 64) and mHC at the stage shape."""
    import numpy as np
    import torch

    from ssengine_b200 import indexer, mla
    from ssengine_b200.kda import KdaLayer, seq_table

    out = {}
    lens, prefix = attention_pair_requests()
    T, R = int(lens.sum()), len(lens)
    order = np.argsort(-lens)
    starts = np.concatenate([[0], np.cumsum(lens)])
    g = torch.Generator(device=device).manual_seed(SEED)
    rnd = lambda *shape: torch.randn(*shape, device=device, generator=g)

    # KDA layer: conv + chunked scan + state pages (every request continues a cached prefix: has initial state)
    H, P = 32, 32 * 128
    x = rnd(T, 3 * P).to(torch.bfloat16)
    gr = rnd(T, P).to(torch.bfloat16)
    beta = rnd(T, H).to(torch.bfloat16)
    layer = KdaLayer((torch.rand(3 * P, 4, device=device, generator=g) - 0.5).to(torch.bfloat16),
                     torch.rand(H, device=device, generator=g) * 2 - 1, rnd(P) * 0.5, -5.0)
    cst = rnd(R + 1, 3, 3 * P).to(torch.bfloat16)
    rst = rnd(R + 1, H, 128, 128) * 0.05
    o = torch.empty(T, P, dtype=torch.bfloat16, device=device)
    st = seq_table([(int(starts[i]), int(starts[i + 1]), 1 + int(i), 1) for i in order], device)
    ms = _event_ms(lambda: layer.prefill(x, gr, beta, o, st, cst, rst))
    byts = T * (5 * P * 2 + 2 * H) + 2 * R * H * 128 * 128 * 4
    out["kda_prefill"] = {"ms": ms, "tokens": T, "heads": H, "requests": R, "bound": "hbm",
                          "achieved_gbs": byts / ms / 1e6, "frac": byts / ms / 1e6 / pk["hbm_gbs"],
                          "algorithmic_bytes": byts}
    del x, gr, beta, layer, cst, rst, o
    torch.cuda.empty_cache()

    # DSA: indexer logits -> canonical top-512 pools -> tokens -> sparse MLA
    positions = np.concatenate([np.arange(p0, p0 + n) for p0, n in zip(prefix, lens)]).astype(np.int64)
    n_pages = [-(-(int(p0) + int(n)) // 128) for p0, n in zip(prefix, lens)]
    width = max(n_pages)
    table = np.full((R, width), -1, np.int32)
    at = 1
    for r, n in enumerate(n_pages):
        table[r, :n] = np.arange(at, at + n)
        at += n
    qsl = starts.astype(np.int32)
    pos = torch.from_numpy(positions).to(device)
    tab = torch.from_numpy(table).to(device)
    groups = torch.from_numpy(indexer.work_groups(qsl[:-1], lens, prefix)).to(device)
    q_idx = rnd(T, 32, 128).to(torch.bfloat16)
    w = torch.rand(T, 32, device=device, generator=g).to(torch.bfloat16)
    kpool = rnd(at * 32, 128).to(torch.bfloat16)
    ldl = int(((positions.max() + 1) // 4 + 127) // 128 * 128)
    logits = torch.empty(T, ldl, device=device)
    ms = _event_ms(lambda: indexer.logits(q_idx, w, kpool, tab, groups, logits))
    vis = float(((positions + 1) // 4).sum())
    fl = vis * 32 * 128 * 2
    out["indexer_logits"] = {"ms": ms, "bound": "tensor", "achieved_tflops": fl / ms / 1e9,
                             "frac": fl / ms / 1e9 / pk["bf16_tflops"], "algorithmic_flop": fl,
                             "peak": f"dense bf16 {pk['bf16_tflops']} TFLOP/s"}
    ids = torch.empty(T, 512, dtype=torch.int32, device=device)
    ms = _event_ms(lambda: indexer.topk(logits, pos, 512, ids))
    byts = vis * 4 + T * 512 * 4
    out["indexer_topk"] = {"ms": ms, "bound": "hbm", "achieved_gbs": byts / ms / 1e6,
                           "frac": byts / ms / 1e6 / pk["hbm_gbs"], "algorithmic_bytes": byts}
    tok = torch.empty(T, 2051 + 5, dtype=torch.int32, device=device)
    out["indexer_expand"] = {"ms": _event_ms(lambda: indexer.expand(ids, pos, tok))}
    del logits, q_idx, kpool
    torch.cuda.empty_cache()
    # FP8 query and latent cache (e4m3 bytes; the values stay inside the e4m3 range)
    q = (rnd(T, 64, 576) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    kv = rnd(at * 128, 576).to(torch.float8_e4m3fn).view(torch.uint8)
    mo = torch.empty(T, 64, 512, dtype=torch.bfloat16, device=device)
    qsl_d = torch.from_numpy(qsl).to(device)
    ms = _event_ms(lambda: mla.sparse_mla(q, kv, tok, qsl_d, tab, 192 ** -0.5, mo, n_idx=2051), reps=3, warm=1)
    sel = float((tok[:, :2051] >= 0).sum().item())
    fl = sel * 64 * (576 + 512) * 2
    fp8_peak = 2 * pk["bf16_tflops"]
    out["sparse_mla"] = {"ms": ms, "bound": "tensor", "achieved_tflops": fl / ms / 1e9,
                         "frac": fl / ms / 1e9 / fp8_peak, "algorithmic_flop": fl,
                         "peak": f"dense fp8 {fp8_peak:.0f} TFLOP/s (2 x measured bf16)",
                         "selected_tokens_per_row": sel / T}
    del q, kv, mo, tok, ids
    torch.cuda.empty_cache()

    # mHC layer boundary (post + pre + Sinkhorn + RMSNorm) at the stage shape, T = 8192, H = 4096
    from ssengine_b200 import lib
    import ctypes

    Tm, Hm = 8192, 4096
    xm = rnd(Tm, Hm).to(torch.bfloat16)
    res = rnd(Tm, 4, Hm).to(torch.bfloat16)
    pin = torch.rand(Tm, 4, device=device, generator=g) + 0.5
    cin = torch.softmax(rnd(Tm, 4, 4), dim=1)
    fn = rnd(24, 4 * Hm) / 128.0
    scale = torch.tensor([0.8, 0.6, 1.5], device=device)
    base = rnd(24) * 0.3
    nw = torch.ones(Hm, device=device).to(torch.bfloat16)
    nr = torch.empty_like(res)
    po = torch.empty(Tm, 4, device=device)
    co = torch.empty(Tm, 4, 4, device=device)
    y = torch.empty_like(xm)
    prm = lib.MhcParamsC(Hm, 4, fn.data_ptr(), scale.data_ptr(), base.data_ptr(), nw.data_ptr(), 1e-6, 1e-2, 1e-6,
                         2.0, 1e-6, 20)
    so = lib.load()
    ws = torch.empty(int(so.ssb_mhc_workspace_bytes(Tm)), dtype=torch.uint8, device=device)

    def mhc():
        lib.check("ssb_mhc_ws", so.ssb_mhc_ws(ctypes.byref(prm), xm.data_ptr(), res.data_ptr(), pin.data_ptr(),
                                              cin.data_ptr(), nr.data_ptr(), po.data_ptr(), co.data_ptr(),
                                              y.data_ptr(), Tm, ws.data_ptr(), ws.numel(),
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))

    ms = _event_ms(mhc)
    byts = Tm * (4 * Hm * 2 * 2 + Hm * 2 * 2) + 24 * 4 * Hm * 4
    out["mhc_post_pre"] = {"ms": ms, "tokens": Tm, "bound": "hbm", "achieved_gbs": byts / ms / 1e6,
                           "frac": byts / ms / 1e6 / pk["hbm_gbs"], "algorithmic_bytes": byts}
    del xm, res, nr, y
    torch.cuda.empty_cache()

    # one full KDA + MoE decoder layer at the stage shape (boundary, KDA attention 64 x 128 with NVFP4 projections,
    # boundary, NVFP4 MoE 128 experts top-8 + shared), T = 8192 from 4 requests continuing cached prefixes
    from ssengine_b200.layers import KdaDecoderLayer

    Tl, heads = 8192, 64
    layer = KdaDecoderLayer(SEED, 4096, heads, F, E, K_TOP, device)
    lens_l = [3000, 2500, 1700, 992]
    st_l = np.concatenate([[0], np.cumsum(lens_l)])
    seqs_l = seq_table([(int(st_l[i]), int(st_l[i + 1]), i + 1, 1) for i in range(4)], device)
    res_l = rnd(Tl, 4, 4096).to(torch.bfloat16)
    x_l = rnd(Tl, 4096).to(torch.bfloat16)
    post_l = torch.rand(Tl, 4, device=device, generator=g) + 0.5
    comb_l = torch.softmax(rnd(Tl, 4, 4), dim=1)
    cst_l = rnd(5, 3, 3 * heads * 128).to(torch.bfloat16)
    rst_l = rnd(5, heads, 128, 128) * 0.05
    st_w = torch.zeros(1, dtype=torch.int32, device=device)
    ms = _event_ms(lambda: layer.forward(res_l, x_l, post_l, comb_l, seqs_l, cst_l, rst_l, st_w), reps=3, warm=1)
    out["kda_decoder_layer"] = {"ms": ms, "tokens": Tl, "tok_per_s": Tl / ms * 1e3, "heads": heads,
                                "note": "boundary + KDA attention (NVFP4 in_proj / f_b / g_b / o_proj, conv + scan, "
                                        "gated norm) + boundary + NVFP4 MoE; a 12-layer stage slice of such layers "
                                        "takes about 12 x this"}
    del layer, res_l, x_l, cst_l, rst_l
    torch.cuda.empty_cache()

    out["workload"] = (f"BASELINE config 3 attention pair: {T} tokens from {R} requests (new tokens lognormal median "
                       f"2k, cached prefixes 0-64k; KDA 32 x 128, DSA indexer 32 x 128 top-512 pools of 4, sparse MLA "
                       f"64 heads latent 512 + rope 64, FP8 e4m3 query and latent cache); mHC at T = 8192, H = 4096")
    return out




def run_moe_layer(args, rank: int, world: int, local: int) -> None:
    import torch

    from ssengine_b200 import lib

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    T = args.tokens
    layer, x = build_layer(device, T, rank)
    out = torch.empty_like(x)
    steps, warm = args.steps, max(3, args.warmup)
    for _ in range(warm):
        layer.forward(x, out)
    torch.cuda.synchronize()
    layer.check_status()

    # clocks: sample through ~1 s of the same work right before the timed region and through the timed region
    props = torch.cuda.get_device_properties(device)
    gpu_id = str(getattr(props, "uuid", local))
    gpu_id = gpu_id if gpu_id.startswith("GPU-") or not gpu_id.count("-") else "GPU-" + gpu_id
    clocks = Clocks(gpu_id)
    if not args.no_clocks:
        clocks.start()
        t_end = time.time() + 1.0
        while time.time() < t_end:
            layer.forward(x, out)
            torch.cuda.synchronize()

    nst = len(lib.MOE_STEPS)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nst + 1)] for _ in range(steps)]
    for row in evs:
        for e in row:
            e.record()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start.record()
    for i in range(steps):
        layer.forward_profiled(x, out, evs[i])
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if dist is not None:
        dist.barrier()
    layer.check_status()
    elapsed_ms = start.elapsed_time(end)
    per_kernel = {name: statistics.mean(evs[i][s].elapsed_time(evs[i][s + 1]) for i in range(steps))
                  for s, name in enumerate(lib.MOE_STEPS)}

    # e2e through the public API, host buffers: every step copies its input from pinned host memory to the device,
    # runs MoELayer.forward and reads its output back to pinned host memory; the steps are pipelined the way a serving
    # loop runs them (upload of step i + 1, compute of step i and read-back of step i - 1 on three streams, device
    # buffers double-buffered, PCIe full duplex), all inside the timed region
    e2e_ms = None
    if not args.no_e2e:
        xh = x.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        xd = [torch.empty_like(x), torch.empty_like(x)]
        od = [torch.empty_like(x), torch.empty_like(x)]
        s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event(), torch.cuda.Event()]
        ev_cmp = [torch.cuda.Event(), torch.cuda.Event()]
        ev_out = [torch.cuda.Event(), torch.cuda.Event()]

        def pipelined(n_steps: int) -> None:
            for i in range(n_steps):
                b = i & 1
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(ev_cmp[b])           # step i - 2 has finished reading xd[b]
                    xd[b].copy_(xh, non_blocking=True)
                    ev_in[b].record(s_in)
                s_cmp.wait_event(ev_in[b])
                if i >= 2:
                    s_cmp.wait_event(ev_out[b])              # step i - 2's output has left od[b]
                layer.forward(xd[b], out=od[b], stream=s_cmp)
                ev_cmp[b].record(s_cmp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_cmp[b])
                    oh.copy_(od[b], non_blocking=True)
                    ev_out[b].record(s_out)

        pipelined(warm)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        pipelined(steps)
        s_in.wait_stream(s_out)
        s_in.wait_stream(s_cmp)
        e1.record(s_in)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        layer.check_status()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    elapsed_ms = max_over_ranks(elapsed_ms)
    e2e_ms = max_over_ranks(e2e_ms) if e2e_ms is not None else None
    gate_ms = max_over_ranks(per_kernel["gate_up_gemm"])

    if rank == 0:
        pk, src = peaks()
        ms_step = elapsed_ms / steps
        value = world * T * steps / (elapsed_ms / 1e3)
        gate_flops = 2.0 * (T * K_TOP + T) * (2 * F) * H
        fp4_peak = 4.0 * pk["bf16_tflops"]
        achieved = gate_flops / (gate_ms / 1e3) / 1e12
        line = {
            "metric": "prefill tok/s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, ue4m3 per-16 scales, fp32 accumulate)",
            "data": "synthetic: hidden N(0,1) bf16, seeded random-init NVFP4 weights",
            "config": {"workload": workload(T), "global_batch": world * T, "seq_len": T,
                       "parallelism": f"replicas x{world}" if world > 1 else "single stage slice",
                       "l2": "inputs larger than L2 (0.9 GB of expert weights + 1 GB workspace per step)"},
            "roofline": {"kernel": "gate_up grouped NVFP4 GEMM (SwiGLU + requant epilogue)", "bound": "tensor",
                         "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s", "frac": achieved / fp4_peak,
                         "traffic": GATE_UP_TRAFFIC_T8192 if T == 8192 else None,
                         "traffic_unit": "bytes per launch (ncu capture)",
                         "peak_source": f"4 x {src} dense bf16 {pk['bf16_tflops']} TFLOP/s (B200 dense NVFP4 rate "
                                        f"is 4x bf16)",
                         "algorithmic": f"2 * {T * K_TOP + T} rows * {2 * F} * {H} = {gate_flops:.4e} FLOP/launch",
                         "layer_frac": layer_flops(T) / (ms_step / 1e3) / 1e12 / fp4_peak},
            "kernels_ms": {k: round(v, 5) for k, v in per_kernel.items()},
            "gpu_launches": steps * lib.MOE_KERNELS,
            "clocks": clk,
        }
        if e2e_ms is not None:
            line["e2e"] = {"value": world * T * steps / (e2e_ms / 1e3), "unit": "tok/s",
                           "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2,
                           "pipelining": "each step's upload, forward and read-back on 3 streams, overlapped with the "
                                         "neighbouring steps (device buffers double-buffered)"}
        if world == 1 and not args.no_components:
            line["components"] = time_components(device, pk)
        if world == 1 and not args.no_cpu_baseline:
            import numpy as np

            torch.set_num_threads(cpu_threads())
            p, dense = dense_on_host(layer)
            sample = min(max(args.cpu_tokens, 1024), T)
            x_np = x[:sample].float().cpu().numpy()
            time_oracle(p, dense, x_np[: min(64, sample)])
            sec = time_oracle(p, dense, x_np)
            line["cpu_baseline"] = {"value": sample / sec, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
                                    "sample": f"{sample} of the {T} tokens through oracle.moe.moe_forward (numpy "
                                              f"fp32, weights dequantized before timing), {sec:.2f} s"}
            del np
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()



def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import __graft_entry__

    __graft_entry__.import_package()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.impl == "vllm-cutlass":
        run_vllm_cutlass(args, rank)
        return
    if args.workload == "moe-layer":
        run_moe_layer(args, rank, world, local)
    elif args.workload == "components":
        import torch

        torch.cuda.set_device(local)
        pk, src = peaks()
        print(json.dumps({"components": time_components(torch.device("cuda", local), pk), "peaks": src}), flush=True)
    elif args.workload == "sessions":
        run_sessions(args, rank, world, local)
    else:
        run_pipeline(args, rank, world, local)


if __name__ == "__main__":
    main()
