"""`StageModel`: the reference's stage interface over the CUDA library (the drop-in boundary).

Mirrors ssengine/model/stage.py:216-762 of the reference and its contract in ssengine/runtime/README.md:72-100:
- construction `StageModel(cfg, stage, device, *, num_blocks=None, warmup=True, cuda_graphs=None, ipc_kv=False,
  extra_blocks=0)`, cfg a `StageConfig` or the reference's run config (`stage_settings`, stage.py:130-135); attributes `num_blocks` (counts the null block), `hidden_width`, `first`, `last`, `layer_range`;
- `prepare(plan) -> Batch`: host work only (no wait on queued GPU work): row order with decode-class chunks
  (<= 256 tokens) first, stably (ssengine/model/metadata.py:43,214), query start offsets, each request's KV pages,
  stage-0 token ids and the last stage's rows, packed into ONE pinned buffer and copied in stream order; the
  expanded metadata (positions, g0 slot mapping, kernel-block table) is then built on the device by
  `ssb_stage_metadata` (the reference expands it with numpy on the host, metadata.py:79-96);
- `run(batch, hidden_in)`: stage 0 embeds the token ids; the stage's layers run in order; stages 0..n-2 return
  [T, hidden_width] bf16 on the device, the last stage returns int64 greedy tokens, one per `is_last` chunk in plan
  chunk order; enqueues GPU work only, a fresh output per call;
- `forward(plan, hidden_in) = run(prepare(plan), hidden_in)`; `tier_ranges()`.

Layer kinds (`StageConfig.layer_kind`):
- "hybrid": the Glm5Next split, decoder layers on the 4-stream mHC residual, DSA + MoE at layers 3, 7, ..., KDA + MoE
  elsewhere (`layers.DsaDecoderLayer`, `layers.KdaDecoderLayer`: boundary, attention with NVFP4 projections,
  boundary, NVFP4 MoE); stage 0 expands its embeddings to 4 streams (hc_expand), a later stage starts with a
  pre-only boundary on the received [T, 4H] rows (edge_recv), a stage that is not the last ends with a post-only
  boundary (edge_send). The KV and state pages follow the reference's block layout (`kvpages.StageKv`): a DSA
  layer's latent rows and pool keys are addressed through the chunk's `kv_pages`, its kpool tail ring by
  `state_blocks[5]`; a KDA layer of state group g (its ordinal among the model's KDA layers, mod 5) keeps its conv and
  recurrent state in block `state_blocks[g]` of the latent tensor it aliases (has state = the chunk continues its
  request). With `dense_layers` > 0 the leading layers carry a dense SwiGLU FFN instead of the MoE (the reference
  model's layers 0-2); `routing` "sigmoid" selects the reference model's MoE routing.
- "kda": every layer KDA + MoE (no DSA layers).
- "moe": NVFP4 MoE layers with a plain residual (x + MoE(x)), hidden [T, H], no state (BASELINE config 2's slice).
The last stage's head: the mean of the 4 streams ("kda"), RMSNorm of each request's last row, BF16 lm_head GEMM
(fp32 logits), argmax (lowest index on ties).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import layout, lib, moe, weights

DECODE_THRESHOLD = 256
PAGE_TOKENS = 128
BLOCK_TOKENS = 8576
KERNEL_BLOCK = 64
GRAPH_BUCKETS = (128,) + tuple(range(256, 8192 + 1, 256))
PACK_ALIGN = 256


def row_order(num_tokens: list[int]) -> list[int]:
    """Chunk indices in row order: decode-class chunks (<= 256 tokens) first, stable (metadata.py:214)."""
    return sorted(range(len(num_tokens)), key=lambda i: num_tokens[i] > DECODE_THRESHOLD)


def graph_bucket(num_tokens: int, buckets=GRAPH_BUCKETS):
    """The smallest bucket that holds the microbatch, or None (stage.py:67-69)."""
    return next((b for b in sorted(buckets) if b >= num_tokens), None)


def table_width(blocks: int, page_tokens: int = PAGE_TOKENS, block_tokens: int = BLOCK_TOKENS) -> int:
    """Kernel-block columns of the g0 table: the longest request's blocks rounded up to a power of two
    (metadata.py:181-189, without vLLM's full-width cap)."""
    per_block = block_tokens // KERNEL_BLOCK
    return (1 << max(blocks - 1, 0).bit_length()) * per_block


def check_blocks(chunks, num_blocks: int, kv_pages=None) -> None:
    """The block contract the state pages rely on (ssengine/model/kv_tensors.py:1-14: a block holds a request's KV
    pages or one of its states, never both): every non-null state block of the plan belongs to one (request, group)
    only and is no request's KV block; blocks within the pool. Block 0 is the null block (a dummy request may use it
    for every state). `kv_pages`: the chunks' KV page ids as int64 arrays, when the caller has them. Raises
    ValueError."""
    seen = {}
    for c in chunks:
        if len(c.state_blocks) < 6:
            raise ValueError(f"chunk {c.req_id}: {len(c.state_blocks)} state blocks (6 needed)")
        for g, b in enumerate(c.state_blocks[:6]):
            b = int(b)
            if not 0 <= b < num_blocks:
                raise ValueError(f"chunk {c.req_id}: state block {b} outside the pool of {num_blocks}")
            if b == 0:
                continue
            if b in seen and seen[b] != (c.req_id, g):
                raise ValueError(f"state block {b} held twice: {seen[b]} and {(c.req_id, g)}")
            seen[b] = (c.req_id, g)
    if not seen:
        return
    if kv_pages is None:
        kv_pages = [np.asarray(c.kv_pages, dtype=np.int64).reshape(-1) for c in chunks]
    pages = np.concatenate(kv_pages)
    both = np.intersect1d(pages // (BLOCK_TOKENS // PAGE_TOKENS), np.fromiter(seen, np.int64, len(seen)))
    if both.size:
        raise ValueError(f"blocks {both[:8].tolist()} are both KV and state blocks")


@dataclass
class StageConfig:
    """What a stage reads of the run config (the reference's RunConfig fields `layer_split`, `scheduler.mb_tokens`,
    `cuda_graphs`, plus the model dimensions the random-init weights need)."""
    layer_split: tuple = (2,)
    hidden: int = 4096
    inter: int = 1024
    experts: int = 128
    top_k: int = 8
    vocab: int = 151_552
    mb_tokens: int = 8192
    cuda_graphs: bool = False
    num_blocks: int = 64
    seed: int = 0
    norm_eps: float = 1e-5
    layer_kind: str = "moe"            # "moe": residual NVFP4 MoE layers, hidden [T, H]; "kda": KDA + MoE decoder
                                       # layers on the 4-stream mHC residual, hidden [T, 4H] across stage edges;
                                       # "hybrid": as "kda" with every 4th layer (3, 7, ...) a DSA + MoE layer
    kda_heads: int = 64
    q_lora: int = 1536
    mla_nope: int = 192
    mla_v_dim: int = 256
    dense_layers: int = 0              # leading layers with a dense SwiGLU FFN instead of the MoE (the reference model:
                                       # 3, `first_kda_dense` / `kda_dense`, ssengine/kernels.py:283-289)
    dense_inter: int = 12288           # their intermediate size (gate_up 4096 -> 2 x 12288)
    routing: str = "softmax"           # MoE routing: "softmax" or "sigmoid" (the reference model:
                                       # sigmoid + correction bias, routed scale 5/2)
    n_group: int = 1
    topk_group: int = 1
    weight_init: str = "uniform"       # NVFP4 weights: "uniform" (codes uniform, scales
                                       # log-uniform) or "normal" (N(0, init_std) quantized)
    init_std: float = 0.02
    max_context: int = 131_072         # the longest context a request reaches (sizes the indexer's logits buffer)
    reserve_reqs: int = 64             # requests per microbatch the KDA chunk workspace is reserved for
    indexer_fp8: bool = False          # the FP8 indexer over the reference's 132-byte pool entries (its kernels
                                       # validated, the whole stage not yet; the bf16 indexer by default)


@dataclass
class Batch:
    num_tokens: int
    order: list[int]                   # plan chunk indices in row order
    positions: torch.Tensor            # int64 [bucket or T], device
    slots: torch.Tensor                # int64 [bucket or T], device (pad rows -1)
    table: torch.Tensor                # int32 [R, width], device (g0 kernel-block table)
    token_ids: torch.Tensor | None     # int64 [T], device (stage 0)
    last_rows: torch.Tensor            # int64 [#is_last], rows whose token the last stage returns, plan chunk order
    bucket: int | None = None
    keep: list = field(default_factory=list)   # host / device buffers that must outlive the queued work
    kda_seqs: torch.Tensor | None = None       # int32 [5, R, 4] per KDA state group g2..g6: {first row, end row,
                                               # state_blocks[g], has state}, device
    dsa: dict | None = None                    # DSA layers' metadata (positions, slots, qsl, page table, kpool, groups)
    tier_ops: list = field(default_factory=list)   # the plan's DRAM tier copies, applied before its forward


class _Pack:
    """Arrays of one microbatch in one pinned host buffer, copied to the device with one stream-ordered copy."""

    def __init__(self):
        self.items, self.size = [], 0

    def add(self, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        off = -(-self.size // PACK_ALIGN) * PACK_ALIGN
        self.items.append((off, a))
        self.size = off + a.nbytes
        return len(self.items) - 1

    def copy(self, device) -> tuple[torch.Tensor, torch.Tensor]:
        host = torch.empty(max(self.size, 8), dtype=torch.uint8, pin_memory=True)
        hv = host.numpy()
        for off, a in self.items:
            hv[off:off + a.nbytes] = a.reshape(-1).view(np.uint8)
        return host, host.to(device, non_blocking=True)

    def view(self, dev: torch.Tensor, h: int, dtype: torch.dtype) -> torch.Tensor:
        off, a = self.items[h]
        return dev[off:off + a.nbytes].view(dtype).view(a.shape)


def kda_tables(chunks, order, qsl) -> np.ndarray:
    """int32 [5, R, 4]: one sequence table per KDA state group g2..g6, a row per chunk = {first row, end row, the
    chunk's state_blocks[g], has state (the chunk continues its request)}. `order`: the chunks in row order, `qsl`
    their row starts (R + 1). Rows longest first: the scan runs one CTA per (sequence, head, value half) in table
    order, so the longest sequences start first (an LPT order, in the place of the reference's head-split plan,
    ssengine/native/kda_split_heads.cpp:17-91); each sequence's result does not depend on its place in the table."""
    R = len(order)
    qsl = np.asarray(qsl, np.int64)
    lpt = np.argsort(-np.diff(qsl), kind="stable")                     # ties keep row order
    blocks = np.array([chunks[i].state_blocks[:5] for i in order], np.int64).reshape(R, 5)
    cont = np.array([chunks[i].start > 0 for i in order], np.int64)
    out = np.empty((5, R, 4), np.int32)
    out[:, :, 0], out[:, :, 1] = qsl[lpt], qsl[lpt + 1]
    out[:, :, 2], out[:, :, 3] = blocks[lpt].T, cont[lpt]
    return out


# The reference model's dimensions, as its op manifest states them (ssengine/kernels.py:109-121 dense FFN, :174-191
# router and MoE: 288 experts, top 8, intermediate 2048, sigmoid + correction bias with routed scale 5/2, :277 split):
# what a stage built from the reference's own run config gets, with random-init weights of that architecture
REFERENCE_MODEL = dict(hidden=4096, inter=2048, experts=288, top_k=8, vocab=151_552, kda_heads=64, q_lora=1536,
                       mla_nope=192, mla_v_dim=256, dense_layers=3, dense_inter=12288, routing="sigmoid",
                       layer_kind="hybrid")


def stage_settings(cfg) -> StageConfig:
    """The `StageConfig` of a run config. A `StageConfig` is returned as it is. Anything else is read as the
    reference's `RunConfig` (or a bench's namespace with its fields) the way the reference's `stage_settings` reads
    it (ssengine/model/stage.py:130-135): `layer_split`, `checkpoint`, `scheduler.mb_tokens`, `pool_tokens`,
    `cuda_graphs`, each read directly, so that a missing field raises here. The model is `REFERENCE_MODEL` with
    random-init weights: a checkpoint path raises (this library loads no weights). The workspaces are sized for
    max(mb_tokens, 8192) rows, as the reference sizes its stage; `pool_tokens` gives the KV blocks (rounded up to
    whole 8,576-token blocks, plus the null block), else `StageConfig`'s default."""
    if isinstance(cfg, StageConfig):
        return cfg
    split, ckpt = tuple(int(n) for n in cfg.layer_split), cfg.checkpoint
    mb, pool, graphs = int(cfg.scheduler.mb_tokens), cfg.pool_tokens, bool(cfg.cuda_graphs)
    if ckpt:
        raise ValueError(f"checkpoint {ckpt!r}: this library builds random-init weights and loads none")
    blocks = {} if pool is None else {"num_blocks": -(-int(pool) // BLOCK_TOKENS) + 1}
    return StageConfig(layer_split=split, mb_tokens=max(mb, 8192), cuda_graphs=graphs, **blocks, **REFERENCE_MODEL)


def bench_config(mb_tokens: int, checkpoint: str | None = None, cuda_graphs: bool = False, split=(12, 11, 11, 11)):
    """A run-config stand-in with the fields `stage_settings` reads (the reference's `bench_config`,
    ssengine/model/stage.py:138-144), for benches and tests."""
    from types import SimpleNamespace

    return SimpleNamespace(layer_split=list(split), checkpoint=checkpoint, pool_tokens=None,
                           scheduler=SimpleNamespace(mb_tokens=mb_tokens), cuda_graphs=cuda_graphs)


class StageModel:
    def __init__(self, cfg, stage: int, device, *, num_blocks: int | None = None, warmup: bool = True,
                 cuda_graphs: bool | None = None, ipc_kv: bool = False, extra_blocks: int = 0):
        """cfg: a `StageConfig`, or the reference's run config (read by `stage_settings`)."""
        cfg = stage_settings(cfg)
        self.cfg, self.stage = cfg, stage
        self.device = torch.device(device)
        split = list(cfg.layer_split)
        if not 0 <= stage < len(split):
            raise ValueError(f"stage {stage} outside the split {split}")
        self.first, self.last = stage == 0, stage == len(split) - 1
        start = sum(split[:stage])
        self.layer_range = range(start, start + split[stage])
        self.kda = cfg.layer_kind in ("kda", "hybrid")
        if cfg.layer_kind not in ("moe", "kda", "hybrid"):
            raise ValueError(f"layer_kind {cfg.layer_kind!r}")
        self.is_dsa = [self.layer_is_dsa(i) for i in self.layer_range]
        self.hidden_width = 4 * cfg.hidden if self.kda else cfg.hidden
        self.num_blocks = (num_blocks if num_blocks is not None else cfg.num_blocks) + extra_blocks
        self.cuda_graphs = cfg.cuda_graphs if cuda_graphs is None else cuda_graphs
        self.ipc_kv = ipc_kv
        self.layer_hook = None          # optional callable(layer, res, x_prev, post, comb) after each layer (checks)
        self.moe_profile = None         # optional list: each MoE layer's forward records per-step CUDA events into it
        self._lib = lib.load()
        H, F, E = cfg.hidden, cfg.inter, cfg.experts
        if self.kda:
            from .kvpages import StageKv
            from .layers import DsaDecoderLayer, KdaDecoderLayer

            # KV and state pages in the reference's block layout: KDA group g2..g6 states alias the DSA layers'
            # latent blocks (kvpages.StageKv)
            self.kv = StageKv(list(self.layer_range), self.layer_is_dsa, self.num_blocks, cfg.kda_heads, self.device,
                              pool_fp8=cfg.indexer_fp8)
            route = None if cfg.routing == "softmax" else dict(routing=cfg.routing, n_group=cfg.n_group,
                                                               topk_group=cfg.topk_group)
            self.layers, self.kda_states, self.kda_group = [], [], []
            for i, dsa in zip(self.layer_range, self.is_dsa):
                seed = cfg.seed * 1000 + 10 * i
                dense = i < cfg.dense_layers
                ffn = dict(ffn="dense" if dense else "moe", routing=route, init=cfg.weight_init, std=cfg.init_std)
                inter = cfg.dense_inter if dense else F
                if dsa:
                    self.layers.append(DsaDecoderLayer(seed, H, inter, E, cfg.top_k, self.device, q_lora=cfg.q_lora,
                                                       nope=cfg.mla_nope, v_dim=cfg.mla_v_dim,
                                                       indexer_fp8=cfg.indexer_fp8, **ffn))
                    # latent cache e4m3 [slots, 576], pool-key cache [pages * 32, 128], tail ring [blocks, 2, 4, 128]
                    self.kda_states.append((self.kv.latent(i), self.kv.pool_keys(i), self.kv.tail_ring(i)))
                    self.kda_group.append(None)
                else:
                    self.layers.append(KdaDecoderLayer(seed, H, cfg.kda_heads, inter, E, cfg.top_k, self.device,
                                                       **ffn))
                    # KDA conv state [blocks, 3, 3P] bf16 and recurrent state [blocks, heads, 128, 128] fp32, views
                    # into the aliased latent pages
                    self.kda_states.append((self.kv.conv_state(i), self.kv.rec_state(i)))
                    self.kda_group.append(self.kv.group[i])
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        else:
            self.layers = [moe.MoELayer.from_logical(weights.moe_logical(cfg.seed * 1000 + i, H, F, E,
                                                                         device=self.device),
                                                     cfg.top_k, self.device, add_input=True) for i in self.layer_range]
        if self.first:
            g = torch.Generator(device=self.device)
            g.manual_seed(cfg.seed * 1000 + 999)
            self.embed = torch.randn(cfg.vocab, H, generator=g, device=self.device).to(torch.bfloat16)
        if self.last:
            self._init_head()
        if warmup:
            self._warm()

    def layer_is_dsa(self, i: int) -> bool:
        """Model layer i is a DSA layer: layers 3, 7, ..., 43 of the hybrid interleave (ssengine/kernels.py:278)."""
        return self.cfg.layer_kind == "hybrid" and i % 4 == 3

    # ---------------------------------------------------------------- construction helpers
    def _init_head(self) -> None:
        """The lm_head in BF16, as the reference keeps it (ssengine/kernels.py:203-205, config 35: BF16 `F.linear` on
        the finished rows; its NVFP4 GEMMs are the dense FFN and the experts): weights N(0, 1 / H) for unit-variance
        logits ("uniform" recipe) or N(0, init_std) ("normal")."""
        cfg, H, V = self.cfg, self.cfg.hidden, self.cfg.vocab
        g = torch.Generator(device=self.device)
        g.manual_seed(cfg.seed * 1000 + 998)
        std = cfg.init_std if cfg.weight_init == "normal" else H ** -0.5
        self.head_w = (torch.randn(V, H, generator=g, device=self.device) * std).to(torch.bfloat16)
        self.norm_weight = torch.ones(H, dtype=torch.bfloat16, device=self.device)

    def _warm(self) -> None:
        """Reserves the device memory a microbatch needs, so that no forward maps new memory (a cudaMalloc inside a
        forward stalls the host for up to tens of milliseconds while the GPU drains its queue): the indexer's logits
        rows at `max_context` (one buffer the stage's DSA layers share; they run in order on one stream), the KDA /
        mHC chunk workspace for `reserve_reqs` requests, and one forward of a dummy request of a full microbatch
        (written into the null block's pages and state) that loads every kernel and leaves its temporaries in the
        caching allocator for the next microbatches; then the MoE layers' shared workspace."""
        from .messages import Chunk, Plan

        cfg = self.cfg
        if any(self.is_dsa):
            from .layers import DsaAttention

            width = -(-(-(-cfg.max_context // PAGE_TOKENS) * DsaAttention.POOLS_PER_PAGE) // 128) * 128
            logits_ws = torch.empty(cfg.mb_tokens * width, dtype=torch.float32, device=self.device)
            for layer, dsa in zip(self.layers, self.is_dsa):
                if dsa:
                    layer.attn.logits_ws = logits_ws
        if self.kda:
            from . import kda

            lib.scratch(self.device, max(kda.workspace_bytes(cfg.kda_heads, cfg.mb_tokens, cfg.reserve_reqs),
                                         int(self._lib.ssb_mhc_workspace_bytes(cfg.mb_tokens))))
        n = min(cfg.mb_tokens, (BLOCK_TOKENS // PAGE_TOKENS - 1) * PAGE_TOKENS)
        pages = list(range(1, -(-n // PAGE_TOKENS) + 1))
        plan = Plan(-1, [Chunk("warmup", 0, n, pages, [0] * 6, True, [0] * n if self.first else None)])
        hidden = None if self.first else torch.zeros(n, self.hidden_width, dtype=torch.bfloat16, device=self.device)
        self.forward(plan, hidden)
        moes = [layer.moe if self.kda else layer for layer in self.layers]
        moes = [m for m in moes if isinstance(m, moe.MoELayer)]
        ws = max(m.workspace_bytes(self.cfg.mb_tokens) for m in moes) if moes else 0
        shared = torch.empty(ws, dtype=torch.uint8, device=self.device) if ws else None
        for m in moes:
            m._ws = shared
        torch.cuda.synchronize(self.device)

    # ---------------------------------------------------------------- the interface
    def tier_ranges(self) -> list:
        """This stage's cache views as `kvpages.ViewRange`s (the reference's `StageModel.tier_ranges`,
        ssengine/model/stage.py:710): what a tier mover copies for a KV block or a request's state blocks. Empty for
        the MoE-only stage kind, which holds no KV."""
        return self.kv.tier_ranges(self.stage) if self.kda else []

    def prepare(self, plan) -> Batch:
        chunks = plan.chunks
        order = row_order([c.num_tokens for c in chunks])
        R = len(order)
        q_lens = np.array([chunks[i].num_tokens for i in order], dtype=np.int64)
        starts = np.array([chunks[i].start for i in order], dtype=np.int64)
        qsl = np.zeros(R + 1, dtype=np.int64)
        np.cumsum(q_lens, out=qsl[1:])
        T = int(qsl[-1])
        seq = starts + q_lens
        need = -(-seq // PAGE_TOKENS)
        full = [np.asarray(c.kv_pages, dtype=np.int64).reshape(-1) for c in chunks]    # plan order, converted once
        page_lists = []
        for r, i in enumerate(order):
            pg = full[i]
            if len(pg) < need[r]:
                raise ValueError(f"chunk {chunks[i].req_id}: {len(pg)} KV pages for {int(seq[r])} tokens")
            page_lists.append(pg[: need[r]])
        page_ptr = np.zeros(R + 1, dtype=np.int64)
        np.cumsum([len(p) for p in page_lists], out=page_ptr[1:])
        pages = np.concatenate(page_lists) if page_lists else np.zeros(0, dtype=np.int64)
        if pages.size and (pages.max() >= 2 ** 31 or pages.min() < 0):
            raise ValueError("page id outside int32")
        row_end = {i: int(qsl[r + 1]) - 1 for r, i in enumerate(order)}
        last = np.array([row_end[i] for i, c in enumerate(chunks) if c.is_last], dtype=np.int64)
        bucket = graph_bucket(T) if self.cuda_graphs else None
        width = table_width(int(max((-(-int(s) // BLOCK_TOKENS) for s in seq), default=1)))

        pk = _Pack()
        h = {"qsl": pk.add(qsl.astype(np.int32)), "starts": pk.add(starts.astype(np.int32)),
             "page_ptr": pk.add(page_ptr.astype(np.int32)), "pages": pk.add(np.maximum(pages, 0).astype(np.int32)),
             "last": pk.add(last)}
        if self.kda:
            check_blocks(chunks, self.num_blocks, full)
            h["kda"] = pk.add(kda_tables(chunks, order, qsl))
        if any(self.is_dsa):
            from .indexer import work_groups

            wp = max(1, max((len(p) for p in page_lists), default=1))
            ptab = np.full((max(R, 1), wp), -1, dtype=np.int32)
            n_pg = np.diff(page_ptr)
            ptab[np.repeat(np.arange(R), n_pg), np.arange(pages.size) - np.repeat(page_ptr[:-1], n_pg)] = pages
            tails = np.array([chunks[i].state_blocks[5] for i in order], np.int64)
            kreq = np.stack([qsl[:-1], q_lens, starts, tails], axis=1).astype(np.int32).reshape(-1, 4)
            grp = work_groups(qsl[:-1], q_lens, starts)
            h["dsa_qsl"] = pk.add(qsl.astype(np.int32))
            h["dsa_pages"] = pk.add(ptab)
            h["dsa_kreq"] = pk.add(kreq)
            h["dsa_groups"] = pk.add(grp if grp.size else np.zeros((1, 4), np.int32))
            dsa_max_rows, dsa_ng = int(q_lens.max()) if R else 0, int(grp.shape[0])
        if self.first:
            tok = np.concatenate([np.asarray(chunks[i].token_ids, dtype=np.int64) for i in order]) if R else \
                np.zeros(0, dtype=np.int64)
            if tok.shape[0] != T:
                raise ValueError(f"stage 0 needs every chunk's token ids ({tok.shape[0]} for {T} rows)")
            h["tok"] = pk.add(tok)
        host, dev = pk.copy(self.device)
        rows_out = bucket if bucket is not None else T
        positions = torch.empty(max(rows_out, 1), dtype=torch.int64, device=self.device)
        slots = torch.empty(max(rows_out, 1), dtype=torch.int64, device=self.device)
        table = torch.empty(max(R * width, 1), dtype=torch.int32, device=self.device)
        v = {k: pk.view(dev, i, torch.int64 if k in ("last", "tok") else torch.int32) for k, i in h.items()}
        rc = self._lib.ssb_stage_metadata(v["qsl"].data_ptr(), v["starts"].data_ptr(), v["page_ptr"].data_ptr(),
                                          v["pages"].data_ptr(), R, T, rows_out, PAGE_TOKENS, width,
                                          positions.data_ptr(), slots.data_ptr(), table.data_ptr(), lib.stream_ptr())
        lib.check("ssb_stage_metadata", rc)
        dsa = None
        if any(self.is_dsa):
            dsa = dict(positions=positions[:T], slots=slots[:T], qsl=v["dsa_qsl"], page_table=v["dsa_pages"],
                       kpool_reqs=v["dsa_kreq"], max_rows=dsa_max_rows, groups=v["dsa_groups"][:dsa_ng])
        return Batch(T, order, positions[:rows_out], slots[:rows_out], table[: R * width].view(R, width),
                     v.get("tok"), v["last"], bucket, keep=[host, dev], kda_seqs=v.get("kda"), dsa=dsa,
                     tier_ops=list(getattr(plan, "tier_ops", None) or []))

    def run(self, batch: Batch, hidden_in: torch.Tensor | None, edge_out=None) -> torch.Tensor | None:
        """edge_out: a device address, or a callable returning one when called right before the last kernel (the
        next stage's receive slot, a peer pointer), into which a non-last hybrid stage's final boundary kernel stores
        its [T, 4H] rows directly (the fused stage edge); the call then returns None. Without it the rows come back as
        a fresh tensor (the reference's contract)."""
        if self.kda:
            return self._run_kda(batch, hidden_in, edge_out)
        T, H = batch.num_tokens, self.hidden_width
        s = lib.stream_ptr()
        if self.first:
            x = torch.empty(T, H, dtype=torch.bfloat16, device=self.device)
            lib.check("ssb_embed_rows", self._lib.ssb_embed_rows(self.embed.data_ptr(), self.cfg.vocab, H,
                                                                 batch.token_ids.data_ptr(), T, x.data_ptr(), s))
        else:
            if hidden_in is None or tuple(hidden_in.shape) != (T, H) or hidden_in.dtype != torch.bfloat16:
                raise ValueError(f"stage {self.stage} needs hidden_in bf16 [{T}, {H}]")
            x = hidden_in
        for layer in self.layers:
            x = layer.forward(x, out=torch.empty(T, H, dtype=torch.bfloat16, device=self.device))
        if not self.last:
            return x
        return self._head(x, batch.last_rows)

    def _run_kda(self, batch: Batch, hidden_in: torch.Tensor | None, edge_out=None):
        """KDA + MoE decoder layers on the 4-stream residual: stage 0 expands its embeddings (hc_expand), a later stage
        starts from the received residual with a pre-only boundary (edge_recv); a stage that is not the last ends with
        a post-only boundary into the [T, 4H] rows it sends (edge_send, ssengine/model/pp_patch.py:156-163); the last
        stage folds the final MoE rows in, averages the streams of the returned rows and runs the head."""
        T, H = batch.num_tokens, self.cfg.hidden
        s = lib.stream_ptr()
        if self.first:
            x = torch.empty(T, H, dtype=torch.bfloat16, device=self.device)
            lib.check("ssb_embed_rows", self._lib.ssb_embed_rows(self.embed.data_ptr(), self.cfg.vocab, H,
                                                                 batch.token_ids.data_ptr(), T, x.data_ptr(), s))
            res = torch.empty(T, 4, H, dtype=torch.bfloat16, device=self.device)
            lib.check("ssb_hc_expand", self._lib.ssb_hc_expand(x.data_ptr(), T, H, res.data_ptr(), s))
        else:
            if hidden_in is None or tuple(hidden_in.shape) != (T, 4 * H) or hidden_in.dtype != torch.bfloat16:
                raise ValueError(f"stage {self.stage} needs hidden_in bf16 [{T}, {4 * H}]")
            res = hidden_in.view(T, 4, H)
        x_prev = post = comb = None
        for layer in self.layers:
            layer.moe_profile = self.moe_profile
        for layer, state, dsa, grp in zip(self.layers, self.kda_states, self.is_dsa, self.kda_group):
            if dsa:
                res, x_prev, post, comb = layer.forward(res, x_prev, post, comb, batch.dsa, state, self.status)
            else:
                res, x_prev, post, comb = layer.forward(res, x_prev, post, comb, batch.kda_seqs[grp], *state,
                                                        self.status)
            if self.layer_hook is not None:
                self.layer_hook(layer, res, x_prev, post, comb)
        if edge_out is not None and not self.last and x_prev is not None:
            dst = edge_out() if callable(edge_out) else edge_out
            self._edge_post(x_prev, res, post, comb, dst)              # straight into the peer's receive slot
            return None
        out = torch.empty(T, 4, H, dtype=torch.bfloat16, device=self.device)
        if x_prev is None:
            out.copy_(res)
        else:
            self._edge_post(x_prev, res, post, comb, out.data_ptr())
        if not self.last:
            return out.view(T, 4 * H)
        n = batch.last_rows.shape[0]
        merged = torch.empty(max(n, 1), H, dtype=torch.bfloat16, device=self.device)
        lib.check("ssb_hc_mean", self._lib.ssb_hc_mean(out.data_ptr(), H, batch.last_rows.data_ptr(), n,
                                                       merged.data_ptr(), s))
        return self._head(merged[:n], torch.arange(n, dtype=torch.int64, device=self.device))

    def _edge_post(self, x, res, post, comb, out_ptr: int) -> None:
        """Post-only boundary: out = post * x + comb^T res (the last sub-block's rows folded into the residual), stored
        at device address out_ptr ([T, 4, H] bf16)."""
        b = self.layers[-1].bound_b
        rc = self._lib.ssb_mhc(ctypes.byref(b._c), x.data_ptr(), res.data_ptr(), post.data_ptr(), comb.data_ptr(),
                               out_ptr, None, None, None, res.shape[0], lib.stream_ptr())
        lib.check("ssb_mhc", rc)

    def forward(self, plan, hidden_in: torch.Tensor | None = None) -> torch.Tensor:
        return self.run(self.prepare(plan), hidden_in)

    def tier_ranges(self) -> list:
        """Byte ranges (device pointer, bytes) of the stage's KV and state tensors for the capacity tiers: every
        latent / state page tensor, pool-key cache and tail ring (none for MoE-only stages)."""
        if not self.kda:
            return []
        return self.kv.ranges()

    # ---------------------------------------------------------------- last stage
    def _head(self, x: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
        n, H, V = rows.shape[0], self.cfg.hidden, self.cfg.vocab
        tokens = torch.empty(n, dtype=torch.int64, device=self.device)
        if n == 0:
            return tokens
        s = lib.stream_ptr()
        y = torch.empty(n, H, dtype=torch.bfloat16, device=self.device)
        lib.check("ssb_rmsnorm", self._lib.ssb_rmsnorm(x.data_ptr(), H, rows.data_ptr(), n, self.norm_weight.data_ptr(),
                                                       self.cfg.norm_eps, y.data_ptr(), s))
        # BF16 x BF16 -> fp32 logits of the finished rows: a plain library GEMM (cuBLAS through torch.mm), like the
        # reference's lm_head call
        logits = torch.mm(y, self.head_w.t(), out_dtype=torch.float32)
        lib.check("ssb_argmax_rows", self._lib.ssb_argmax_rows(logits.data_ptr(), V, V, n, tokens.data_ptr(), s))
        self.last_logits, self.last_normed = logits, y
        return tokens
