"""A stage's KV and state pages in the reference's block layout (ssengine/model/kv_tensors.py:1-14, 33-37, 157-196).

The controller hands out block ids from one space; block 0 is the null block. A block is 8,576 tokens of DSA KV or
one KDA layer's recurrent + conv state. Groups (vLLM's GLM-5 hybrid grouping, as the reference binds it):
- g0: the DSA layers' latent (MLA) rows and indexer pool keys, addressed through the chunk's KV pages (128 tokens;
  page p = page p % 67 of block p // 67);
- g1: the kpool tail ring, one block per request: `state_blocks[5]`;
- g2..g6: five KDA state groups, one block per request each: `state_blocks[0..4]`. A KDA layer's group is its
  ordinal among the model's KDA layers modulo 5 (the reference's known answer: group 0 holds layers 0, 6, 13, 20, 26,
  33, 40 -- tests/test_model_cpu.py:147-160 of the reference).
On a stage, the i-th KDA layer of group g ALIASES the i-th DSA layer's latent region: its state for a request lives in
block `state_blocks[g]` of that DSA layer's latent tensor (a block id held as a state block is never a KV block of
another request, so the two uses never meet). Inside such a block: the conv state [3, 3P] bf16 at offset 0, then the
recurrent state [H, 128, 128] fp32 (vLLM's Mamba-style state page: states in spec order, the page padded to the
latent block's size).

Differences from the reference, by necessity or choice (stated where they live):
- latent rows are 576 bytes (e4m3 latent 512 + rope 64, BASELINE's DSA dims) at slot * 576 of the layer's latent
  tensor (the reference's fork stores 512 bytes a token);
- the pool-key cache keeps bf16 rows of 128 (256 bytes) in pages of 32 pools (the reference: FP8 + scale, 132 bytes;
  `StageKv(pool_fp8=True)` lays the pages out that way, 33 rows of 128 bytes a page, for the FP8 indexer kernels);
- the tail ring is its own [blocks, 2, 4, 128] bf16 tensor per DSA layer, indexed by `state_blocks[5]` (the
  reference aliases it into the indexer region).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

BLOCK_TOKENS = 8576
PAGE_TOKENS = 128
PAGES_PER_BLOCK = BLOCK_TOKENS // PAGE_TOKENS          # 67
LATENT_ROW = 576                                        # e4m3 bytes per token: latent 512 + rope 64
POOL_ROW = 128                                          # bf16 pool key
KDA_GROUPS = 5
TAIL_STATE = 5                                          # state_blocks[5]: the kpool tail ring
STATE_ALIGN = 256


def kda_group(layer: int, is_dsa) -> int:
    """The KDA state group (0..4 = g2..g6) of model layer `layer`: its ordinal among the KDA layers, modulo 5.
    `is_dsa(i)` tells whether layer i is a DSA layer."""
    ordinal = sum(1 for i in range(layer) if not is_dsa(i))
    return ordinal % KDA_GROUPS


def kda_state_bytes(heads: int) -> tuple[int, int, int]:
    """(conv bytes, offset of the recurrent state, page bytes) of one KDA layer's state block."""
    P = heads * 128
    conv = 3 * 3 * P * 2
    rec_off = -(-conv // STATE_ALIGN) * STATE_ALIGN
    rec = heads * 128 * 128 * 4
    return conv, rec_off, -(-(rec_off + rec) // STATE_ALIGN) * STATE_ALIGN


def _latent_slots(layers, is_dsa) -> tuple[list, dict, dict, int]:
    """(DSA layers, KDA group per KDA layer, slot per KDA layer, block-sized tensors needed) of a stage."""
    dsa = [i for i in layers if is_dsa(i)]
    group, slot, seen = {}, {}, [0] * KDA_GROUPS
    for i in layers:
        if not is_dsa(i):
            g = kda_group(i, is_dsa)
            group[i], slot[i] = g, seen[g]
            seen[g] += 1
    return dsa, group, slot, max([len(dsa)] + [s + 1 for s in slot.values()])


POOL_PAGE_BYTES = 32 * POOL_ROW * 2                    # bf16 pool keys of one 128-token page
POOL_PAGE_BYTES_FP8 = 33 * 128                          # the reference's 32 entries of 132 bytes (codes, then scales)


def block_bytes(layers, is_dsa, kda_heads: int, pool_fp8: bool = False) -> int:
    """Device bytes one block id costs a stage holding `layers`: the latent (or state-only) block of every slot, plus
    each DSA layer's pool-key pages and tail ring for that block."""
    dsa, _, _, n_slots = _latent_slots(layers, is_dsa)
    state_page = kda_state_bytes(kda_heads)[2]
    latent_page = BLOCK_TOKENS * LATENT_ROW
    pages = sum(latent_page if j < len(dsa) else state_page for j in range(n_slots))
    pool = POOL_PAGE_BYTES_FP8 if pool_fp8 else POOL_PAGE_BYTES
    return pages + len(dsa) * (PAGES_PER_BLOCK * pool + 2 * 4 * POOL_ROW * 2)


class StageKv:
    """The pages of one stage's layers `layers` (model layer ids; `is_dsa(i)` for the kind) over `num_blocks` blocks.

    Per local DSA layer j: `latent[j]` uint8 [num_blocks, BLOCK_TOKENS * 576] (rows at slot * 576), `pool[j]` bf16
    [num_blocks * 67 * 32, 128], `tail[j]` bf16 [num_blocks, 2, 4, 128]. Per local KDA layer: (group, slot) where slot
    is the index of the latent tensor its state aliases (extra state-only tensors when the stage has fewer DSA layers
    than a group has KDA layers here)."""

    def __init__(self, layers, is_dsa, num_blocks: int, kda_heads: int, device, pin: bool = False,
                 pool_fp8: bool = False):
        dev = torch.device(device)
        self.device = dev
        self.num_blocks = num_blocks
        self.kda_heads = kda_heads
        self.layers, self.is_dsa = list(layers), is_dsa
        mem = dict(pin_memory=True) if pin else {}       # a host-memory copy of the views (the DRAM tier)
        self.conv_bytes, self.rec_off, state_page = kda_state_bytes(kda_heads)
        self.dsa_layers, self.group, self.slot, n_slots = _latent_slots(layers, is_dsa)
        self.kda_layers = [i for i in layers if not is_dsa(i)]
        latent_page = BLOCK_TOKENS * LATENT_ROW
        if self.kda_layers and self.dsa_layers and state_page > latent_page:
            raise ValueError(f"a KDA state page ({state_page} B) does not fit a latent block ({latent_page} B)")
        self.pages = []
        for j in range(n_slots):
            page = latent_page if j < len(self.dsa_layers) else state_page
            self.pages.append(torch.zeros(num_blocks, page, dtype=torch.uint8, device=dev, **mem))
        self.pool_fp8 = pool_fp8
        if pool_fp8:       # the reference's indexer pages: 33 rows of 128 bytes a page (32 code rows, the scales)
            self.pool = [torch.zeros(num_blocks * PAGES_PER_BLOCK * 33, 128, dtype=torch.uint8, device=dev, **mem)
                         for _ in self.dsa_layers]
        else:
            self.pool = [torch.zeros(num_blocks * PAGES_PER_BLOCK * 32, POOL_ROW, dtype=torch.bfloat16, device=dev,
                                     **mem) for _ in self.dsa_layers]
        self.tail = [torch.zeros(num_blocks, 2, 4, POOL_ROW, dtype=torch.bfloat16, device=dev, **mem)
                     for _ in self.dsa_layers]

    # ------------------------------------------------------------------ views
    def latent(self, layer: int) -> torch.Tensor:
        """uint8 [num_blocks * BLOCK_TOKENS, 576]: the DSA layer's latent rows by slot."""
        j = self.dsa_layers.index(layer)
        return self.pages[j].view(self.num_blocks * BLOCK_TOKENS, LATENT_ROW)

    def pool_keys(self, layer: int) -> torch.Tensor:
        return self.pool[self.dsa_layers.index(layer)]

    def tail_ring(self, layer: int) -> torch.Tensor:
        return self.tail[self.dsa_layers.index(layer)]

    def conv_state(self, layer: int) -> torch.Tensor:
        """bf16 [num_blocks, 3, 3P] view into the aliased page (block stride = the page)."""
        t = self.pages[self.slot[layer]]
        P = self.kda_heads * 128
        page = t.shape[1]
        return t.view(torch.bfloat16).as_strided((self.num_blocks, 3, 3 * P), (page // 2, 3 * P, 1))

    def rec_state(self, layer: int) -> torch.Tensor:
        """fp32 [num_blocks, H, 128, 128] view into the aliased page, after the conv state."""
        t = self.pages[self.slot[layer]]
        H = self.kda_heads
        page = t.shape[1]
        return t.view(torch.float32).as_strided((self.num_blocks, H, 128, 128), (page // 4, 128 * 128, 128, 1),
                                                self.rec_off // 4)

    def state_offsets(self, layer: int, block: int) -> tuple[int, int]:
        """Byte offsets (conv, recurrent) of a KDA layer's state for state block `block`, from the start of the latent
        tensor it aliases (the reference's page arithmetic)."""
        page = self.pages[self.slot[layer]].shape[1]
        return block * page, block * page + self.rec_off

    def ranges(self) -> list:
        """(device pointer, bytes) of every tensor (the capacity tiers' view ranges)."""
        ts = self.pages + self.pool + self.tail
        return [(t.data_ptr(), t.numel() * t.element_size()) for t in ts]

    def tier_ranges(self, stage: int) -> list["ViewRange"]:
        """Every byte range a context owns on this stage, as one block's row of one cache view (the reference's
        `kvpool.layout.from_stage_kv`, ssengine/kvpool/layout.py:32-59): KV ranges (kind "kv") -- each DSA layer's
        latent block and its pool-key rows, one logical block = 8,576 tokens -- then state ranges (kind "state") --
        each DSA layer's tail ring row (group 5), and each KDA layer's conv and recurrent state inside the latent
        block it aliases (group = its KDA group, the index into the request's state_blocks)."""
        out = []
        for j, layer in enumerate(self.dsa_layers):
            t = self.pages[j]
            out.append(ViewRange(stage, f"layers.{layer}.latent", "kv", t.data_ptr(), t.stride(0), t.shape[1]))
        for j, layer in enumerate(self.dsa_layers):
            t = self.pool[j]
            row = PAGES_PER_BLOCK * (POOL_PAGE_BYTES_FP8 if self.pool_fp8 else POOL_PAGE_BYTES)
            out.append(ViewRange(stage, f"layers.{layer}.pool_keys", "kv", t.data_ptr(), row, row))
        for j, layer in enumerate(self.dsa_layers):
            t = self.tail[j]
            row = t[0].numel() * t.element_size()
            out.append(ViewRange(stage, f"layers.{layer}.tail", "state", t.data_ptr(), row, row, TAIL_STATE))
        rec = self.kda_heads * 128 * 128 * 4
        for g in range(KDA_GROUPS):
            for layer in self.kda_layers:
                if self.group[layer] != g:
                    continue
                t = self.pages[self.slot[layer]]
                out.append(ViewRange(stage, f"layers.{layer}.conv", "state", t.data_ptr(), t.stride(0),
                                     self.conv_bytes, g))
                out.append(ViewRange(stage, f"layers.{layer}.recurrent", "state", t.data_ptr() + self.rec_off,
                                     t.stride(0), rec, g))
        return out


@dataclass(frozen=True)
class ViewRange:
    """One cache view's row for a logical block on one stage (the reference's `kvpool.layout.ViewRange`, same
    fields): block b's bytes are [base + b * stride, base + b * stride + nbytes)."""
    stage: int
    name: str
    kind: str                 # "kv" or "state"
    base: int                 # device address of logical block 0's row
    stride: int               # bytes from one logical block's row to the next
    nbytes: int               # bytes of one logical block's row
    group: int = -1           # state: index into the request's state_blocks
