"""Generate the golden fixtures of tests/golden/ by calling the reference's own Python functions.

Run from the repository root in a container that has the reference checked out (read-only is fine):

    SSENGINE_HANDOFF=/tmp/empty REF=/path/to/SSEngine-GLM5.3-Flash python tests/golden/make_golden.py

It imports (never copies) these reference functions and records their outputs on seeded inputs:
- ssengine/model/topk_canon.py:33-52  `canonical_topk_torch`      -> topk_canon.npz
- ssengine/model/metadata.py:79-96    `g0_table`                  -> g0_table.npz
- ssengine/model/metadata.py:65-76    `graph_rows`                -> (in g0_table.npz)
- ssengine/model/stage.py:63-69       `GRAPH_BUCKETS`, `graph_bucket` -> buckets.json
- ssengine/engine/kv.py:60-75         `block_pages`, `kv_pages_for`   -> (in g0_table.npz)
- ssengine/model/pp_patch.py          `kpool_heads`, `kpool_compress_insert`, `kpool_seed_tail_cache`, driven as the
  reference's tests/test_kpool_cpu.py drives them (`indexer_call`, with its torch reference ops `ref_compress` /
  `ref_seed`): pools written by chunked prefills that start inside a pool, several requests in one microbatch
                                                                       -> kpool_ref.npz (`--parts kpool`)
- ssengine/model/moe_tuning.py         `scale_hist`, `forced_logits`, with the reference's own routing check
  `(logits.sigmoid() + bias).topk(8)` as tests/test_moe_tuning_cpu.py:55-64 runs it (512 tokens, 288 experts, a bias
  of 12.4 + U[0, 0.52))                                                -> routing_ref.npz (`--parts routing`)
The fixtures are small (tens of KB) and committed; the tests never read the reference at run time.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


# (request, start, tokens) microbatches over prompts of KPOOL_LENS tokens; chunk starts inside pools, a request resumed
# right after another's rows, a microbatch shorter than one pool
KPOOL_LENS = [40, 24, 30]
KPOOL_SCHEDULE = [[(0, 0, 13), (2, 0, 13)], [(2, 13, 3)], [(0, 13, 14), (1, 0, 24), (2, 16, 14)], [(0, 27, 13)]]


def kpool_inputs(seed: int = 20261207):
    """Per request bf16 key and gate rows [L, 8] and the pool position embedding ape [4, 8] (fp32)."""
    rng = np.random.default_rng(seed)

    def b16(a):
        import torch

        return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).float().numpy()

    k = [b16(rng.standard_normal((n, 8))) for n in KPOOL_LENS]
    g = [b16(rng.standard_normal((n, 8))) for n in KPOOL_LENS]
    return k, g, rng.standard_normal((4, 8)).astype(np.float32)


def make_kpool(ref: str) -> None:
    import torch

    sys.path.insert(0, str(Path(ref) / "tests"))
    import test_kpool_cpu as rk                  # the reference's own CPU driver and torch reference ops

    k, g, ape = kpool_inputs()
    k_all = [torch.from_numpy(a).to(torch.bfloat16) for a in k]
    g_all = [torch.from_numpy(a).to(torch.bfloat16) for a in g]
    cache = torch.zeros(10000 * len(KPOOL_LENS), rk.HD)
    tail = torch.zeros(len(KPOOL_LENS), 2, rk.KPOOL, rk.HD, dtype=torch.bfloat16)
    for mb in KPOOL_SCHEDULE:
        rk.indexer_call(mb, k_all, g_all, torch.from_numpy(ape), cache, tail)
    pools = np.concatenate([cache[r * 10000:r * 10000 + n // rk.KPOOL].numpy() for r, n in enumerate(KPOOL_LENS)])
    np.savez_compressed(HERE / "kpool_ref.npz", pools=pools, tail=tail.float().numpy())


def make_routing() -> None:
    """The reference's routing test case (tests/test_moe_tuning_cpu.py:55-64): a Pareto-shaped expert histogram scaled
    to 512 tokens, the logits `forced_logits` builds for it (+-30), a layer bias, and the experts the reference's rule
    `(logits.sigmoid() + bias).topk(8)` selects (stored sorted per token; torch.topk's slot order is not part of the
    rule)."""
    import random

    import torch

    from ssengine.model import moe_tuning as mt

    rnd = random.Random(0)
    tokens = 512
    w = [rnd.paretovariate(1.2) for _ in range(288)]
    h = mt.scale_hist([int(x * 100) + 1 for x in w], tokens)
    logits = mt.forced_logits(h, tokens, torch.float32, "cpu")
    gen = torch.Generator().manual_seed(0)
    bias = 12.4 + torch.rand(288, generator=gen) * 0.52
    ids = (logits.sigmoid() + bias).topk(8, dim=1).indices
    assert torch.bincount(ids.flatten(), minlength=288).tolist() == h
    np.savez_compressed(HERE / "routing_ref.npz", selected=np.packbits((logits > 0).numpy(), axis=1),
                        bias=bias.numpy().astype(np.float32), hist=np.asarray(h, np.int32),
                        ids_sorted=np.sort(ids.numpy(), axis=1).astype(np.int32))


def main() -> None:
    ref = os.environ.get("REF")
    if not ref:
        raise SystemExit("set REF to the reference checkout")
    if sys.argv[1:] == ["--parts", "routing"]:
        os.environ.setdefault("SSENGINE_HANDOFF", "/tmp/empty_handoff")
        sys.path.insert(0, ref)
        make_routing()
        print("wrote routing_ref.npz")
        return
    if sys.argv[1:] == ["--parts", "kpool"]:
        os.environ.setdefault("SSENGINE_HANDOFF", "/tmp/empty_handoff")
        sys.path.insert(0, ref)
        make_kpool(ref)
        print("wrote kpool_ref.npz")
        return
    os.environ.setdefault("SSENGINE_HANDOFF", "/tmp/empty_handoff")
    sys.path.insert(0, ref)
    import torch

    from ssengine.engine.kv import block_pages, kv_pages_for
    from ssengine.model.metadata import g0_table, graph_rows
    from ssengine.model.stage import GRAPH_BUCKETS, graph_bucket
    from ssengine.model.topk_canon import canonical_topk_torch

    rng = np.random.default_rng(20261201)

    # -- canonical top-k: rows with ties at the k-th value, short rows, empty rows, ranges that start past column 0
    cases = {}
    for name, (rows, width, k, levels) in {"ties": (64, 300, 16, 7), "dense": (32, 2048, 512, 0),
                                           "wide_ties": (16, 4096, 512, 3)}.items():
        if levels:
            logits = rng.integers(0, levels, size=(rows, width)).astype(np.float32)
        else:
            logits = rng.standard_normal((rows, width)).astype(np.float32)
        ks = rng.integers(0, width // 3, size=rows).astype(np.int32)
        ke = np.minimum(width, ks + rng.integers(0, width, size=rows)).astype(np.int32)
        ke[0] = ks[0]                      # an empty row
        ke[1] = min(width, ks[1] + k // 2)  # a row shorter than k
        # a valid kernel answer to rewrite: the first k keys of a stable descending sort (any valid answer works)
        dst = np.full((rows, k), -1, dtype=np.int32)
        for r in range(rows):
            seg = logits[r, ks[r]:ke[r]]
            sel = np.argsort(-seg, kind="stable")[:k]
            rng.shuffle(sel)
            dst[r, : sel.size] = sel
        d = torch.from_numpy(dst.copy())
        canonical_topk_torch(torch.from_numpy(logits), torch.from_numpy(ks), torch.from_numpy(ke), d, k)
        cases[name] = dict(logits=logits, ks=ks, ke=ke, k=np.int32(k), out=d.numpy())
    np.savez_compressed(HERE / "topk_canon.npz", **{f"{c}__{f}": v for c, d in cases.items() for f, v in d.items()})

    # -- g0 page table and slots: scattered pages, prefixes that start inside a page and a block, decode-class rows
    specs = [(0, 5000), (8571, 700), (20_000, 255), (130, 1), (0, 129)]
    pool = block_pages(range(1, 40))
    rng.shuffle(pool)
    pages, k = [], 0
    for s, n in specs:
        m = kv_pages_for(s + n)
        pages.append(pool[k:k + m])
        k += m
    seq = np.array([s + n for s, n in specs], dtype=np.int64)
    pos = np.concatenate([np.arange(s, s + n) for s, n in specs])
    qsl = np.r_[0, np.cumsum([n for _, n in specs])].astype(np.int64)
    width = 8 * 134
    table, slots = g0_table(pages, seq, pos, qsl, width, 128)
    tok = rng.integers(0, 151_552, size=len(pos)).astype(np.int64)
    bucket = graph_bucket(len(pos), GRAPH_BUCKETS)
    grow = graph_rows(pos, slots, tok, bucket)
    lens = np.array([len(p) for p in pages], dtype=np.int64)
    np.savez_compressed(HERE / "g0_table.npz", starts=np.array([s for s, _ in specs], dtype=np.int64),
                        num_tokens=np.array([n for _, n in specs], dtype=np.int64),
                        pages=np.concatenate([np.asarray(p, dtype=np.int64) for p in pages]), page_counts=lens,
                        width=np.int64(width), table=table, slots=slots, token_ids=tok, bucket=np.int64(bucket),
                        graph_rows=grow, block_pages_1_3=np.asarray(block_pages([1, 3]), dtype=np.int64))
    probe = [0, 1, 127, 128, 129, 255, 256, 257, 3000, 7937, 8192, 8193]
    (HERE / "buckets.json").write_text(json.dumps({
        "GRAPH_BUCKETS": list(GRAPH_BUCKETS), "probe": probe,
        "bucket": [graph_bucket(n, GRAPH_BUCKETS) for n in probe],
        "kv_pages_for": {str(n): kv_pages_for(n) for n in [0, 1, 127, 128, 129, 8576, 8577]}}, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
