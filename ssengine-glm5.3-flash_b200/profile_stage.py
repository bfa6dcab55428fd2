"""Three forwards of one hybrid stage slice (layers 4-7 of a 3 x 4 split: KDA, KDA, KDA, DSA, each with the NVFP4 MoE
and mHC boundaries; 8,192 tokens of 4 fresh requests, hidden 4096, 64 KDA heads, 128 experts top-8): the program the
stage-slice launch lists are captured from (the last forward is the measured one; the stage's constructor runs a
256-token warm-up forward first)."""
import sys
import pathlib

import torch

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent.parent))
import __graft_entry__ as g  # noqa: E402

g.import_package()
from ssengine_b200.messages import Chunk, Plan  # noqa: E402
from ssengine_b200.stage import StageConfig, StageModel  # noqa: E402

dev = torch.device("cuda:0")
cfg = StageConfig(layer_split=(4, 4, 4), hidden=4096, inter=1024, experts=128, top_k=8, vocab=1024, num_blocks=6,
                  mb_tokens=8192, layer_kind="hybrid", kda_heads=64)
stage = StageModel(cfg, 1, dev)
lens, at, chunks = [3000, 2500, 1700, 992], 1, []
for i, n in enumerate(lens):
    npg = -(-n // 128)
    chunks.append(Chunk(f"r{i}", 0, n, list(range(at, at + npg)), [i + 1] * 6, True, None))
    at += npg
plan = Plan(0, chunks)
hid = torch.randn(8192, 4 * 4096, device=dev).to(torch.bfloat16)
for _ in range(3):
    stage.forward(plan, hid)
torch.cuda.synchronize()
print("ok")
