"""CPU oracle for the prefill-stage hot path -- TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s `cpu_baseline` / `--impl reference` legs may import this
package, and only as the checker or the timed CPU baseline. The product (the `ssengine_b200` package and its CUDA
library) never imports, links or executes anything here; it fails loudly when its CUDA library is missing.

Modules:
- `nvfp4`: the NVFP4 codec (e2m1 values, e4m3 per-16 scales, fp32 global scale) in numpy, bit-exact.
- `moe`: one MoE layer (router, softmax top-k routing, expert permutation, SwiGLU experts, weighted combine, shared
  expert) in fp32 over the dequantized NVFP4 operands.
- `topk`: the canonical top-k rule of the indexer (ssengine/model/topk_canon.py:33-52).
- `pages`: page-table / slot addressing and graph buckets (ssengine/model/metadata.py:65-96,
  ssengine/engine/kv.py:60-75, ssengine/model/stage.py:63-69).

Parity status per module is stated in each module header: `topk` and `pages` are pinned to fixtures generated from
the reference's own functions (tests/golden/make_golden.py); `nvfp4` and `moe` restate published algorithms whose
reference implementation (FlashInfer trtllm NVFP4 MoE, vLLM `scaled_fp4_quant`) is a third-party library absent
from the reference tree -- parity unpinned against the reference itself, pinned only by known-answer tests of the
format.
"""
