"""ssengine_b200: a B200-native (sm_100a) prefill-stage engine behind the reference's stage interface.

Import name `ssengine_b200`; the package directory is `ssengine-glm5.3-flash_b200/` (loaded by
`__graft_entry__.import_package`). Compute runs only in libssengine_b200.so (include/ssengine_b200.h); the Python
modules are the host side: device memory, layouts, the random-init generator, and the reference-facing classes.

- `lib`      ctypes bindings of the C ABI (fails loudly when the library is missing)
- `layout`   NVFP4 operand layouts (packed e2m1 codes, 128x4 scale atoms, gate/up tile interleave)
- `weights`  seeded random-init NVFP4 parameters
- `moe`      `MoELayer`: one NVFP4 MoE layer through `ssb_moe_forward`
- `stage`    `StageModel`: the reference's stage interface (prepare / run / forward) over the library
- `worker`, `edge`  the stage worker loop and the P2P stage edge
- `scheduler`, `pagepool`, `dispatch`  the control plane on stage 0's host: microbatch forming (FIFO / SRPT, budgets,
             force-schedule), the page pool with the exact prefix cache, and when to form (host only, no device code)
- `controller`  serving a session load: stage 0's loop (arrivals -> plans -> reports -> TTFT), the other stages' loop
- `tier`     the DRAM tier under HBM's kept contexts and the in-stream-order copies that move them
"""

__all__ = ["lib", "layout", "weights", "moe"]
