"""Writes tests/golden/control_ref.json.gz: the reference's own control plane (ssengine/engine/scheduler.py,
ssengine/engine/kv.py, ssengine/runtime/dispatch.py) run through the scenarios of tests/control_sim.py.

Run from the repository root in a container that has the reference checked out (read-only is fine); it imports, never
copies, the reference's modules. The fixture it writes is what the CPU tests compare this package's scheduler, KV
manager and dispatch rule against, microbatch for microbatch:

    SSENGINE_HANDOFF=/tmp/empty REF=/path/to/SSEngine-GLM5.3-Flash python tests/golden/make_control_golden.py
"""

import gzip
import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

HERE = Path(__file__).resolve().parent


def main(ref: str):
    sys.path.insert(0, ref)
    sys.path.insert(0, str(HERE.parent))
    import control_sim
    from ssengine.config import SchedulerConfig
    from ssengine.engine import kv, scheduler
    from ssengine.runtime import dispatch

    ns = SimpleNamespace(Request=scheduler.Request, KvManager=kv.KvManager, Scheduler=scheduler.Scheduler,
                         SchedulerConfig=SchedulerConfig, kv_pages_for=kv.kv_pages_for)
    out = {"scenarios": {}, "dispatch": {}}
    for name, sc in control_sim.SCENARIOS.items():
        out["scenarios"][name] = rec = control_sim.run(ns, **sc)
        print(f"{name}: {len(rec['microbatches'])} microbatches, {len(rec['requests'])} requests, "
              f"kv {rec['kv_stats']}")
    consts = (dispatch.NOW, dispatch.WAIT, dispatch.NO)
    for name, kw in {"host_stamps": dict(seed=11), "no_stamps": dict(seed=12, with_host=False),
                     "pp8": dict(seed=13, stages=8)}.items():
        out["dispatch"][name] = control_sim.dispatch_trace(dispatch.DispatchRule, consts, **kw)
        print(f"dispatch {name}: {len(out['dispatch'][name])} decisions")
    with gzip.open(HERE / "control_ref.json.gz", "wt") as f:
        json.dump(out, f, separators=(",", ":"))


if __name__ == "__main__":
    if not os.environ.get("REF"):
        raise SystemExit("set REF to the reference checkout")
    os.environ.setdefault("SSENGINE_HANDOFF", "/tmp/empty_handoff")
    main(os.environ["REF"])
