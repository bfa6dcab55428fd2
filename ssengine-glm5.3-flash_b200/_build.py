"""Build libssengine_b200.so in-tree with nvcc for sm_100a (no JIT cache: the built file travels with the tree).

Each source compiles to its own object under `_build/` (in parallel, only sources newer than their object or than a
shared header), then one nvcc link makes the shared library."""

from __future__ import annotations

import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libssengine_b200.so"
OBJ = PKG.parent / "_build"
SOURCES = ["gemm_nvfp4.cu", "moe_ops.cu", "capi.cu", "moe_noalloc.cu", "topk.cu", "stage.cu", "mhc.cu", "kda.cu",
           "edge.cu", "indexer.cu", "mla.cu", "kpool.cu", "dsa.cu", "tier.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(home) / "bin" / "nvcc")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [PKG.parent / "include" / "ssengine_b200.h"]


def _obj(src: str) -> Path:
    return OBJ / (Path(src).stem + ".o")


def _stale_obj(src: str, newest_header: float) -> bool:
    o = _obj(src)
    if not o.exists():
        return True
    t = o.stat().st_mtime
    return (CSRC / src).stat().st_mtime > t or newest_header > t


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + _headers()
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    newest = max((p.stat().st_mtime for p in _headers() if p.exists()), default=0.0)
    todo = [s for s in SOURCES if force or _stale_obj(s, newest)]

    def compile_one(src: str) -> None:
        tmp = _obj(src).with_suffix(".o.tmp")
        cmd = [nvcc(), *NVCC_FLAGS, "-c", "-o", str(tmp), str(CSRC / src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True, cwd=PKG)
        os.replace(tmp, _obj(src))

    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(compile_one, s) for s in todo]:
            f.result()
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(_obj(s)) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=PKG)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
