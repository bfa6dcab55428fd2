"""The C-ABI library: it loads, exports every symbol include/ssengine_b200.h declares, and its host-only entry points
(workspace sizing, argument checks) answer without a GPU."""

import ctypes
import re

import pytest

from tests.conftest import ROOT


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "ssengine_b200.h").read_text()
    return sorted(set(re.findall(r"\b(ssb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_what_the_bindings_bind():
    from ssengine_b200 import lib

    assert declared_symbols() == sorted(lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from ssengine_b200 import lib

    so = lib.load()
    for name in declared_symbols():
        assert hasattr(so, name), name
    assert so.ssb_version().decode().startswith("ssengine_b200")
    assert so.ssb_sf_atom_cols(4096) == 64 and so.ssb_sf_atom_cols(128) == 4 and so.ssb_sf_atom_cols(257) == 8


def layer_c(H=4096, F=1024, E=128, k=8):
    from ssengine_b200 import lib

    return lib.MoeLayerC(H, F, E, k, 336.0, 84.0, 0, 0, 128, 1.0, 0, 0, 0, 0, 0, 0, 0)


def test_workspace_layout_on_the_host():
    from ssengine_b200 import lib

    so = lib.load()
    L = layer_c()
    n = so.ssb_moe_workspace_bytes(ctypes.byref(L), 8192)
    n_off = lib.WS["END"] + 1
    arr = (ctypes.c_int64 * n_off)()
    assert so.ssb_moe_workspace_offsets(ctypes.byref(L), 8192, arr, n_off) == 0
    off = list(arr)
    assert off[-1] == n and all(o % 256 == 0 for o in off) and off == sorted(off)
    rcap = -(-(8192 * 9 + 129 * 127) // 128) * 128
    assert off[lib.WS["END"]] - off[lib.WS["Y"]] >= rcap * 4096 * 2
    assert 0.9e9 < n < 1.3e9
    bad = layer_c(H=4000)
    assert so.ssb_moe_workspace_bytes(ctypes.byref(bad), 8192) == -1


def test_forward_rejects_bad_arguments_before_touching_the_device():
    from ssengine_b200 import lib

    so = lib.load()
    L = layer_c()
    assert so.ssb_moe_forward(ctypes.byref(L), None, 16, None, None, 0, None, None) == 1
    assert so.ssb_moe_route(None, 16, 128, 8, None, None, None) == 1
    assert so.ssb_nvfp4_gemm(0, None, None, 16, 256, None, None, 128, 1.0, None, 128, None, 1.0, None, None) == 1
    with pytest.raises(lib.SsbError):
        lib.check("ssb_moe_forward", 3)
