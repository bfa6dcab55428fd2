"""ctypes bindings of libssengine_b200.so (the C ABI of include/ssengine_b200.h).

The library is the only compute path: there is no CPU or PyTorch fallback. `load()` raises if the shared object is
missing or was built without an entry point the header declares, and every call raises `SsbError` on a non-zero
return code.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libssengine_b200.so"

# every symbol include/ssengine_b200.h declares
EXPORTS = ("ssb_version", "ssb_sf_atom_cols", "ssb_nvfp4_quantize", "ssb_nvfp4_gemm", "ssb_moe_route",
           "ssb_moe_workspace_bytes", "ssb_moe_workspace_offsets", "ssb_moe_forward", "ssb_moe_forward_profiled",
           "ssb_moe_route_permute_noalloc", "ssb_topk_canonical", "ssb_stage_metadata", "ssb_embed_rows",
           "ssb_rmsnorm", "ssb_argmax_rows", "ssb_mhc", "ssb_mhc_ws", "ssb_mhc_workspace_bytes", "ssb_kda_prefill", "ssb_kda_prefill_ws",
           "ssb_kda_workspace_bytes", "ssb_kda_conv",
           "ssb_ipc_export", "ssb_ipc_open", "ssb_ipc_close", "ssb_flag_wait", "ssb_flag_write", "ssb_p2p_copy",
           "ssb_indexer_logits", "ssb_indexer_expand", "ssb_sparse_mla", "ssb_mla_cache_append", "ssb_mla_q_pack",
           "ssb_kpool_insert", "ssb_gated_rmsnorm", "ssb_gated_rmsnorm_nvfp4", "ssb_hc_expand", "ssb_hc_mean",
           "ssb_nvfp4_gemm_grouped", "ssb_rmsnorm_cols", "ssb_rope", "ssb_transpose_heads", "ssb_concat_cols",
           "ssb_head_tiles", "ssb_moe_route_sigmoid", "ssb_copy_runs", "ssb_indexer_logits_fp8",
           "ssb_indexer_q_quant", "ssb_kpool_insert_fp8")

EPI_F32, EPI_BF16, EPI_SWIGLU = 0, 1, 2
ROUTE_SOFTMAX, ROUTE_SIGMOID_BIAS = 0, 1

WS = dict(XQ=0, XSF=1, LOGITS=2, IDS=3, WEIGHTS=4, ROWS=5, COUNTS=6, OFFSETS=7, MASKS=8, BLOCKS=9, MTILES=10,
          NUM_MTILES=11, XQ_PERM=12, XSF_PERM=13, ACT=14, ACT_SF=15, Y=16, ROW_SRC=17, END=18)

STATUS = {0: "ok", 1: "bad arguments", 2: "CUDA launch error", 3: "workspace too small",
          4: "a bounded device wait expired", 5: "cuTensorMapEncodeTiled unavailable", 6: "device table overflow",
          7: "size beyond the no-alloc entry point's static scratch"}


class SsbError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {code} ({STATUS.get(code, 'unknown')})")
        self.code = code


class MoeLayerC(ctypes.Structure):
    """Mirror of `ssb_moe_layer`."""
    _fields_ = [("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("gs_x", ctypes.c_float), ("gs_h", ctypes.c_float),
                ("router_codes", ctypes.c_void_p), ("router_sf", ctypes.c_void_p), ("router_rows", ctypes.c_int64),
                ("router_alpha", ctypes.c_float), ("w1_codes", ctypes.c_void_p), ("w1_sf", ctypes.c_void_p),
                ("w1_alpha", ctypes.c_void_p), ("w2_codes", ctypes.c_void_p), ("w2_sf", ctypes.c_void_p),
                ("w2_alpha", ctypes.c_void_p), ("add_input", ctypes.c_int32), ("routing", ctypes.c_int32),
                ("n_group", ctypes.c_int32), ("topk_group", ctypes.c_int32), ("routed_scale", ctypes.c_float),
                ("route_bias", ctypes.c_void_p)]


class KdaLayerC(ctypes.Structure):
    """Mirror of `ssb_kda_layer`."""
    _fields_ = [("heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("conv_weight", ctypes.c_void_p),
                ("a_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p), ("lower_bound", ctypes.c_float),
                ("scale", ctypes.c_float), ("conv_state", ctypes.c_void_p), ("conv_state_stride", ctypes.c_int64),
                ("rec_state", ctypes.c_void_p), ("rec_state_stride", ctypes.c_int64)]


class MhcParamsC(ctypes.Structure):
    """Mirror of `ssb_mhc_params`."""
    _fields_ = [("hidden", ctypes.c_int32), ("hc_mult", ctypes.c_int32), ("fn", ctypes.c_void_p),
                ("scale", ctypes.c_void_p), ("base", ctypes.c_void_p), ("norm_weight", ctypes.c_void_p),
                ("rms_eps", ctypes.c_float), ("pre_eps", ctypes.c_float), ("sinkhorn_eps", ctypes.c_float),
                ("post_mult", ctypes.c_float), ("norm_eps", ctypes.c_float), ("sinkhorn_repeat", ctypes.c_int32),
                ("status", ctypes.c_void_p)]


_LIB = None

# Kernels each entry point launches (1 unless listed), for the count of this library's launches in a timed region
KERNELS_PER_CALL = {"ssb_moe_forward": 10, "ssb_moe_forward_profiled": 10, "ssb_mhc_ws": 2,
                    "ssb_kda_prefill": 2, "ssb_kda_prefill_ws": 2, "ssb_kpool_insert": 2, "ssb_kpool_insert_fp8": 2,
                    "ssb_stage_metadata": 2}


class _Counting:
    """The loaded library with a launch counter: every entry-point call adds its kernel count to `launches` while
    `on` is set."""

    def __init__(self, lib):
        self._lib = lib
        self.on = False
        self.launches = 0
        self._wrapped = {}

    def __getattr__(self, name):
        fn = getattr(self._lib, name)
        if not name.startswith("ssb_"):
            return fn
        w = self._wrapped.get(name)
        if w is None:
            k = KERNELS_PER_CALL.get(name, 1)
            counter = self

            def w(*args, _fn=fn, _k=k):
                if counter.on:
                    counter.launches += _k
                return _fn(*args)

            self._wrapped[name] = w
        return w

_P, _I32, _I64, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
_SIGS = {
    "ssb_version": ([], ctypes.c_char_p),
    "ssb_sf_atom_cols": ([_I64], _I64),
    "ssb_nvfp4_quantize": ([_P, _I64, _I64, _I64, _F, _P, _I64, _P, _P], ctypes.c_int),
    "ssb_nvfp4_gemm": ([_I32, _P, _P, _I64, _I64, _P, _P, _I64, _F, _P, _I64, _P, _F, _P, _P], ctypes.c_int),
    "ssb_moe_route": ([_P, _I64, _I32, _I32, _P, _P, _P], ctypes.c_int),
    "ssb_moe_route_sigmoid": ([_P, _I64, _I32, _I32, _P, _I32, _I32, _F, _P, _P, _P], ctypes.c_int),
    "ssb_moe_workspace_bytes": ([ctypes.POINTER(MoeLayerC), _I64], _I64),
    "ssb_moe_workspace_offsets": ([ctypes.POINTER(MoeLayerC), _I64, ctypes.POINTER(ctypes.c_int64), _I32],
                                  ctypes.c_int),
    "ssb_moe_forward": ([ctypes.POINTER(MoeLayerC), _P, _I64, _P, _P, _I64, _P, _P], ctypes.c_int),
    "ssb_moe_forward_profiled": ([ctypes.POINTER(MoeLayerC), _P, _I64, _P, _P, _I64, _P, _P,
                                  ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "ssb_moe_route_permute_noalloc": ([_P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "ssb_topk_canonical": ([_P, _I64, _I64, _P, _P, _I32, _P, _I32, _P], ctypes.c_int),
    "ssb_stage_metadata": ([_P, _P, _P, _P, _I32, _I64, _I64, _I32, _I32, _P, _P, _P, _P], ctypes.c_int),
    "ssb_embed_rows": ([_P, _I64, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "ssb_rmsnorm": ([_P, _I64, _P, _I64, _P, _F, _P, _P], ctypes.c_int),
    "ssb_argmax_rows": ([_P, _I64, _I64, _I64, _P, _P], ctypes.c_int),
    "ssb_mhc": ([ctypes.POINTER(MhcParamsC), _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P], ctypes.c_int),
    "ssb_mhc_ws": ([ctypes.POINTER(MhcParamsC), _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _I64, _P], ctypes.c_int),
    "ssb_mhc_workspace_bytes": ([_I64], ctypes.c_int64),
    "ssb_kda_prefill": ([ctypes.POINTER(KdaLayerC), _P, _I64, _P, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _P],
                        ctypes.c_int),
    "ssb_kda_prefill_ws": ([ctypes.POINTER(KdaLayerC), _P, _I64, _P, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _P,
                            _I64, _P, _P], ctypes.c_int),
    "ssb_kda_workspace_bytes": ([ctypes.c_int32, _I64, _I64], ctypes.c_int64),
    "ssb_kda_conv": ([ctypes.POINTER(KdaLayerC), _P, _I64, _I64, _P, _I64, _P, _P, _P, _P], ctypes.c_int),
    "ssb_ipc_export": ([_P, _P, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ssb_ipc_open": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "ssb_ipc_close": ([_P], ctypes.c_int),
    "ssb_flag_wait": ([_P, ctypes.c_uint32, _I64, _P, _P], ctypes.c_int),
    "ssb_flag_write": ([_P, ctypes.c_uint32, _P], ctypes.c_int),
    "ssb_p2p_copy": ([_P, _P, _I64, _P], ctypes.c_int),
    "ssb_copy_runs": ([_P, _I64, _P, _P], ctypes.c_int),
    "ssb_indexer_logits_fp8": ([_P, _P, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P],
                               ctypes.c_int),
    "ssb_indexer_q_quant": ([_P, _I64, _P, _P, _P], ctypes.c_int),
    "ssb_kpool_insert_fp8": ([_P, _P, _I64, _P, _P, _I64, _I32, _P, _I64, _P, _P, _P], ctypes.c_int),
    "ssb_indexer_logits": ([_P, _P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "ssb_indexer_expand": ([_P, _I64, _I32, _P, _I64, _P, _I64, _P], ctypes.c_int),
    "ssb_sparse_mla": ([_P, _I64, _P, _P, _I64, _I32, _P, _I32, _P, _I64, _F, _F, _P, _P, _P], ctypes.c_int),
    "ssb_mla_cache_append": ([_P, _I64, _P, _I64, _P, _F, _P], ctypes.c_int),
    "ssb_mla_q_pack": ([_P, _I64, _P, _I64, _I64, _I64, _P, _F, _P], ctypes.c_int),
    "ssb_kpool_insert": ([_P, _P, _I64, _P, _P, _I64, _I32, _P, _I64, _P, _P, _P], ctypes.c_int),
    "ssb_gated_rmsnorm": ([_P, _I64, _P, _I64, _P, _F, _P, _I64, _I64, _I32, _P], ctypes.c_int),
    "ssb_gated_rmsnorm_nvfp4": ([_P, _I64, _P, _I64, _P, _F, _F, _P, _I64, _P, _I64, _I32, _P], ctypes.c_int),
    "ssb_hc_expand": ([_P, _I64, _I64, _P, _P], ctypes.c_int),
    "ssb_hc_mean": ([_P, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "ssb_nvfp4_gemm_grouped": ([_I32, _P, _P, _I64, _I64, _P, _P, _I64, _I32, _P, _P, _P, _I32, _P, _I64, _P, _P],
                               ctypes.c_int),
    "ssb_rmsnorm_cols": ([_P, _I64, _I32, _I64, _P, _F, _P, _I64, _P], ctypes.c_int),
    "ssb_rope": ([_P, _I64, _I32, _I64, _P, _I64, _F, _P], ctypes.c_int),
    "ssb_transpose_heads": ([_P, _P, _I64, _I64, _I32, _I32, _I64, _I64, _I32, _P], ctypes.c_int),
    "ssb_concat_cols": ([_P, _I64, _I32, _P, _I64, _I32, _P, _I64, _I64, _P], ctypes.c_int),
    "ssb_head_tiles": ([_I32, _I64, _P, _I64, _P, _P], ctypes.c_int),
}

MOE_KERNELS = 10      # kernels ssb_moe_forward launches (+ a memset when F % 256 != 0)
MOE_STEPS = ("quantize", "router_gemm", "route", "count", "offsets", "scatter", "gate_up_gemm", "down_gemm",
             "combine")


def load(path: Path | None = None):
    """Load the library (once). Raises FileNotFoundError / AttributeError when it is missing or incomplete. The shared
    instance counts this library's kernel launches while `load().on` is set (`load().launches`)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is not built: run `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(str(p))
    for name in EXPORTS:
        fn = getattr(lib, name)        # AttributeError when the symbol is missing
        args, res = _SIGS[name]
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _LIB = _Counting(lib)
        return _LIB
    return lib


_SCRATCH: dict = {}


def scratch(device, nbytes: int):
    """A per-device uint8 workspace of at least `nbytes`, grown on demand and shared by the calls that take one
    (`ssb_kda_prefill_ws`, `ssb_mhc_ws`); for calls on one stream, as a stage's layers run."""
    import torch

    dev = torch.device(device)
    key = (dev.type, dev.index)
    t = _SCRATCH.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        _SCRATCH[key] = t
    return t


def check(name: str, rc: int) -> None:
    if rc != 0:
        raise SsbError(name, rc)


def stream_ptr(stream=None) -> int:
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)
