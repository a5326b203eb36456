"""ctypes binding of ``libdsv4moe.so`` (the C ABI declared in include/dsv4moe.h).

The library is loaded from this package directory.  There is no fallback:
if it is missing or fails to load, every op raises ``Dsv4LibraryError``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

LIB_NAME = "libdsv4moe.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

DSV4_OK = 0
DSV4_EINVAL = -1
DSV4_ENOMEM = -2
DSV4_ECUDA = -3
DSV4_ETIMEOUT = -4
DSV4_ENCCL = -5
DSV4_ENOTFOUND = -6
DSV4_EUNSUPPORTED = -7

SCORE_FUNCS = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}
PROFILES = {"bf16": 0, "a4w4": 1}
# token row formats of the expert-parallel dispatch (DSV4_ROWS_*)
ROWS_BF16, ROWS_FP8, ROWS_MXFP4 = 0, 1, 2

_p, _i32, _i64, _f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float

# name -> (restype, argtypes); mirrors include/dsv4moe.h
SIGNATURES = {
    "dsv4_last_error_string": (C.c_char_p, []),
    "dsv4_abi_version": (C.c_int, []),
    "dsv4_expert_slot_bytes": (_i64, [_i32, _i32]),
    "dsv4_pack_expert_host": (C.c_int, [_p, _p, _p, _p, _p, _p, _i32, _i32, _p]),
    "dsv4_unpack_expert_host": (C.c_int, [_p, _i32, _i32, _p, _p, _p, _p, _p, _p]),
    "dsv4_dequant_mxfp4": (C.c_int, [_p, _p, _p, _i64, _i64, _p]),
    "dsv4_slot_dequant": (C.c_int, [_p, _i32, _i32, _p, _p, _p, _p]),
    "dsv4_act_quant_fp8_rt": (C.c_int, [_p, _i64, _i64, _p]),
    "dsv4_act_quant_mxfp4": (C.c_int, [_p, _i64, _i64, _p, _p, _p]),
    "dsv4_route_workspace_bytes": (_i64, [_i64, _i32, _i32]),
    "dsv4_route_topk": (C.c_int, [_p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _p, _p, _p,
                                  _i64, _p]),
    "dsv4_route_topk_noalloc": (C.c_int, [_p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _p,
                                          _p, _p]),
    "dsv4_mma_peak": (C.c_int, [_i32, _i32, _i64, _i32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "dsv4_moe_align": (C.c_int, [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p]),
    "dsv4_moe_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32, _i64]),
    "dsv4_moe_plan_create": (C.c_int, [C.POINTER(_p), _i32, _i32, _i32, _i32, _i64, _f32, _p, _i64, _p, _i64]),
    "dsv4_moe_plan_destroy": (C.c_int, [_p]),
    "dsv4_moe_forward": (C.c_int, [_p, _i32, _p, _i64, _p, _p, _p, _p, _p]),
    "dsv4_moe_forward_rows": (C.c_int, [_p, _i32, _p, _i64, _p, _p, _p, _p, _p, _p]),
    "dsv4_moe_output_rows": (C.c_int, [_p, C.POINTER(_p), C.POINTER(_p)]),
    "dsv4_moe_forward_scatter": (C.c_int, [_p, _i32, _p, _i64, _p, _p, _p, _p, _p, _p]),
    "dsv4_moe_forward_scatter_q": (C.c_int, [_p, _i32, _p, _i32, _i64, _p, _p, _p, _p, _p, _p]),
    "dsv4_shared_slot_bytes": (_i64, [_i32, _i32]),
    "dsv4_pack_shared_host": (C.c_int, [_p, _p, _p, _p, _p, _p, _i32, _i32, _p]),
    "dsv4_moe_workspace_bytes_ex": (_i64, [_i32, _i32, _i32, _i32, _i64, _i32]),
    "dsv4_moe_plan_create_ex": (C.c_int, [C.POINTER(_p), _i32, _i32, _i32, _i32, _i64, _f32, _p, _i64, _p, _i64,
                                          _i32]),
    "dsv4_moe_forward_shared": (C.c_int, [_p, _i32, _p, _i64, _p, _p, _p, _p, _p, _p]),
    "dsv4_moe_status": (C.c_int, [_p, _p]),
    "dsv4_moe_enable_timing": (C.c_int, [_p, _i32]),
    "dsv4_moe_set_gemm_tile": (C.c_int, [_p, _i32]),
    "dsv4_moe_set_ffn_fusion": (C.c_int, [_p, _i32]),
    "dsv4_moe_route": (C.c_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i32, _i32, _f32, _p, _p, _p]),
    "dsv4_slotcache_create": (C.c_int, [C.POINTER(_p), _i64]),
    "dsv4_slotcache_destroy": (C.c_int, [_p]),
    "dsv4_slotcache_lookup": (C.c_int, [_p, _p, _p, _i64, _p, _p]),
    "dsv4_slotcache_slot_of": (_i32, [_p, _i64, _i64]),
    "dsv4_slotcache_stats": (C.c_int, [_p, _p]),
    "dsv4_slotcache_snapshot": (C.c_int, [_p, _p, _p, _p, _i64, _p]),
    "dsv4_slotcache_clear": (C.c_int, [_p]),
    "dsv4_slotdir_workspace_bytes": (_i64, [_i32, _i32, _i64]),
    "dsv4_slotdir_create": (C.c_int, [C.POINTER(_p), _i32, _i32, _p, _i64, _i64, _p, _i64]),
    "dsv4_slotdir_destroy": (C.c_int, [_p]),
    "dsv4_slotdir_set_sources": (C.c_int, [_p, _i64, _p, _p, _p]),
    "dsv4_slotdir_acquire": (C.c_int, [_p, _i32, _p, _i64, _i32, _p]),
    "dsv4_slotdir_table": (C.c_int, [_p, _i32, C.POINTER(_p)]),
    "dsv4_slotdir_stats": (C.c_int, [_p, _p, _p]),
    "dsv4_slotdir_status": (C.c_int, [_p, _p]),
    "dsv4_slotdir_snapshot": (C.c_int, [_p, _p, _p, _p]),
    "dsv4_slotdir_clear": (C.c_int, [_p, _p]),
    "dsv4_ep_dispatch_pack": (C.c_int, [_p, _p, _p, _i64, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p]),
    "dsv4_ep_ipc_handle_bytes": (C.c_int, []),
    "dsv4_ep_create": (C.c_int, [C.POINTER(_p), _i32, _i32, _i32, _i64, _i32, _i32, _p]),
    "dsv4_ep_connect": (C.c_int, [_p, _p]),
    "dsv4_ep_buffers": (C.c_int, [_p, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p), C.POINTER(_p), C.POINTER(_p)]),
    "dsv4_ep_dispatch": (C.c_int, [_p, _p, _p, _p, _i64, _i32, _p, _p, _p, _p]),
    "dsv4_ep_dispatch_q": (C.c_int, [_p, _p, _p, _p, _i64, _i32, _p, _p, _i32, _p, _p]),
    "dsv4_ep_row_bytes": (C.c_int64, [_i32, _i32]),
    "dsv4_ep_return": (C.c_int, [_p, _p, _p, _p, _p]),
    "dsv4_ep_return_targets": (C.c_int, [_p, C.POINTER(_p)]),
    "dsv4_ep_return_published": (C.c_int, [_p, _p, _p]),
    "dsv4_ep_destroy": (C.c_int, [_p]),
    "dsv4_moe_combine_ordered": (C.c_int, [_p, _p, _i64, _i32, _i32, _p, _p]),
    "dsv4_moe_stage_times": (C.c_int, [_p, C.POINTER(C.c_float), _i32]),
    "dsv4_moe_debug_align": (C.c_int, [_p, C.POINTER(_p), C.POINTER(_p), C.POINTER(_p), C.POINTER(_p),
                                       C.POINTER(_p), C.POINTER(_p)]),
}


class Dsv4LibraryError(RuntimeError):
    pass


class Dsv4Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def lib():
    """Load (once) and return the CUDA library.  Raises when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise Dsv4LibraryError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python deepseek-v4-flash-offload_b200/build_ext.py` (there is no CPU fallback)")
            try:
                L = C.CDLL(LIB_PATH)
            except OSError as exc:
                raise Dsv4LibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != DSV4_OK:
        msg = lib().dsv4_last_error_string()
        raise Dsv4Error(int(rc), msg.decode() if msg else "unknown error")


def header_symbols(header_path: str | None = None) -> list[str]:
    """Names of every entry point declared in include/dsv4moe.h."""
    import re
    if header_path is None:
        header_path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(LIB_PATH))), "include",
                                   "dsv4moe.h")
    text = open(header_path).read()
    return sorted(set(re.findall(r"\b(dsv4_[a-z0-9_]+)\s*\(", text)))
