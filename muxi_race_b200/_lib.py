"""ctypes binding of ``libmoe_b200.so`` (the C ABI in ``include/moe_b200.h``).

The library is loaded from this package directory only. There is no fallback: if it is missing
or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

# enums mirrored from include/moe_b200.h
MOE_F16, MOE_BF16, MOE_F32, MOE_I32, MOE_I64, MOE_I8, MOE_F8E4M3 = range(7)
MOE_OK = 0
STATUS_NAMES = {
    -1: "MOE_ERR_INVALID_ARG",
    -2: "MOE_ERR_UNSUPPORTED",
    -3: "MOE_ERR_ALIGNMENT",
    -4: "MOE_ERR_CUDA",
    -5: "MOE_ERR_WORKSPACE",
}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_size = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "moe_version": (ctypes.c_char_p, []),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_device_status": (_int, [_c_void_p, _int, ctypes.POINTER(ctypes.c_uint32)]),
    "moe_set_profile_events": (_int, [ctypes.POINTER(_c_void_p), _int]),
    "moe_set_tile": (_int, [_int, ctypes.c_char_p]),
    "moe_set_a_path": (_int, [ctypes.c_char_p]),
    "moe_set_single_kernel": (_int, [_int]),
    "moe_ep_region_bytes": (_size, [_i64, _i64, _i64, _i64]),
    "moe_ep_region_alloc": (_int, [_size, ctypes.POINTER(_c_void_p)]),
    "moe_ep_region_free": (_int, [_c_void_p]),
    "moe_ep_ipc_get": (_int, [_c_void_p, _c_void_p]),
    "moe_ep_ipc_open": (_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "moe_ep_ipc_close": (_int, [_c_void_p]),
    "moe_ep_p2p_stage": (_int, [_c_void_p, _c_void_p, _c_void_p, _int, _c_void_p, _int, _i64, _i64, _i64, _i64, _i64,
                                _int, _c_void_p]),
    "moe_ep_p2p_barrier": (_int, [_c_void_p, _int, _int, ctypes.c_uint32, _c_void_p]),
    "moe_ep_p2p_workspace_bytes": (_size, [_i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "moe_ep_p2p_compute": (_int, [_c_void_p, _c_void_p, _int, _int, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64,
                                  _c_void_p, _c_void_p, _i64, _int, _c_void_p, _size, _c_void_p]),
    "moe_ep_p2p_combine": (_int, [_c_void_p, _int, _int, _i64, _i64, _i64, _i64, _c_void_p, _i64, _int, _c_void_p,
                                  _c_void_p]),
    "moe_ep_p2p_compute_push": (_int, [_c_void_p, _c_void_p, _int, _int, _i64, _i64, _i64, _i64, _c_void_p,
                                       _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _int, _c_void_p, _size,
                                       _c_void_p]),
    "moe_ep_p2p_push_prepare": (_int, [_c_void_p, _i64, _i64, _i64, _i64, _int, _int, _c_void_p]),
    "moe_ep_p2p_push_finish": (_int, [_c_void_p, _i64, _i64, _i64, _i64, _int, _i64, _int, _c_void_p, _c_void_p]),
    "moe_run_kernel_workspace_bytes": (_size, [_i64, _i64, _int]),
    "moe_run_kernel": (
        _int,
        [_c_void_p] * 5 + [_int] + [_c_void_p] * 5 + [_i64] * 6 + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_run_kernel_noalloc": (
        _int,
        [_c_void_p] * 5 + [_int] + [_c_void_p] * 5 + [_i64] * 6 + [_int, _c_void_p],
    ),
    "moe_max_padded_rows": (_i64, [_i64, _i64, _i64]),
    "moe_align_workspace_bytes": (_size, [_i64, _i64]),
    "moe_align": (_int, [_c_void_p, _int, _i64, _i64, _i64] + [_c_void_p] * 7 + [_c_void_p, _size, _c_void_p]),
    "moe_fused_workspace_bytes": (_size, [_i64] * 5 + [_int]),
    "moe_fused": (
        _int,
        [_c_void_p] * 4 + [_int, _c_void_p, _int, _c_void_p] + [_i64] * 5 + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_fused_ordered_workspace_bytes": (_size, [_i64] * 5 + [_int]),
    "moe_fused_ordered": (
        _int,
        [_c_void_p] * 4 + [_int, _c_void_p, _int, _c_void_p] + [_i64] * 5 + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_router_grouped_topk": (_int, [_c_void_p, _int, _c_void_p, _i64, _i64, _i64, _i64, _i64, _int,
                                       ctypes.c_float, _c_void_p, _c_void_p, _c_void_p]),
    "moe_router_topk": (_int, [_c_void_p, _int, _i64, _i64, _i64, _int, _c_void_p, _c_void_p, _c_void_p]),
    "moe_fused_router": (
        _int,
        [_c_void_p] * 4 + [_int, _int, _c_void_p, _c_void_p, _c_void_p] + [_i64] * 5
        + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_quantize_rows_int8": (_int, [_c_void_p, _int, _i64, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "moe_fused_int8_workspace_bytes": (_size, [_i64] * 5 + [_int]),
    "moe_quantize_rows_fp8": (_int, [_c_void_p, _int, _i64, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "moe_fused_fp8_workspace_bytes": (_size, [_i64] * 5 + [_int]),
    "moe_fused_fp8": (
        _int,
        [_c_void_p] * 6 + [_int, _c_void_p, _int, _c_void_p] + [_i64] * 5 + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_packed_weights_layout": (_int, [_i64, _i64, _i64, _int, ctypes.POINTER(_size), ctypes.POINTER(_size)]),
    "moe_pack_weights": (_int, [_c_void_p] * 3 + [_int, _i64, _i64, _i64, _int, _c_void_p, _size, _c_void_p]),
    "moe_fused_packed_workspace_bytes": (_size, [_i64] * 5 + [_int, _int]),
    "moe_fused_packed": (
        _int,
        [_c_void_p, _c_void_p, _int, _c_void_p, _int, _c_void_p, _int, _c_void_p] + [_i64] * 5
        + [_int, _c_void_p, _size, _c_void_p],
    ),
    "moe_ep_plan_workspace_bytes": (_size, [_i64, _i64]),
    "moe_ep_plan": (_int, [_c_void_p, _int, _i64, _i64, _c_void_p, _i64, _i64] + [_c_void_p] * 5 + [_c_void_p, _size, _c_void_p]),
    "moe_ep_pack": (
        _int,
        [_c_void_p, _c_void_p, _int, _c_void_p, _int, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p]
        + [_i64] * 4 + [_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
    "moe_ep_combine": (_int, [_c_void_p, _c_void_p, _i64, _i64, _i64, _int, _c_void_p, _c_void_p]),
    "moe_fused_int8": (
        _int,
        [_c_void_p] * 6 + [_int, _c_void_p, _int, _c_void_p] + [_i64] * 5 + [_int, _c_void_p, _size, _c_void_p],
    ),
}

_lock = threading.Lock()
_lib = None


class MoeError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load the CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m muxi_race_b200.build` "
                    "(the operators have no non-CUDA fallback)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(fn_name: str, code: int) -> None:
    if code != MOE_OK:
        msg = lib().moe_last_error().decode(errors="replace")
        raise MoeError(fn_name, code, msg)


def call(fn_name: str, *args) -> None:
    check(fn_name, getattr(lib(), fn_name)(*args))


def set_profile_events(events) -> None:
    """Install (list of torch.cuda.Event, each recorded once so its handle exists) or clear (None)
    the stage-boundary profiling events of the fused paths, for the calling thread."""
    global _prof_array
    if not events:
        _prof_array = None
        lib().moe_set_profile_events(None, 0)
        return
    _prof_array = (_c_void_p * len(events))(*[e.cuda_event for e in events])
    lib().moe_set_profile_events(_prof_array, len(events))


_prof_array = None


def set_a_path(name) -> None:
    """Select how the fused entry points' Stage1 loads its token rows for all later calls of the
    process: "tma" (stacked copy read by TMA boxes), "gather" (TMA tile::gather4 of the token
    rows inside Stage1) or "lsu"; None or "auto" restores the default."""
    call("moe_set_a_path", None if name is None else str(name).encode())


def set_single_kernel(on) -> None:
    """Whether later run_kernel / fused_moe calls of the process run Stage1 and Stage2 as one
    cooperative launch: True (wherever the single kernel applies), False (two launches) or None
    (automatic, the default: where it applies and the call averages fewer than 1.8 routing blocks
    per expert)."""
    call("moe_set_single_kernel", 2 if on is None else (1 if on else 0))


def set_tile(stage: int, name) -> None:
    """Force the grouped-GEMM tile configuration of `stage` (1, 2, or 0 for both) by name for all
    later calls of the process; None or "auto" restores the per-call choice."""
    call("moe_set_tile", int(stage), None if name is None else str(name).encode())
