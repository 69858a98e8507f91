"""ctypes binding of libdflash_b200.so (the C ABI in ``include/dflash_b200.h``).

The shared library is the only compute path: if it is missing or a call
fails, the caller gets an exception -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p

DFL_OK = 0
STATUS_NAMES = {
    0: "DFL_OK",
    1: "DFL_ERR_NULL_POINTER",
    2: "DFL_ERR_BAD_SHAPE",
    3: "DFL_ERR_MISALIGNED",
    4: "DFL_ERR_WORKSPACE",
    5: "DFL_ERR_CUDA",
    6: "DFL_ERR_UNSUPPORTED",
    7: "DFL_ERR_SCRATCH_LIMIT",
}

# name -> (restype, argtypes); must match include/dflash_b200.h
SIGNATURES = {
    "dfl_status_string": (ctypes.c_char_p, [_c_int]),
    "dfl_version": (ctypes.c_char_p, []),
    "dfl_get_device_error": (_c_int, [ctypes.POINTER(_c_int)]),
    "dfl_gdn_tree_forward": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "dfl_tree_depthwise_conv1d": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                           _c_int, _c_int, _vp]),
    "dfl_verify_qmm_w4g64": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int, _c_int,
                                      _c_int, _vp]),
    "dfl_verify_qmm_w4g64_f16": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int, _c_int,
                                          _c_int, _vp]),
    "dfl_verify_qmm_w4g64_pairs": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int, _c_int,
                                            _c_int, _vp]),
    "dfl_verify_qmm_w4g64_pairs_f16": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int,
                                                _c_int, _c_int, _vp]),
    "dfl_repack_w4_pairs": (_c_int, [_vp, _vp, _c_size, _vp]),
    "dfl_verify_qmm_w4g64_pairs_silu": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int,
                                                 _c_int, _c_int, _vp]),
    "dfl_verify_qmm_w4g64_pairs_silu_f16": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size,
                                                     _c_int, _c_int, _c_int, _vp]),
    "dfl_qmm_stream_k_ranges": (_c_int, [_c_int, _c_int, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "dfl_verify_qmm_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "dfl_verify_qmm_w4g64_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                              _vp]),
    "dfl_gdn_tape_replay": (_c_int, [_vp, _vp, _c_int, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int,
                                     _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "dfl_gdn_forward_tape": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "dfl_lmhead_argmax": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                   _c_size, _vp]),
    "dfl_lmhead_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "dfl_lmhead_accept": (_c_int, [_vp, _c_int, _vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]),
    "dfl_match_acceptance": (_c_int, [_vp, _vp, _c_int, _c_int, _vp, _vp]),
    "dfl_moe_route": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp]),
    "dfl_moe_route_table_ints": (_c_size, [_c_int]),
    "dfl_moe_qmm_w4g64": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                   _c_int, _vp, _c_size, _vp]),
    "dfl_moe_qmm_w4g64_silu": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                        _c_int, _c_int, _vp, _c_size, _vp]),
    "dfl_verify_qmm_w4g64_silu": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int, _c_int,
                                           _c_int, _vp]),
    "dfl_moe_qmm_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "dfl_silu_mul_bf16": (_c_int, [_vp, _vp, _vp, _c_int, _vp]),
    "dfl_silu_mul_rows_bf16": (_c_int, [_vp, _vp, _c_int, _vp, _c_int, _c_int, _vp]),
    "dfl_moe_combine": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "dfl_moe_sorted_route_ints": (_c_size, []),
    "dfl_moe_sort_pairs": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp, _vp,
                                    _vp]),
    "dfl_moe_route_sorted": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp,
                                      _vp, _vp, _vp, _vp]),
    "dfl_w4_tiled_bytes": (_c_size, [_c_int, _c_int]),
    "dfl_repack_w4_tiled": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "dfl_qmm_plan_bytes": (_c_size, [_c_int]),
    "dfl_qmm_plan_encode": (_c_int, [_vp, _c_int, _vp, _c_size]),
    "dfl_qmm_plan_workspace_bytes": (_c_size, [_vp, ctypes.POINTER(_c_int)]),
    "dfl_qmm_plan_run": (_c_int, [_vp, _vp, _vp, _c_size, _vp]),
    "dfl_qmm_plan_set_test_fault": (_c_int, [_vp, _c_int, ctypes.c_uint64]),
    "dfl_qmm_plan_last_timeout": (_c_int, [_vp, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                           ctypes.POINTER(_c_int)]),
}

_lock = threading.Lock()
_lib = None


class DflashError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{fn} failed: {name} ({status_string(status)})")


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the library, with argtypes set for every symbol."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is not built ({p}); run __graft_entry__.build() -- "
                "dflash-b200 has no fallback path")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().dfl_status_string(int(status)).decode()
    except Exception:  # pragma: no cover - library missing
        return STATUS_NAMES.get(status, "unknown")


def check(fn: str, status: int) -> None:
    if status != DFL_OK:
        raise DflashError(fn, status)


def device_error() -> int:
    """Read and clear the kernels' device error word (synchronises the device).

    A non-zero word also zeroes the package's cached workspaces again: a
    kernel that timed out may have left split-K partial sums in them.
    """
    v = _c_int(0)
    check("dfl_get_device_error", load().dfl_get_device_error(ctypes.byref(v)))
    if v.value != 0:
        from ._runtime import reset_workspaces

        reset_workspaces()
    return int(v.value)
