"""ctypes binding of the sm_100a engine library (include/tensor0_b200.h).

The library is built in-tree by ``tensor0_b200.build`` (``__graft_entry__.build()``
runs it).  Loading fails loudly when it is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

from . import build as _build

LIBRARY_PATH = _build.LIBRARY

S32, F32, F64, C64, C128 = 4, 11, 12, 15, 18
OP_COPY, OP_UPDATE, OP_DOT, OP_ACCUMULATION, OP_REDUCTION, OP_GROUPED = 0, 1, 2, 3, 4, 5
PLAN_OUTPUTS_DISJOINT = 1
PLAN_WIDE_OFFSETS = 2
PLAN_CONJUGATE_SOURCE = 4

c_i64p = ctypes.POINTER(ctypes.c_int64)


class PlanInfo(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in (
        "source_size", "output_size", "records", "tiles", "kernels_per_call", "full_coverage", "bytes_moved")]


class NativeError(RuntimeError):
    """Internal failure reported by the engine (status 2)."""


_LIB: ctypes.CDLL | None = None

# Every symbol include/tensor0_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "t0b_version": (ctypes.c_char_p, []),
    "t0b_plan_create": (ctypes.c_int, [ctypes.c_int32, c_i64p, ctypes.c_size_t, c_i64p, ctypes.c_size_t,
                                       ctypes.c_int32, ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_plan_destroy": (None, [ctypes.c_void_p]),
    "t0b_plan_table": (c_i64p, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "t0b_plan_scratch_elements": (ctypes.c_uint64, [ctypes.c_void_p]),
    "t0b_plan_query": (None, [ctypes.c_void_p, ctypes.POINTER(PlanInfo)]),
    "t0b_plan_created_count": (ctypes.c_uint64, []),
    "t0b_plan_destroyed_count": (ctypes.c_uint64, []),
    "t0b_copy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_accumulation": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p,
                                        ctypes.c_size_t]),
    "t0b_reduction": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p,
                                     ctypes.c_size_t]),
    "t0b_reduction_static_scratch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                                    ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                                    ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
                                                    ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_update": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_dot": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                               ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                               ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_grouped_transform": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_plan_matrix_elements": (ctypes.c_uint64, [ctypes.c_void_p]),
    "t0b_axpby": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int64, ctypes.c_double, ctypes.c_double,
                                 ctypes.c_void_p, ctypes.c_double, ctypes.c_double, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_gemm_table_words": (ctypes.c_size_t, [ctypes.c_int64]),
    "t0b_gemm_table_build": (ctypes.c_int, [ctypes.c_int64, c_i64p, c_i64p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_sector_gemm": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int64, c_i64p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "t0b_kernel_launches": (ctypes.c_uint64, []),
}


def lib() -> ctypes.CDLL:
    """Load the engine library; raise if it was not built."""
    global _LIB
    if _LIB is None:
        if not Path(LIBRARY_PATH).exists():
            raise RuntimeError(
                f"tensor0_b200 engine library not found at {LIBRARY_PATH}; run tensor0_b200.build.build() "
                "(there is no CPU fallback for the stride engine)")
        handle = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            function = getattr(handle, name)
            function.restype = restype
            function.argtypes = argtypes
        _LIB = handle
    return _LIB


def check(status: int, buffer: ctypes.Array) -> None:
    """Raise ValueError for invalid arguments (1) and NativeError for internal errors (2)."""
    if status == 0:
        return
    message = buffer.value.decode(errors="replace")
    if status == 1:
        raise ValueError(message)
    raise NativeError(message)


def error_buffer() -> ctypes.Array:
    return ctypes.create_string_buffer(512)
