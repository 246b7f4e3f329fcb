"""The XLA FFI handler library: symbols, registration data and descriptors.

``_lib/libtensor0_b200_xla.so`` exports the symbol table of the reference's
CUDA companion library (crates/tensor0-py/src/stride.rs:284-330): per
operation an instantiate handler, the prepared-state type id / type info and
its created/destroyed counters, and one execute handler per storage dtype.
A JAX process registers them as the reference's registration module does
(src/tensor0/_stride/_ffi/_registration.py:57-242); ``register_with_jax``
does exactly that where JAX is installed.

``descriptor`` is the lowering-time half of the boundary: the reference
lowers with ``_stride_pack_owner_fiber`` (_ffi/_calls.py:230-240) and passes
the packed words as the descriptor operand; with this library the operand is
the engine's packed table for the same layout and element size.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from threading import Lock

import numpy as np

from . import _native, stride

OPERATIONS = ("copy", "update", "dot", "accumulation", "reduction")
DTYPE_SUFFIXES = ("F32", "F64", "C64", "C128")
_OPERATION_CODES = {
    "copy": _native.OP_COPY, "update": _native.OP_UPDATE, "dot": _native.OP_DOT,
    "accumulation": _native.OP_ACCUMULATION, "reduction": _native.OP_REDUCTION,
}
_ELEMENT_BYTES = {"float32": 4, "float64": 8, "complex64": 8, "complex128": 16}
_STORAGE_SUFFIXES = {"float32": "f32", "float64": "f64", "complex64": "c64", "complex128": "c128"}


def _capitalized(operation: str) -> str:
    return operation[0].upper() + operation[1:]


def handler_symbols() -> tuple[str, ...]:
    """Every symbol the library exports, in the reference's order per operation."""
    names = []
    for operation in OPERATIONS:
        stem = "Tensor0StrideCuda" + _capitalized(operation)
        names.append(stem + "InstantiateV1Handler")
        names += [stem + suffix + "V1Handler" for suffix in DTYPE_SUFFIXES]
        names += [stem + "Prepared" + part for part in ("TypeId", "TypeInfo", "CreatedCount", "DestroyedCount")]
    return tuple(names)


_library: ctypes.CDLL | None = None
_lock = Lock()


def library_path() -> Path:
    return Path(__file__).resolve().parent / "_lib" / "libtensor0_b200_xla.so"


def library() -> ctypes.CDLL:
    """Load the handler library (after the engine library it links)."""
    global _library
    with _lock:
        if _library is None:
            path = library_path()
            if not path.is_file():
                raise RuntimeError(f"XLA FFI handler library missing at {path}; build it with "
                                   "tensor0_b200.build.build_xla() where the XLA FFI headers are available")
            _native.lib()
            lib = ctypes.CDLL(str(path))
            for name in handler_symbols():
                function = getattr(lib, name)
                function.argtypes = []
                function.restype = ctypes.c_uint64 if name.endswith("Count") else ctypes.c_void_p
            _library = lib
        return _library


def registration() -> dict[str, int]:
    """Addresses keyed as the reference's ``_stride_cuda_registration()`` dict:
    ``{op}_instantiate``, ``{op}_{f32,f64,c64,c128}``, ``{op}_type_id`` and
    ``{op}_type_info``."""
    return registration_of(library())


def registration_of(lib: ctypes.CDLL) -> dict[str, int]:
    """The same addresses from any library exporting the symbol table (the
    reference's own companion too)."""
    for name in handler_symbols():
        function = getattr(lib, name)
        function.argtypes = []
        function.restype = ctypes.c_uint64 if name.endswith("Count") else ctypes.c_void_p
    table = {}
    for operation in OPERATIONS:
        stem = "Tensor0StrideCuda" + _capitalized(operation)
        table[f"{operation}_instantiate"] = getattr(lib, stem + "InstantiateV1Handler")()
        for suffix in DTYPE_SUFFIXES:
            table[f"{operation}_{suffix.lower()}"] = getattr(lib, stem + suffix + "V1Handler")()
        table[f"{operation}_type_id"] = getattr(lib, stem + "PreparedTypeId")()
        table[f"{operation}_type_info"] = getattr(lib, stem + "PreparedTypeInfo")()
    return table


def prepared_counts(operation: str, lib: ctypes.CDLL | None = None) -> tuple[int, int]:
    """(created, destroyed) prepared states of one operation (copy.cu:130-152),
    of this library or of another that exports the table."""
    lib = lib or library()
    stem = "Tensor0StrideCuda" + _capitalized(operation) + "Prepared"
    return int(getattr(lib, stem + "CreatedCount")()), int(getattr(lib, stem + "DestroyedCount")())


def descriptor(operation: str, words, dtype, coefficient_records=()) -> np.ndarray:
    """The descriptor operand for one call site: the engine's packed table for
    ``words`` at the storage dtype's element size (int64, rank one)."""
    name = np.dtype(dtype).name
    if name not in _ELEMENT_BYTES:
        raise NotImplementedError(f"native CUDA {operation} supports only F32/F64/C64/C128 storage; got {name}")
    plan = stride.Plan(_OPERATION_CODES[operation], np.asarray(words, dtype=np.int64),
                       element_bytes=_ELEMENT_BYTES[name], coefficient_records=coefficient_records)
    return plan.table.copy()


_REGISTERED: set[str] = set()


def register_with_jax(operation: str, dtype) -> str:
    """Register one target with JAX under the reference's target and type names."""
    import jax  # not installed in every image; registration needs it

    name = np.dtype(dtype).name
    suffix = _STORAGE_SUFFIXES.get(name)
    if suffix is None or operation not in OPERATIONS:
        raise NotImplementedError(f"native CUDA {operation} does not support {name}")
    target = f"tensor0_stride_{operation}_{suffix}_cuda_v1"
    with _lock:
        if target in _REGISTERED:
            return target
    table = registration()
    capsule = jax.ffi.pycapsule
    with _lock:
        if not any(t.startswith(f"tensor0_stride_{operation}_") for t in _REGISTERED):
            jax.ffi.register_ffi_type(
                f"tensor0_stride_cuda_{operation}_prepared_v1",
                {"type_id": capsule(ctypes.c_void_p(table[f"{operation}_type_id"])),
                 "type_info": capsule(ctypes.c_void_p(table[f"{operation}_type_info"]))},
                platform="CUDA")
        jax.ffi.register_ffi_target(
            target,
            {"instantiate": capsule(ctypes.c_void_p(table[f"{operation}_instantiate"])),
             "execute": capsule(ctypes.c_void_p(table[f"{operation}_{suffix}"]))},
            platform="CUDA", api_version=1)
        _REGISTERED.add(target)
    return target
