"""Test infrastructure: ctypes bindings of the compiled reference (oracle/_ref).

``oracle/_ref/libt0ref.so`` is the reference's own native CPU stride executor
library, built from the reference sources by ``oracle/Makefile`` and driven by
``oracle/ref_driver.cc``.  Only tests, the smoke check and bench.py's CPU
baseline use it, as the checker; the product never loads it.
"""

from __future__ import annotations

import ctypes
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_ref" / "libt0ref.so"

_DTYPES = {np.dtype(np.float32): 11, np.dtype(np.float64): 12, np.dtype(np.complex64): 15,
           np.dtype(np.complex128): 18, np.dtype(np.int32): 4}
_LIB = None
c_i64p = ctypes.POINTER(ctypes.c_int64)


def available() -> bool:
    return LIBRARY.exists()


def reference_root() -> str:
    """Where the reference sources lie: $TENSOR0_REFERENCE, else the checkout
    this build recipe was written against."""
    return os.environ.get("TENSOR0_REFERENCE", "/root/reference")


def build(reference: str | None = None) -> Path:
    """Compile the reference executors (only where the reference sources exist)."""
    import subprocess
    reference = reference or reference_root()
    if not Path(reference).exists():
        raise RuntimeError("reference sources are not present; oracle/_ref cannot be rebuilt here")
    subprocess.run(["make", "-C", str(HERE), f"REFERENCE={reference}", f"-j{os.cpu_count() or 4}"], check=True)
    # The reference's CUDA companion for sm_100a (a same-GPU reference for the
    # tests); a toolchain that cannot build it leaves those tests skipped.
    companion = subprocess.run(["make", "-C", str(HERE), "cuda", f"REFERENCE={reference}",
                                f"-j{os.cpu_count() or 4}"])
    if companion.returncode != 0:
        print("oracle: the reference's CUDA companion did not build; its tests will skip", file=sys.stderr)
    return LIBRARY


def lib():
    global _LIB
    if _LIB is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is missing; build it with `make -C oracle`")
        _LIB = ctypes.CDLL(str(LIBRARY))
    return _LIB


class ReferenceError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _call(function, *args):
    err = ctypes.create_string_buffer(512)
    status = function(*args, err, ctypes.c_size_t(len(err)))
    if status != 0:
        raise ReferenceError(status, err.value.decode(errors="replace"))


def _words(words) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(words, dtype=np.int64))


def _coefficients(coefficients, coefficient_records):
    records = _words(coefficient_records)
    arrays = [np.ascontiguousarray(np.asarray(c)) for c in (coefficients or [])]
    if len(arrays) != records.size:
        raise ValueError("one coefficient per coefficient record")
    pointers = (ctypes.c_void_p * max(len(arrays), 1))(*[a.ctypes.data for a in arrays])
    dtypes = (ctypes.c_int * max(len(arrays), 1))(*[_DTYPES[a.dtype] for a in arrays])
    counts = (ctypes.c_int64 * max(len(arrays), 1))(*[(-1 if a.ndim == 0 else a.shape[0]) for a in arrays])
    return records, arrays, pointers, dtypes, counts


def set_threads(limit: int) -> None:
    lib().t0ref_set_worker_limit(ctypes.c_uint64(limit))


def prepare_layout(operation: int, words) -> np.ndarray:
    """The reference's Tensor0StridePrepareLayout (validated, sorted and fused words)."""
    words = _words(words)
    out = np.zeros(max(words.size, 8) * 2, np.int64)
    count = ctypes.c_size_t()
    err = ctypes.create_string_buffer(512)
    status = lib().t0ref_prepare_layout(ctypes.c_int32(operation), words.ctypes.data_as(c_i64p),
                                        ctypes.c_size_t(words.size), out.ctypes.data_as(c_i64p),
                                        ctypes.c_size_t(out.size), ctypes.byref(count), err,
                                        ctypes.c_size_t(len(err)))
    if status != 0:
        raise ReferenceError(status, err.value.decode(errors="replace"))
    return out[: count.value].copy()


def copy(words, source: np.ndarray, output_size: int, threads: int = 1) -> np.ndarray:
    source = np.ascontiguousarray(source)
    batches = int(np.prod(source.shape[:-1], dtype=np.int64))
    out = np.full((*source.shape[:-1], output_size), 7, dtype=source.dtype)
    words = _words(words)
    _call(lib().t0ref_copy, ctypes.c_int(_DTYPES[source.dtype]), words.ctypes.data_as(c_i64p),
          ctypes.c_size_t(words.size), ctypes.c_void_p(source.ctypes.data), ctypes.c_int64(source.shape[-1]),
          ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(output_size), ctypes.c_int64(batches),
          ctypes.c_int64(threads))
    return out


def accumulation(words, source: np.ndarray, output_size: int, coefficients=(), coefficient_records=(),
                 outputs_disjoint: bool = False, threads: int = 1, out: np.ndarray | None = None) -> np.ndarray:
    source = np.ascontiguousarray(source)
    batches = int(np.prod(source.shape[:-1], dtype=np.int64))
    if out is None:
        out = np.full((*source.shape[:-1], output_size), 7, dtype=source.dtype)
    words = _words(words)
    records, arrays, pointers, dtypes, counts = _coefficients(list(coefficients), coefficient_records)
    _call(lib().t0ref_accumulation, ctypes.c_int(_DTYPES[source.dtype]), words.ctypes.data_as(c_i64p),
          ctypes.c_size_t(words.size), records.ctypes.data_as(c_i64p), ctypes.c_size_t(records.size),
          pointers, dtypes, counts, ctypes.c_int64(int(outputs_disjoint)), ctypes.c_void_p(source.ctypes.data),
          ctypes.c_int64(source.shape[-1]), ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(output_size),
          ctypes.c_int64(batches), ctypes.c_int64(threads))
    del arrays
    return out


def reduction(words, source: np.ndarray, output_size: int, coefficients=(), coefficient_records=(),
              threads: int = 1) -> np.ndarray:
    source = np.ascontiguousarray(source)
    batches = int(np.prod(source.shape[:-1], dtype=np.int64))
    out = np.full((*source.shape[:-1], output_size), 7, dtype=source.dtype)
    data = np.ascontiguousarray(np.asarray(words, dtype=np.int64)).view(np.uint8)
    records, arrays, pointers, dtypes, counts = _coefficients(list(coefficients), coefficient_records)
    _call(lib().t0ref_reduction, ctypes.c_int(_DTYPES[source.dtype]),
          data.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), ctypes.c_size_t(data.size),
          records.ctypes.data_as(c_i64p), ctypes.c_size_t(records.size), pointers, dtypes, counts,
          ctypes.c_void_p(source.ctypes.data), ctypes.c_int64(source.shape[-1]), ctypes.c_void_p(out.ctypes.data),
          ctypes.c_int64(output_size), ctypes.c_int64(batches), ctypes.c_int64(threads))
    del arrays
    return out


def dot(words, left: np.ndarray, right: np.ndarray, conjugate_left: bool = False, threads: int = 1) -> np.ndarray:
    left = np.ascontiguousarray(left)
    right = np.ascontiguousarray(right)
    batches = int(np.prod(left.shape[:-1], dtype=np.int64))
    out = np.full(left.shape[:-1], 7, dtype=left.dtype)
    words = _words(words)
    _call(lib().t0ref_dot, ctypes.c_int(_DTYPES[left.dtype]), words.ctypes.data_as(c_i64p),
          ctypes.c_size_t(words.size), ctypes.c_int64(int(conjugate_left)), ctypes.c_void_p(left.ctypes.data),
          ctypes.c_int64(left.shape[-1]), ctypes.c_void_p(right.ctypes.data), ctypes.c_int64(right.shape[-1]),
          ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(batches), ctypes.c_int64(threads))
    return out


def update(words, source: np.ndarray, base: np.ndarray, alpha, beta, threads: int = 1,
           out: np.ndarray | None = None) -> np.ndarray:
    source = np.ascontiguousarray(source)
    base = np.ascontiguousarray(base)
    batches = int(np.prod(base.shape[:-1], dtype=np.int64))
    if out is None:
        out = np.full(base.shape, 7, dtype=base.dtype)
    a = np.ascontiguousarray(np.asarray(alpha))
    b = np.ascontiguousarray(np.asarray(beta))
    words = _words(words)
    _call(lib().t0ref_update, ctypes.c_int(_DTYPES[base.dtype]), words.ctypes.data_as(c_i64p),
          ctypes.c_size_t(words.size), ctypes.c_void_p(source.ctypes.data), ctypes.c_int64(source.shape[-1]),
          ctypes.c_void_p(base.ctypes.data), ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(base.shape[-1]),
          ctypes.c_void_p(a.ctypes.data), ctypes.c_int(_DTYPES[a.dtype]), ctypes.c_int64(-1 if a.ndim == 0 else a.shape[0]),
          ctypes.c_void_p(b.ctypes.data), ctypes.c_int(_DTYPES[b.dtype]), ctypes.c_int64(-1 if b.ndim == 0 else b.shape[0]),
          ctypes.c_int64(batches), ctypes.c_int64(threads))
    return out


class Prepared:
    """An instantiated accumulation (3) or update (1) call of the reference:
    decode, validation and preparation run once here, so that `execute_*`
    times execution alone, as one XLA executable reuses its prepared state."""

    def __init__(self, operation: int, words, coefficient_records=(), outputs_disjoint: bool = False):
        self._lib = lib()
        self._lib.t0ref_prepare.restype = ctypes.c_void_p
        self.words = _words(words)
        self.records = _words(coefficient_records)
        err = ctypes.create_string_buffer(512)
        handle = self._lib.t0ref_prepare(ctypes.c_int32(operation), self.words.ctypes.data_as(c_i64p),
                                         ctypes.c_size_t(self.words.size), self.records.ctypes.data_as(c_i64p),
                                         ctypes.c_size_t(self.records.size), ctypes.c_int64(int(outputs_disjoint)),
                                         err, ctypes.c_size_t(len(err)))
        if not handle:
            raise ReferenceError(1, err.value.decode(errors="replace"))
        self._handle = ctypes.c_void_p(handle)

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.t0ref_release(handle)
            self._handle = None

    def accumulation(self, source: np.ndarray, out: np.ndarray, coefficients=(), threads: int = 1) -> np.ndarray:
        batches = int(np.prod(source.shape[:-1], dtype=np.int64))
        _, arrays, pointers, dtypes, counts = _coefficients(list(coefficients), self.records)
        _call(self._lib.t0ref_execute_accumulation, self._handle, ctypes.c_int(_DTYPES[source.dtype]), pointers,
              dtypes, counts, ctypes.c_void_p(source.ctypes.data), ctypes.c_int64(source.shape[-1]),
              ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(out.shape[-1]), ctypes.c_int64(batches),
              ctypes.c_int64(threads))
        del arrays
        return out

    def update(self, source: np.ndarray, base: np.ndarray, out: np.ndarray, alpha, beta,
               threads: int = 1) -> np.ndarray:
        batches = int(np.prod(base.shape[:-1], dtype=np.int64))
        a = np.ascontiguousarray(np.asarray(alpha))
        b = np.ascontiguousarray(np.asarray(beta))
        _call(self._lib.t0ref_execute_update, self._handle, ctypes.c_int(_DTYPES[base.dtype]),
              ctypes.c_void_p(source.ctypes.data), ctypes.c_int64(source.shape[-1]), ctypes.c_void_p(base.ctypes.data),
              ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(base.shape[-1]), ctypes.c_void_p(a.ctypes.data),
              ctypes.c_int(_DTYPES[a.dtype]), ctypes.c_int64(-1 if a.ndim == 0 else a.shape[0]),
              ctypes.c_void_p(b.ctypes.data), ctypes.c_int(_DTYPES[b.dtype]),
              ctypes.c_int64(-1 if b.ndim == 0 else b.shape[0]), ctypes.c_int64(batches), ctypes.c_int64(threads))
        return out
