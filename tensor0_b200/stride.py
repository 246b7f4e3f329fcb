"""Stride primitives on device storage: the host mirror of the reference's
``tensor0._stride`` FFI layer for this path.

The reference builds ``AffineRecord``s (src/tensor0/_stride/_layout.py:13-18),
encodes them as i64 layout words (_ffi/_descriptor.py:8-76) and calls one
native custom call per operation (_ffi/_calls.py:17-223).  Here the same words
build a ``Plan`` (the prepared state), whose packed device table is uploaded
once per device, and each ``execute_*`` is one stream-ordered call into the
sm_100a engine.  Storage is a torch CUDA tensor of shape ``[*batch, size]``;
torch only provides device memory and the stream.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from math import prod

import numpy as np
import torch

from . import _native

UINT64_MAX = (1 << 64) - 1
INT64_MIN = -(1 << 63)
INT64_MAX = (1 << 63) - 1

_STORAGE = {torch.float32: _native.F32, torch.float64: _native.F64,
            torch.complex64: _native.C64, torch.complex128: _native.C128}
_COEFFICIENT = {torch.int32: _native.S32, **_STORAGE}


@dataclass(frozen=True, slots=True)
class AffineRecord:
    """One strided sub-block pair (the reference's AffineRecord)."""

    logical_shape: tuple[int, ...]
    source_strides: tuple[int, ...]
    source_offset: int
    destination_strides: tuple[int, ...]
    destination_offset: int


def contiguous_strides(shape: tuple[int, ...]) -> tuple[int, ...]:
    """Row-major strides preserving empty-axis metadata (_layout.py:21-29)."""
    stride = 1
    result = [0] * len(shape)
    for axis in range(len(shape) - 1, -1, -1):
        result[axis] = stride
        stride *= max(shape[axis], 1)
    return tuple(result)


def encode_layout(records, *, source_size: int, output_size: int) -> np.ndarray:
    """v1 layout words ``[1, src_size, out_size, n, {rank, src_off, dst_off, shape, src_strides, dst_strides}...]``."""
    def size(value: int) -> int:
        if type(value) is not int or not 0 <= value <= INT64_MAX:
            raise ValueError("layout sizes and offsets must fit nonnegative int64")
        return value

    words = [1, size(source_size), size(output_size), len(records)]
    for record in records:
        rank = len(record.logical_shape)
        if len(record.source_strides) != rank or len(record.destination_strides) != rank:
            raise ValueError("layout shape and stride ranks must match")
        words.extend((rank, size(record.source_offset), size(record.destination_offset)))
        words.extend(size(extent) for extent in record.logical_shape)
        for stride in (*record.source_strides, *record.destination_strides):
            if type(stride) is not int or not INT64_MIN <= stride <= INT64_MAX:
                raise ValueError("layout strides must fit int64")
            words.append(stride)
    return np.asarray(words, dtype=np.int64)


def encode_layout_arrays(shape: np.ndarray, src_strides: np.ndarray, src_offsets: np.ndarray,
                         dst_strides: np.ndarray, dst_offsets: np.ndarray, *, source_size: int,
                         output_size: int) -> np.ndarray:
    """Vectorised ``encode_layout`` for records of one common rank (arrays [R, rank] / [R])."""
    shape = np.asarray(shape, np.int64)
    records, rank = shape.shape
    if records and (shape.min() < 0 or np.asarray(src_offsets).min() < 0 or np.asarray(dst_offsets).min() < 0):
        raise ValueError("layout sizes and offsets must fit nonnegative int64")
    body = np.empty((records, 3 + 3 * rank), np.int64)
    body[:, 0] = rank
    body[:, 1] = src_offsets
    body[:, 2] = dst_offsets
    body[:, 3:3 + rank] = shape
    body[:, 3 + rank:3 + 2 * rank] = src_strides
    body[:, 3 + 2 * rank:] = dst_strides
    head = np.array([1, source_size, output_size, records], np.int64)
    return np.concatenate([head, body.reshape(-1)])


def encode_reduction_layout(records, *, output_shapes, reduction_axes, source_size: int,
                            output_size: int) -> np.ndarray:
    """Reduction protocol words (u64 bit patterns as i64), _descriptor.py:41-76."""
    def offset(value: int) -> int:
        if type(value) is not int or not 0 <= value <= INT64_MAX:
            raise ValueError("reduction layout offsets must fit nonnegative int64")
        return value

    def usize(value: int) -> int:
        if type(value) is not int or not 0 <= value <= UINT64_MAX:
            raise ValueError("reduction layout sizes must fit uint64")
        return value

    words = [1, usize(source_size), usize(output_size), len(records)]
    for record, output_shape, axes in zip(records, output_shapes, reduction_axes, strict=True):
        rank = len(record.logical_shape)
        if any(len(field) != rank for field in (record.source_strides, output_shape, record.destination_strides, axes)):
            raise ValueError("reduction layout field ranks must match")
        if any(type(flag) is not bool for flag in axes):
            raise ValueError("reduction axis flags must be booleans")
        words.extend((rank, offset(record.source_offset), offset(record.destination_offset)))
        words.extend(usize(v) for v in record.logical_shape)
        words.extend(v & UINT64_MAX for v in record.source_strides)
        words.extend(usize(v) for v in output_shape)
        words.extend(v & UINT64_MAX for v in record.destination_strides)
        words.extend(int(flag) for flag in axes)
    return np.asarray(words, dtype=np.uint64).view(np.int64)


class Plan:
    """Prepared state of one operation over one layout (the reference's instantiate)."""

    def __init__(self, operation: int, words: np.ndarray, *, element_bytes: int,
                 coefficient_records=(), outputs_disjoint: bool = False, wide_offsets: bool = False,
                 conjugate_source: bool = False):
        self._lib = _native.lib()
        words = np.ascontiguousarray(words, dtype=np.int64)
        records = np.ascontiguousarray(np.asarray(coefficient_records, dtype=np.int64))
        handle = ctypes.c_void_p()
        err = _native.error_buffer()
        status = self._lib.t0b_plan_create(
            operation, words.ctypes.data_as(_native.c_i64p), words.size,
            records.ctypes.data_as(_native.c_i64p) if records.size else None, records.size,
            element_bytes, (_native.PLAN_OUTPUTS_DISJOINT if outputs_disjoint else 0)
            | (_native.PLAN_WIDE_OFFSETS if wide_offsets else 0)
            | (_native.PLAN_CONJUGATE_SOURCE if conjugate_source else 0),
            ctypes.byref(handle), err, len(err))
        _native.check(status, err)
        self._handle = handle
        self.operation = operation
        self.element_bytes = element_bytes
        self.coefficient_rows = int(records.size)
        count = ctypes.c_size_t()
        pointer = self._lib.t0b_plan_table(handle, ctypes.byref(count))
        self.table = np.ctypeslib.as_array(pointer, shape=(count.value,)).copy()
        info = _native.PlanInfo()
        self._lib.t0b_plan_query(handle, ctypes.byref(info))
        self.info = {name: int(getattr(info, name)) for name, _ in _native.PlanInfo._fields_}
        self.scratch_elements = int(self._lib.t0b_plan_scratch_elements(handle))
        self.matrix_elements = int(self._lib.t0b_plan_matrix_elements(handle))
        self._device_tables: dict[int, torch.Tensor] = {}

    @property
    def source_size(self) -> int:
        return self.info["source_size"]

    @property
    def output_size(self) -> int:
        return self.info["output_size"]

    def device_table(self, device: torch.device) -> torch.Tensor:
        index = torch.device(device).index or 0
        table = self._device_tables.get(index)
        if table is None:
            table = torch.from_numpy(self.table).to(device=torch.device("cuda", index))
            self._device_tables[index] = table
        return table

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.t0b_plan_destroy(handle)
            self._handle = None


def _storage_code(tensor: torch.Tensor) -> int:
    code = _STORAGE.get(tensor.dtype)
    if code is None:
        raise ValueError("CUDA stride storage supports only F32/F64/C64/C128")
    return code


def _require_cuda(*tensors: torch.Tensor) -> None:
    for tensor in tensors:
        if not tensor.is_cuda:
            raise ValueError("stride storage must be a CUDA tensor (there is no CPU fallback)")
        if not tensor.is_contiguous():
            raise ValueError("stride storage must be contiguous")


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _coefficients(values, batch_count: int, rows: int, dtype: torch.dtype, device) -> tuple[torch.Tensor, int]:
    """Coefficient rows [rows, count] as one device array (count 1 or batch_count)."""
    tensor = values if isinstance(values, torch.Tensor) else torch.as_tensor(values)
    tensor = tensor.to(device=device)
    if tensor.dtype not in _COEFFICIENT:
        tensor = tensor.to(dtype)
    if tensor.ndim == 1:
        tensor = tensor.reshape(rows, -1) if rows else tensor.reshape(0, 1)
    if tensor.ndim != 2 or tensor.shape[0] != rows or tensor.shape[1] not in (1, batch_count):
        raise ValueError("coefficients must be [records] or [records, 1 or batch]")
    return tensor.contiguous(), int(tensor.shape[1])


def execute_copy(source: torch.Tensor, plan: Plan, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Bit-preserving copy (the reference's execute_copy, _calls.py:49-72)."""
    _require_cuda(source)
    batch_shape = source.shape[:-1]
    batches = prod(batch_shape)
    if source.shape[-1] != plan.source_size:
        raise ValueError("copy buffer dimensions do not match layout")
    if out is None:
        out = torch.empty((*batch_shape, plan.output_size), dtype=source.dtype, device=source.device)
    _require_cuda(out)
    err = _native.error_buffer()
    status = _native.lib().t0b_copy(plan._handle, _storage_code(source), source.data_ptr(), out.data_ptr(), batches,
                                    plan.device_table(source.device).data_ptr(), _stream(source.device), err, len(err))
    _native.check(status, err)
    return out


def _sum(kind: str, source: torch.Tensor, plan: Plan, coefficients, coefficient_dtype, out, scratch):
    _require_cuda(source)
    batch_shape = source.shape[:-1]
    batches = prod(batch_shape)
    if source.shape[-1] != plan.source_size:
        raise ValueError(f"{kind} buffer dimensions do not match layout")
    if out is None:
        out = torch.empty((*batch_shape, plan.output_size), dtype=source.dtype, device=source.device)
    _require_cuda(out)
    coef_ptr, coef_code, coef_count = None, _native.S32, 1
    if plan.coefficient_rows:
        real = torch.float32 if source.dtype in (torch.float32, torch.complex64) else torch.float64
        tensor, coef_count = _coefficients(coefficients, batches, plan.coefficient_rows,
                                           coefficient_dtype or real, source.device)
        coef_ptr, coef_code = tensor.data_ptr(), _COEFFICIENT[tensor.dtype]
        keep = tensor  # noqa: F841  keeps the buffer alive through the launch
    if plan.scratch_elements and scratch is None:
        scratch = torch.empty((batches, plan.scratch_elements), dtype=source.dtype, device=source.device)
    err = _native.error_buffer()
    function = _native.lib().t0b_accumulation if kind == "accumulation" else _native.lib().t0b_reduction
    status = function(plan._handle, _storage_code(source), source.data_ptr(), out.data_ptr(), batches, coef_ptr,
                      coef_code, coef_count, scratch.data_ptr() if scratch is not None else None,
                      plan.device_table(source.device).data_ptr(), _stream(source.device), err, len(err))
    _native.check(status, err)
    return out


def execute_accumulation(source: torch.Tensor, plan: Plan, coefficients=None, *, coefficient_dtype=None,
                         out: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """out = 0; out[dst] += c * src[src] per record (_calls.py:155-174; accumulation.cu:92-163)."""
    return _sum("accumulation", source, plan, coefficients, coefficient_dtype, out, scratch)


def execute_reduction(source: torch.Tensor, plan: Plan, coefficients=None, *, coefficient_dtype=None,
                      out: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """Strided partial trace (_calls.py:177-223; reduction.cu:92-190)."""
    return _sum("reduction", source, plan, coefficients, coefficient_dtype, out, scratch)


def execute_update(source: torch.Tensor, base: torch.Tensor, alpha, beta, plan: Plan, *,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """out = base; out[dst] = alpha * src[src] + beta * base[dst] (_calls.py:74-124).

    ``out`` may be ``base`` itself (the reference's result aliases base).
    """
    _require_cuda(source, base)
    batch_shape = base.shape[:-1]
    if source.shape[:-1] != batch_shape:
        raise ValueError("update batch shapes must match")
    if source.dtype != base.dtype:
        raise ValueError("update source and base must share a storage dtype")
    batches = prod(batch_shape)
    if out is None:
        out = torch.empty_like(base)
    _require_cuda(out)
    real = torch.float32 if base.dtype in (torch.float32, torch.complex64) else torch.float64

    def coefficient(value):
        if isinstance(value, torch.Tensor):
            tensor = value if value.dtype in _COEFFICIENT else value.to(real)
        elif isinstance(value, complex) and value.imag != 0:
            tensor = torch.tensor([value], dtype=base.dtype)
        else:
            tensor = torch.tensor([complex(value).real if isinstance(value, complex) else value], dtype=real)
        if tensor.is_complex() and not base.is_complex():
            raise ValueError("unsupported CUDA coefficient dtype; expected S32 or matching real/complex precision")
        tensor = tensor.to(base.device).reshape(-1).contiguous()
        return tensor

    a, b = coefficient(alpha), coefficient(beta)
    err = _native.error_buffer()
    status = _native.lib().t0b_update(
        plan._handle, _storage_code(base), source.data_ptr(), base.data_ptr(), out.data_ptr(), batches,
        a.data_ptr(), _COEFFICIENT[a.dtype], a.numel(), b.data_ptr(), _COEFFICIENT[b.dtype], b.numel(),
        plan.device_table(base.device).data_ptr(), _stream(base.device), err, len(err))
    _native.check(status, err)
    return out


def execute_dot(left: torch.Tensor, right: torch.Tensor, plan: Plan, *, conjugate_left: bool = False,
                out: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """out[...] = sum of conj?(left[src]) * right[dst] over the plan's records
    (the reference's execute_dot, _calls.py:126-153; dot.cu:97-160)."""
    _require_cuda(left, right)
    if left.shape[:-1] != right.shape[:-1]:
        raise ValueError("dot batch shapes must match")
    if left.dtype != right.dtype:
        raise ValueError("dot inputs must share a storage dtype")
    if left.shape[-1] != plan.source_size or right.shape[-1] != plan.output_size:
        raise ValueError("dot buffer dimensions do not match layout")
    batch_shape = left.shape[:-1]
    batches = prod(batch_shape)
    if out is None:
        out = torch.empty(batch_shape, dtype=left.dtype, device=left.device)
    if scratch is None:
        scratch = torch.empty((max(batches, 1), plan.scratch_elements), dtype=left.dtype, device=left.device)
    err = _native.error_buffer()
    status = _native.lib().t0b_dot(plan._handle, _storage_code(left), left.data_ptr(), right.data_ptr(),
                                   out.data_ptr(), batches, int(bool(conjugate_left)), scratch.data_ptr(),
                                   plan.device_table(left.device).data_ptr(), _stream(left.device), err, len(err))
    _native.check(status, err)
    return out


def encode_grouped(source_blocks, destination_blocks, permutation, groups, *, source_size: int,
                   output_size: int) -> tuple[np.ndarray, list[np.ndarray]]:
    """Grouped-transform words and the groups' matrices, from the reference's
    inputs (_strided_grouped_transform, _stride/_tensor_ops.py:119-203).

    ``*_blocks`` are sub-blocks with ``sizes``, ``strides`` and ``offset``;
    ``groups`` carry ``src_indices``, ``dst_indices`` and ``transform``
    ([n_dst, n_src]).  Every group's destination blocks have the source block
    shape permuted by ``permutation``; the source strides are permuted into
    that order, as the reference's unpack records are."""
    permutation = tuple(int(p) for p in permutation)
    words = [1, int(source_size), int(output_size), len(groups)]
    matrices = []
    for group in groups:
        src_indices = tuple(int(i) for i in group.src_indices)
        dst_indices = tuple(int(i) for i in group.dst_indices)
        matrix = np.asarray(group.transform)
        if matrix.shape != (len(dst_indices), len(src_indices)):
            raise ValueError("generic tree transform matrix shape does not match its trees")
        source_sizes = tuple(int(n) for n in source_blocks[src_indices[0]].sizes)
        if sorted(permutation) != list(range(len(source_sizes))):
            raise ValueError("permutation does not match the source subblock rank")
        for index in src_indices:
            if tuple(int(n) for n in source_blocks[index].sizes) != source_sizes:
                raise ValueError("generic tree transform source subblock shapes are inconsistent")
        logical_shape = tuple(source_sizes[p] for p in permutation)
        for index in dst_indices:
            if tuple(int(n) for n in destination_blocks[index].sizes) != logical_shape:
                raise ValueError("generic tree transform destination subblock shapes are inconsistent")
        words += [len(logical_shape), len(src_indices), len(dst_indices), *logical_shape]
        for index in src_indices:
            block = source_blocks[index]
            strides = tuple(int(s) for s in block.strides)
            words += [int(block.offset), *(strides[p] for p in permutation)]
        for index in dst_indices:
            block = destination_blocks[index]
            words += [int(block.offset), *(int(s) for s in block.strides)]
        matrices.append(matrix.reshape(-1))
    return np.asarray(words, dtype=np.int64), matrices


def execute_grouped(source: torch.Tensor, plan: Plan, matrices: torch.Tensor, *,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """One grouped-transform launch over [..., source_size] storage; ``matrices``
    holds every group's row-major matrix in group order on the device."""
    _require_cuda(source, matrices)
    if source.shape[-1] != plan.source_size:
        raise ValueError("grouped buffer dimensions do not match layout")
    if matrices.numel() != plan.matrix_elements:
        raise ValueError("grouped matrix count does not match the plan")
    batch_shape = source.shape[:-1]
    batches = prod(batch_shape)
    if out is None:
        out = torch.empty((*batch_shape, plan.output_size), dtype=source.dtype, device=source.device)
    matrix_code = _STORAGE.get(matrices.dtype)
    if matrix_code is None:
        raise ValueError("grouped matrices must be F32/F64/C64/C128")
    err = _native.error_buffer()
    status = _native.lib().t0b_grouped_transform(
        plan._handle, _storage_code(source), source.data_ptr(), out.data_ptr(), batches, matrices.data_ptr(),
        matrix_code, plan.device_table(source.device).data_ptr(), _stream(source.device), err, len(err))
    _native.check(status, err)
    return out


_GROUPED_PLANS: dict[tuple[bytes, int], Plan] = {}
_GROUPED_MATRICES: dict[tuple, torch.Tensor] = {}


def grouped_transform(source: torch.Tensor, source_layout, destination_layout, result_dtype, permutation,
                      data) -> torch.Tensor:
    """The reference's _strided_grouped_transform (_tensor_ops.py:119-203) in
    one launch: single-tree groups follow the direct accumulation rule and
    multi-tree groups multiply their basis matrix into the source blocks.
    Storage keeps its dtype (F32/F64/C64/C128); ``result_dtype`` must be it."""
    if result_dtype is not None and torch.empty(0, dtype=source.dtype).numpy().dtype != np.dtype(result_dtype):
        raise NotImplementedError("the CUDA grouped transform keeps the storage dtype")
    element_bytes = source.element_size()
    words, matrices = encode_grouped(source_layout.subblockstructure, destination_layout.subblockstructure,
                                     permutation, data, source_size=source.shape[-1],
                                     output_size=destination_layout.total_dim)
    key = (words.tobytes(), element_bytes)
    plan = _GROUPED_PLANS.get(key)
    if plan is None:
        plan = Plan(_native.OP_GROUPED, words, element_bytes=element_bytes)
        if len(_GROUPED_PLANS) > 256:
            _GROUPED_PLANS.clear()
        _GROUPED_PLANS[key] = plan
    flat = np.concatenate(matrices) if matrices else np.zeros(0)
    single = source.dtype in (torch.float32, torch.complex64)
    if source.is_complex() and np.iscomplexobj(flat):
        flat = flat.astype(np.complex64 if single else np.complex128)
    else:
        flat = np.real(flat).astype(np.float32 if single else np.float64)
    # The basis matrices of a call site repeat from call to call: keep them on
    # the device (keyed by their bytes) instead of copying them every call.
    matrix_key = (key, str(source.device), flat.dtype.str, flat.tobytes())
    device_matrices = _GROUPED_MATRICES.get(matrix_key)
    if device_matrices is None:
        device_matrices = torch.from_numpy(np.ascontiguousarray(flat)).to(source.device)
        if len(_GROUPED_MATRICES) > 256:
            _GROUPED_MATRICES.clear()
        _GROUPED_MATRICES[matrix_key] = device_matrices
    return execute_grouped(source, plan, device_matrices)


def axpby(alpha, x: torch.Tensor, beta, y: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """alpha * x + beta * y elementwise (TensorMap.add)."""
    _require_cuda(x, y)
    if x.shape != y.shape or x.dtype != y.dtype:
        raise ValueError("add operands must share shape and dtype")
    if out is None:
        out = torch.empty_like(x)
    a, b = complex(alpha), complex(beta)
    err = _native.error_buffer()
    status = _native.lib().t0b_axpby(_storage_code(x), x.numel(), a.real, a.imag, x.data_ptr(), b.real, b.imag,
                                     y.data_ptr(), out.data_ptr(), _stream(x.device), err, len(err))
    _native.check(status, err)
    return out


class GemmPlan:
    """Grouped per-sector GEMM table (rows {m, n, k, a_off, b_off, c_off})."""

    def __init__(self, spec: np.ndarray):
        lib = _native.lib()
        spec = np.ascontiguousarray(np.asarray(spec, np.int64).reshape(-1, 6))
        self.sectors = spec.shape[0]
        self.table = np.zeros(lib.t0b_gemm_table_words(self.sectors), np.int64)
        err = _native.error_buffer()
        status = lib.t0b_gemm_table_build(self.sectors, spec.ctypes.data_as(_native.c_i64p),
                                          self.table.ctypes.data_as(_native.c_i64p), err, len(err))
        _native.check(status, err)
        self.spec = spec
        self.flops_real = int(2 * (spec[:, 0] * spec[:, 1] * spec[:, 2]).sum())
        self._device_tables: dict[int, torch.Tensor] = {}

    def device_table(self, device) -> torch.Tensor:
        index = torch.device(device).index or 0
        if index not in self._device_tables:
            self._device_tables[index] = torch.from_numpy(self.table).to(torch.device("cuda", index))
        return self._device_tables[index]


def sector_gemm(plan: GemmPlan, left: torch.Tensor, right: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """C_g = A_g @ B_g for every sector row of ``plan`` (linalg.py:533-566)."""
    _require_cuda(left, right, out)
    if not (left.dtype == right.dtype == out.dtype):
        raise ValueError("sector GEMM operands must share a dtype")
    err = _native.error_buffer()
    status = _native.lib().t0b_sector_gemm(
        _storage_code(out), plan.sectors, plan.table.ctypes.data_as(_native.c_i64p),
        plan.device_table(out.device).data_ptr(), left.data_ptr(), left.numel(), right.data_ptr(), right.numel(),
        out.data_ptr(), out.numel(), _stream(out.device), err, len(err))
    _native.check(status, err)
    return out


def kernel_launches() -> int:
    """Kernels the engine library has launched in this process."""
    return int(_native.lib().t0b_kernel_launches())
