"""The XLA FFI handler library, driven through a ctypes XLA host.

CPU: the library exports the reference's symbol table
(crates/tensor0-py/src/stride.rs:284-330), and its instantiate handlers
decode attributes, validate layouts, report errors with XLA error codes and
count prepared states (copy.cu:130-152).  GPU: every execute handler, called
with XLA call frames over device buffers, matches the oracle (bit-exact for
copies, updates and unit-coefficient accumulations; within the
precision's tolerance for reductions and dots).
"""

import numpy as np
import pytest

from oracle import stride_oracle as so
from random_layouts import random_layout, random_reduction_layout
from tensor0_b200 import _native, build, stride, xla_ffi
from xla_host import (C64, C128, F32, F64, HandlerError, Host, S32, S64)

if not xla_ffi.library_path().exists() and build.xla_ffi_include() is None:
    pytest.skip("XLA FFI headers absent: the handler library is not built", allow_module_level=True)

CODES = {np.float32: F32, np.float64: F64, np.complex64: C64, np.complex128: C128}
SUFFIX = {np.float32: "f32", np.float64: "f64", np.complex64: "c64", np.complex128: "c128"}
DTYPES = [np.float32, np.float64, np.complex64, np.complex128]
TOL = {np.float32: 1e-6, np.complex64: 1e-6, np.float64: 1e-12, np.complex128: 1e-12}


@pytest.fixture(scope="module")
def host():
    build.build_xla()
    return Host(xla_ffi.library(), xla_ffi.registration())


def small_words(rng=None):
    rng = rng or np.random.default_rng(3)
    records = random_layout(rng, 600, 800, 12)
    return records, stride.encode_layout(records, source_size=600, output_size=800)


def test_exports_the_reference_symbol_table(host):
    names = xla_ffi.handler_symbols()
    assert len(names) == 45 and len(set(names)) == 45
    table = xla_ffi.registration()
    assert len(table) == 35 and all(table.values())
    handlers = [v for k, v in table.items() if not k.endswith(("type_id", "type_info"))]
    assert len(set(handlers)) == len(handlers) == 25
    assert len({table[f"{op}_type_id"] for op in xla_ffi.OPERATIONS}) == 5


def test_header_declares_exactly_the_exported_symbols(host):
    import re
    from pathlib import Path
    header = (Path(__file__).resolve().parents[1] / "include" / "tensor0_b200_xla.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    declared = set(re.findall(r"\b(Tensor0StrideCuda[A-Za-z0-9]+)\s*\(", header))
    assert declared == set(xla_ffi.handler_symbols())
    for name in declared:
        assert hasattr(xla_ffi.library(), name), name


def test_instantiate_counts_and_deletes_prepared_states(host):
    _, words = small_words()
    for operation, attrs in (("copy", {}), ("update", {}), ("dot", {"conjugate_left": 1}),
                             ("accumulation", {"coefficient_records": [0, 3]}),
                             ("reduction", {"coefficient_records": []})):
        layout = words
        if operation == "reduction":
            reduction, shapes, roles, size = random_reduction_layout(np.random.default_rng(5), 400, 6)
            layout = stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                                    source_size=400, output_size=size)
        created, destroyed = xla_ffi.prepared_counts(operation)
        ctx = host.instantiate(operation, layout=list(layout), **attrs)
        assert xla_ffi.prepared_counts(operation) == (created + 1, destroyed)
        host.destroy(operation, ctx)
        assert xla_ffi.prepared_counts(operation) == (created + 1, destroyed + 1)


def test_instantiate_rejects_bad_layouts_and_attributes(host):
    _, words = small_words()
    with pytest.raises(HandlerError) as error:
        host.instantiate("copy", layout=list(words[:-1]))
    assert error.value.code == 3
    with pytest.raises(HandlerError) as error:
        host.instantiate("dot", layout=list(words), conjugate_left=2)
    assert error.value.code == 3 and "conjugate_left" in error.value.message
    with pytest.raises(HandlerError) as error:   # the binding's attribute names are enforced
        host.instantiate("copy", layouts=list(words))
    assert error.value.code == 3
    with pytest.raises(HandlerError) as error:   # coefficient record beyond the layout
        host.instantiate("accumulation", layout=list(words), coefficient_records=[0, 99])
    assert error.value.code == 3


def test_execute_validates_before_any_device_work(host):
    """Shapes and the descriptor are checked on the host; nothing here reaches
    a device (the addresses are never dereferenced)."""
    _, words = small_words()
    ctx = host.instantiate("copy", layout=list(words))
    table = xla_ffi.descriptor("copy", words, np.float64)
    fake = 1 << 20
    with pytest.raises(HandlerError, match="descriptor operand shape"):
        host.execute("copy", "f64", ctx, [(F64, fake, (2, 600)), (S64, fake, (len(table) + 1,))],
                     [(F64, fake, (2, 800))])
    with pytest.raises(HandlerError, match="buffer dimensions"):
        host.execute("copy", "f64", ctx, [(F64, fake, (2, 601)), (S64, fake, (len(table),))],
                     [(F64, fake, (2, 800))])
    with pytest.raises(HandlerError, match="same-dtype"):
        host.execute("copy", "f64", ctx, [(F32, fake, (2, 600)), (S64, fake, (len(table),))],
                     [(F64, fake, (2, 800))])
    host.destroy("copy", ctx)


# ---------------------------------------------------------------------------
# Execute handlers on the GPU.

def _torch():
    import torch
    return torch


def cuda(array):
    return _torch().from_numpy(np.ascontiguousarray(array)).cuda()


def fetch(tensor):
    _torch().cuda.synchronize()
    return tensor.cpu().numpy()


def sample(rng, dtype, shape):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    return rng.standard_normal(shape).astype(dtype)


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def empty(shape, dtype):
    torch = _torch()
    return torch.from_numpy(np.zeros(shape, dtype)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_copy_update_and_accumulation_handlers_bit_exact(host, dtype):
    rng = np.random.default_rng(17)
    records, words = small_words(rng)
    x, base = sample(rng, dtype, (3, 600)), sample(rng, dtype, (3, 800))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64

    ctx = host.instantiate("copy", layout=list(words))
    out = empty((3, 800), dtype)
    host.execute("copy", SUFFIX[dtype], ctx, [cuda(x), cuda(xla_ffi.descriptor("copy", words, dtype))], [out])
    assert np.array_equal(bits(fetch(out)), bits(so.copy(words, x)))
    host.destroy("copy", ctx)

    ctx = host.instantiate("update", layout=list(words))
    table = cuda(xla_ffi.descriptor("update", words, dtype))
    alpha, beta = np.array(-2.0, real), np.array([0.5] * 3, real)
    out = empty((3, 800), dtype)
    host.execute("update", SUFFIX[dtype], ctx, [cuda(x), cuda(base), cuda(alpha), cuda(beta), table], [out])
    assert np.array_equal(bits(fetch(out)), bits(so.update(words, x, base, alpha, real(0.5))))
    host.destroy("update", ctx)

    selected = [0, 2, 5, 7]
    ctx = host.instantiate("accumulation", layout=list(words), coefficient_records=selected)
    table = xla_ffi.descriptor("accumulation", words, dtype, coefficient_records=selected)
    plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=selected)
    values = [np.array(1.0, real), np.array([2.0], real), np.array([0.5, -1.0, 3.0], real), np.array(2, np.int32)]
    out = empty((3, 800), dtype)
    scratch = empty((3, plan.scratch_elements), dtype)
    host.execute("accumulation", SUFFIX[dtype], ctx, [cuda(x), cuda(table), *[cuda(v) for v in values]],
                 [out, scratch])
    got = fetch(out)
    for b in range(3):
        per_record = [1.0] * len(records)
        for record, value in zip(selected, values):
            per_record[record] = value.reshape(-1)[0 if value.size == 1 else b]
        expected = so.accumulation(words, x[b:b + 1], [real(v) for v in per_record], np.arange(len(records)))
        assert np.array_equal(bits(got[b:b + 1]), bits(expected))
    host.destroy("accumulation", ctx)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_reduction_and_dot_handlers_within_tolerance(host, dtype):
    rng = np.random.default_rng(23)
    reduction, shapes, roles, size = random_reduction_layout(rng, 900, 16)
    words = stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                           source_size=900, output_size=size)
    x = sample(rng, dtype, (2, 900))
    selected = list(range(0, len(reduction), 2))
    coefficients = sample(rng, dtype, len(selected))
    ctx = host.instantiate("reduction", layout=list(words), coefficient_records=selected)
    plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=selected)
    out = empty((2, size), dtype)
    scratch = empty((2, plan.scratch_elements), dtype)
    host.execute("reduction", SUFFIX[dtype], ctx,
                 [cuda(x), cuda(plan.table), *[cuda(np.array(c)) for c in coefficients]], [out, scratch])
    per_record = [dtype(1)] * len(reduction)
    for record, value in zip(selected, coefficients):
        per_record[record] = value
    expected = so.reduction(words, x, per_record, np.arange(len(reduction)))
    scale = max(float(np.max(np.abs(expected))), 1e-300)
    assert float(np.max(np.abs(fetch(out) - expected))) / scale <= TOL[dtype]
    host.destroy("reduction", ctx)

    records = [stride.AffineRecord((30, 7), (7, 1), 0, (1, 30), 5), stride.AffineRecord((50,), (-2,), 400, (3,), 300)]
    words = stride.encode_layout(records, source_size=500, output_size=500)
    a, b = sample(rng, dtype, (4, 500)), sample(rng, dtype, (4, 500))
    plan = stride.Plan(_native.OP_DOT, words, element_bytes=np.dtype(dtype).itemsize)
    for conjugate in (0, 1):
        ctx = host.instantiate("dot", layout=list(words), conjugate_left=conjugate)
        out = empty((4,), dtype)
        scratch = empty((4, plan.scratch_elements), dtype)
        host.execute("dot", SUFFIX[dtype], ctx, [cuda(a), cuda(b), cuda(plan.table)], [out, scratch])
        expected = so.dot(words, a, b, bool(conjugate))
        magnitude = so.dot(words, np.abs(a), np.abs(b))
        assert np.all(np.abs(fetch(out) - expected) <= TOL[dtype] * np.maximum(magnitude, 1e-300))
        host.destroy("dot", ctx)


@pytest.mark.gpu
def test_coefficient_dtype_and_count_errors(host):
    rng = np.random.default_rng(29)
    _, words = small_words(rng)
    ctx = host.instantiate("accumulation", layout=list(words), coefficient_records=[1])
    table = cuda(xla_ffi.descriptor("accumulation", words, np.float32, coefficient_records=[1]))
    x = cuda(sample(rng, np.float32, (2, 600)))
    out, scratch = empty((2, 800), np.float32), empty((2, 0), np.float32)
    with pytest.raises(HandlerError, match="coefficient record count"):
        host.execute("accumulation", "f32", ctx, [x, table], [out, scratch])
    with pytest.raises(HandlerError, match="unsupported CUDA coefficient dtype"):
        host.execute("accumulation", "f32", ctx, [x, table, cuda(np.array(1.0))], [out, scratch])
    with pytest.raises(HandlerError, match="batch count"):
        host.execute("accumulation", "f32", ctx, [x, table, cuda(np.ones(3, np.float32))], [out, scratch])
    host.destroy("accumulation", ctx)
