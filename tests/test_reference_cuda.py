"""The reference's own CUDA companion as a same-GPU reference.

``make -C oracle cuda`` builds crates/tensor0-cuda12/native/cuda/*.cu (with
the layout decoder it links) for sm_100a into oracle/_ref/libt0ref_cuda.so.
Its 45 XLA FFI symbols are the table this library's handler library exports
(crates/tensor0-py/src/stride.rs:284-330), so the same ctypes XLA host drives
both.  Call sites are assembled as the reference's lowering does
(src/tensor0/_stride/_ffi/_calls.py:229-293): the layout attribute is the
prepared words (Tensor0StridePrepareLayout), the reference's descriptor
operand its packed owner/fiber words (Tensor0StridePackOwnerFiber,
descriptor.cc:407-440), its accumulation scratch sized by
Tensor0StrideSumScratchCapacity; this library gets its own packed table.

CPU: the companion exports the table and packs descriptors, and both
libraries' instantiate handlers reject the same malformed call sites with the
same error code and message.  GPU: on the same
inputs, this library's copy, update and accumulation handlers reproduce the
companion's results bit for bit, on random layouts and on the U(1) four-leg
permute workload, whose device time per call is printed for both; its dot and
reduction handlers agree within the precision (their summation orders differ),
the reduction on the Z2 x U(1) partial trace, timed for both too.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest

from random_layouts import random_layout, random_reduction_layout
from tensor0_b200 import _native, build, stride, xla_ffi
from xla_host import HandlerError, Host

LIBRARY = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libt0ref_cuda.so"
if not LIBRARY.is_file():
    pytest.skip("the reference's CUDA companion is not built (make -C oracle cuda)", allow_module_level=True)
if not xla_ffi.library_path().exists() and build.xla_ffi_include() is None:
    pytest.skip("XLA FFI headers absent: the handler library is not built", allow_module_level=True)

OPERATIONS = {"copy": 0, "update": 1, "dot": 2, "accumulation": 3, "reduction": 4}
SUFFIX = {np.float32: "f32", np.float64: "f64", np.complex64: "c64", np.complex128: "c128"}
DTYPES = list(SUFFIX)
_RECEIVE = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64), ctypes.c_size_t,
                            ctypes.c_char_p, ctypes.c_size_t)


@pytest.fixture(scope="module")
def companion():
    import torch  # noqa: F401  (the companion forwards to the resident libcudart.so.12 torch loads)
    lib = ctypes.CDLL(str(LIBRARY))
    for name in ("Tensor0StridePrepareLayout", "Tensor0StridePackOwnerFiber", "Tensor0StrideSumScratchCapacity"):
        function = getattr(lib, name)
        function.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, _RECEIVE]
        function.restype = None
    lib.Tensor0StrideDotScratchCapacity.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, _RECEIVE]
    lib.Tensor0StrideDotScratchCapacity.restype = None
    return lib


@pytest.fixture(scope="module")
def hosts(companion):
    build.build_xla()
    return Host(companion, xla_ffi.registration_of(companion)), Host(xla_ffi.library(), xla_ffi.registration())


def native_words(lib, entry: str, operation: str, words) -> np.ndarray:
    """One of the companion's layout entry points, called as stride.rs:632-700 does."""
    result = {}

    def receive(context, status, data, count, message, length):
        result["status"] = status
        result["words"] = np.array([data[i] for i in range(count)], np.int64)
        result["message"] = ctypes.string_at(message, length).decode() if length else ""

    callback = _RECEIVE(receive)
    words = np.ascontiguousarray(words, np.int64)
    if entry == "Tensor0StrideDotScratchCapacity":   # the one entry without an operation code
        lib.Tensor0StrideDotScratchCapacity(words.ctypes.data, len(words), None, callback)
    else:
        getattr(lib, entry)(OPERATIONS[operation], words.ctypes.data, len(words), None, callback)
    if result.get("status") != 0:
        raise ValueError(result.get("message", "no result"))
    return result["words"]


def test_companion_exports_the_handler_table(companion):
    table = xla_ffi.registration_of(companion)
    assert len(table) == 35 and all(table.values())
    assert table != xla_ffi.registration()   # a separate library, not this one resolved twice


def test_companion_packs_and_rejects_layouts(companion):
    records = random_layout(np.random.default_rng(3), 600, 800, 12)
    words = stride.encode_layout(records, source_size=600, output_size=800)
    prepared = native_words(companion, "Tensor0StridePrepareLayout", "copy", words)
    packed = native_words(companion, "Tensor0StridePackOwnerFiber", "copy", prepared)
    assert len(packed) > 0
    capacity = native_words(companion, "Tensor0StrideSumScratchCapacity", "accumulation", prepared)
    assert capacity.shape == (1,) and capacity[0] >= 0
    with pytest.raises(ValueError):
        native_words(companion, "Tensor0StridePackOwnerFiber", "copy", prepared[:-1])


def _instantiate_error(host, operation, attrs):
    try:
        ctx = host.instantiate(operation, **attrs)
    except HandlerError as error:
        message = error.message
        for prefix in ("tensor0-native: ", "tensor0-b200: "):
            message = message.removeprefix(prefix)
        return error.code, message
    host.destroy(operation, ctx)
    return None


def test_instantiate_errors_match_the_companion(hosts):
    """Malformed call sites fail in both libraries' instantiate handlers (host
    code only) with the same XLA error code and the same message after each
    library's name prefix; what the companion accepts, this library accepts."""
    rng = np.random.default_rng(3)
    words = list(stride.encode_layout(random_layout(rng, 600, 800, 12), source_size=600, output_size=800))
    reduction, shapes, roles, size = random_reduction_layout(np.random.default_rng(5), 400, 6)
    reduction_words = list(stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                                          source_size=400, output_size=size))
    cases = [
        ("copy", {"layout": words[:-1]}),
        ("copy", {"layout": []}),
        ("copy", {"layouts": words}),
        ("update", {"layout": words[:3]}),
        ("dot", {"layout": words, "conjugate_left": 2}),
        ("accumulation", {"layout": words, "coefficient_records": [0, 99]}),
        ("accumulation", {"layout": words, "coefficient_records": [3, 3]}),
        ("accumulation", {"layout": words, "coefficient_records": [-1]}),
        ("reduction", {"layout": reduction_words, "coefficient_records": [len(reduction)]}),
        ("reduction", {"layout": reduction_words[:-2], "coefficient_records": []}),
    ]
    # Raw words {version, source size, output size, records, then per record
    # rank, source offset, output offset, shape, source strides, output strides}.
    record = [2, 0, 0, 3, 4, 4, 1, 1, 3]
    cases += [(operation, {"layout": layout}) for operation in ("copy", "update") for layout in (
        [1, 11, 12, 1, *record],                         # source out of bounds
        [1, 12, 11, 1, *record],                         # output out of bounds
        [1, 12, 12, 2, *record, 1, 0, 0, 2, 1, 1],       # two records write output 0 and 1: accepted by both
        [1, 12, 12, 1, 2, 0, 0, -3, 4, 4, 1, 1, 3],      # negative extent
        [2, 12, 12, 1, *record],                         # unknown version
        [1, 12, 12, 2, *record],                         # fewer records than announced
    )]
    reference, ours = hosts
    for operation, attrs in cases:
        expected = _instantiate_error(reference, operation, attrs)
        assert _instantiate_error(ours, operation, attrs) == expected, (operation, attrs, expected)


def test_prepared_state_counts_move_alike(hosts, companion):
    """Per operation, an instantiate creates one prepared state and its
    teardown destroys it, in both libraries; a rejected instantiate creates
    none (copy.cu:130-152)."""
    records = random_layout(np.random.default_rng(3), 600, 800, 12)
    words = list(stride.encode_layout(records, source_size=600, output_size=800))
    reduction, shapes, roles, size = random_reduction_layout(np.random.default_rng(5), 400, 6)
    reduction_words = list(stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                                          source_size=400, output_size=size))
    sites = {"copy": {"layout": words}, "update": {"layout": words},
             "dot": {"layout": words, "conjugate_left": 1},
             "accumulation": {"layout": words, "coefficient_records": [0, 3]},
             "reduction": {"layout": reduction_words, "coefficient_records": []}}
    for operation, attrs in sites.items():
        moves = []
        for host, lib in zip(hosts, (companion, xla_ffi.library())):
            before = xla_ffi.prepared_counts(operation, lib)
            ctx = host.instantiate(operation, **attrs)
            created = xla_ffi.prepared_counts(operation, lib)
            host.destroy(operation, ctx)
            destroyed = xla_ffi.prepared_counts(operation, lib)
            with pytest.raises(HandlerError):
                host.instantiate(operation, **{**attrs, "layout": attrs["layout"][:-1]})
            rejected = xla_ffi.prepared_counts(operation, lib)
            moves.append([tuple(b - a for a, b in zip(before, after)) for after in (created, destroyed, rejected)])
        assert moves[0] == moves[1] == [(1, 0), (1, 1), (1, 1)], (operation, moves)


def test_execute_validation_matches_the_companion(hosts, companion):
    """Execute frames that fail the host-side checks (buffer ranks, dimensions,
    dtypes, descriptor length, coefficient operands) fail in both libraries
    with the same error code and message; the addresses are never
    dereferenced, so no device is needed."""
    from xla_host import F32, F64, S32, S64
    records = random_layout(np.random.default_rng(3), 600, 800, 12)
    raw = stride.encode_layout(records, source_size=600, output_size=800)
    reference, ours = hosts
    for operation, attrs in (("copy", {}), ("update", {}), ("accumulation", {"coefficient_records": [1]})):
        words = native_words(companion, "Tensor0StridePrepareLayout", operation, raw)
        lengths = (len(native_words(companion, "Tensor0StridePackOwnerFiber", operation, words)),
                   len(xla_ffi.descriptor(operation, words, np.float64, **attrs)))
        capacity = scratch_elements = 0
        if operation == "accumulation":
            capacity = int(native_words(companion, "Tensor0StrideSumScratchCapacity", operation, words)[0])
            scratch_elements = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=8,
                                           coefficient_records=[1]).scratch_elements

        def frame(side, x=(2, 600), out=(2, 800), x_dtype=F64, extra_words=0, coefficients=((F64, (2,)),)):
            # Every buffer at its own address, 1 GiB apart, so that no overlap check fires.
            address = iter(range(1 << 30, 1 << 40, 1 << 30))
            table = (S64, next(address), (lengths[side] + extra_words,))
            source, result = (x_dtype, next(address), x), (F64, next(address), out)
            if operation == "copy":
                return [source, table], [result]
            if operation == "update":
                return [source, (F64, next(address), out), (F64, next(address), ()), (F64, next(address), (2,)),
                        table], [result]
            scratch = (F64, next(address), (out[0], (capacity, scratch_elements)[side]))
            return [source, table, *[(c, next(address), d) for c, d in coefficients]], [result, scratch]

        cases = [dict(x=(2, 601)), dict(out=(2, 801)), dict(x=(3, 600)), dict(x=(600,)), dict(x_dtype=F32),
                 dict(extra_words=1)]
        if operation == "accumulation":
            cases += [dict(coefficients=()), dict(coefficients=((F64, (3,)),)), dict(coefficients=((S64, ()),)),
                      dict(coefficients=((S32, ()), (S32, ())))]
        for case in cases:
            results = []
            for side, host in enumerate(hosts):
                ctx = host.instantiate(operation, layout=list(words), **attrs)
                args, rets = frame(side, **case)
                with pytest.raises(HandlerError) as error:
                    host.execute(operation, "f64", ctx, args, rets)
                host.destroy(operation, ctx)
                results.append((error.value.code, error.value.message.removeprefix("tensor0-native: ")))
            assert results[0] == results[1], (operation, case, results)


def test_reduction_and_dot_execute_validation_matches_the_companion(hosts, companion):
    """The same comparison for the reduction and dot handlers."""
    from xla_host import F32, F64, S64
    reduction, shapes, roles, size = random_reduction_layout(np.random.default_rng(5), 400, 6)
    reduction_raw = stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                                   source_size=400, output_size=size)
    dot_raw = stride.encode_layout([stride.AffineRecord((30, 7), (7, 1), 0, (1, 30), 5)], source_size=500,
                                   output_size=500)
    for operation, raw, n_in, n_out in (("reduction", reduction_raw, 400, size), ("dot", dot_raw, 500, None)):
        words = native_words(companion, "Tensor0StridePrepareLayout", operation, raw)
        entry = "Tensor0StrideSumScratchCapacity" if operation == "reduction" else "Tensor0StrideDotScratchCapacity"
        capacity = int(native_words(companion, entry, operation, words)[0])
        plan = stride.Plan(_native.OP_REDUCTION if operation == "reduction" else _native.OP_DOT, words,
                           element_bytes=8)
        lengths = (len(native_words(companion, "Tensor0StridePackOwnerFiber", operation, words)),
                   len(xla_ffi.descriptor(operation, words, np.float64)))

        def frame(side, x=(2, n_in), out=None, dtype=F64, extra_words=0, batches=2):
            address = iter(range(1 << 30, 1 << 40, 1 << 30))
            table = (S64, next(address), (lengths[side] + extra_words,))
            scratch = (F64, next(address), (batches, (capacity, plan.scratch_elements)[side]))
            if operation == "reduction":
                result = (F64, next(address), out or (2, n_out))
                return [(dtype, next(address), x), table], [result, scratch]
            result = (F64, next(address), out or (2,))
            return [(dtype, next(address), x), (F64, next(address), (2, n_in)), table], [result, scratch]

        cases = [dict(x=(2, n_in + 1)), dict(x=(3, n_in)), dict(x=(n_in,)), dict(dtype=F32), dict(extra_words=1),
                 dict(out=(3,) if operation == "dot" else (2, n_out + 1)), dict(batches=3)]
        for case in cases:
            results = []
            for side, host in enumerate(hosts):
                # The attributes the reference's lowering always passes
                # (_calls.py:309-327); the companion's dot instantiate does not
                # survive a missing conjugate_left.
                extra = {"coefficient_records": []} if operation == "reduction" else {"conjugate_left": 0}
                ctx = host.instantiate(operation, layout=list(words), **extra)
                args, rets = frame(side, **case)
                with pytest.raises(HandlerError) as error:
                    host.execute(operation, "f64", ctx, args, rets)
                host.destroy(operation, ctx)
                results.append((error.value.code, error.value.message.removeprefix("tensor0-native: ")))
            assert results[0] == results[1], (operation, case, results)


# ---------------------------------------------------------------------------
# GPU: this library against the companion on the same inputs.

def _torch():
    import torch
    return torch


def cuda(array):
    return _torch().from_numpy(np.ascontiguousarray(array)).cuda()


def bits(tensor):
    _torch().cuda.synchronize()
    return np.ascontiguousarray(tensor.cpu().numpy()).view(np.uint8)


def sample(rng, dtype, shape):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    return rng.standard_normal(shape).astype(dtype)


class Site:
    """One call site on both libraries: instantiate, execute, destroy."""

    def __init__(self, hosts, companion, operation, words, dtype, coefficient_records=None, **attrs):
        self.reference, self.ours = hosts
        self.operation, self.dtype = operation, dtype
        self.words = native_words(companion, "Tensor0StridePrepareLayout", operation, words)
        if coefficient_records is not None:
            attrs["coefficient_records"] = list(coefficient_records)
        self.contexts = (self.reference.instantiate(operation, layout=list(self.words), **attrs),
                         self.ours.instantiate(operation, layout=list(self.words), **attrs))
        self.tables = (cuda(native_words(companion, "Tensor0StridePackOwnerFiber", operation, self.words)),
                       cuda(xla_ffi.descriptor(operation, self.words, dtype,
                                               coefficient_records=coefficient_records or ())))
        entry = {"accumulation": "Tensor0StrideSumScratchCapacity", "reduction": "Tensor0StrideSumScratchCapacity",
                 "dot": "Tensor0StrideDotScratchCapacity"}.get(operation)
        self.capacity = int(native_words(companion, entry, operation, self.words)[0]) if entry else 0

    def call(self, side, args, rets):
        host = (self.reference, self.ours)[side]
        host.execute(self.operation, SUFFIX[self.dtype], self.contexts[side], args(self.tables[side]), rets)

    def close(self):
        self.reference.destroy(self.operation, self.contexts[0])
        self.ours.destroy(self.operation, self.contexts[1])


def scratch_for(site, side, batches, plan_elements):
    elements = site.capacity if side == 0 else plan_elements
    return _torch().zeros((batches, elements), dtype=_torch_dtype(site.dtype), device="cuda")


def _torch_dtype(dtype):
    torch = _torch()
    return {np.float32: torch.float32, np.float64: torch.float64, np.complex64: torch.complex64,
            np.complex128: torch.complex128}[dtype]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
def test_handlers_match_the_reference_companion_bit_for_bit(hosts, companion, dtype):
    torch = _torch()
    rng = np.random.default_rng(41)
    records = random_layout(rng, 600, 800, 12)
    words = stride.encode_layout(records, source_size=600, output_size=800)
    x, base = cuda(sample(rng, dtype, (3, 600))), cuda(sample(rng, dtype, (3, 800)))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    zeros = lambda: torch.zeros((3, 800), dtype=_torch_dtype(dtype), device="cuda")  # noqa: E731

    site = Site(hosts, companion, "copy", words, dtype)
    outs = [zeros(), zeros()]
    for side in (0, 1):
        site.call(side, lambda table: [x, table], [outs[side]])
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    site.close()

    site = Site(hosts, companion, "update", words, dtype)
    alpha, beta = cuda(np.array(-2.0, real)), cuda(np.array([0.5, 0.0, 1.0], real))
    outs = [zeros(), zeros()]
    for side in (0, 1):
        site.call(side, lambda table: [x, base, alpha, beta, table], [outs[side]])
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    site.close()

    selected = [0, 2, 5, 7]
    site = Site(hosts, companion, "accumulation", words, dtype, coefficient_records=selected)
    plan = stride.Plan(_native.OP_ACCUMULATION, site.words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=selected)
    values = [cuda(v) for v in (np.array(1.0, real), np.array([2.0], real), np.array([0.5, -1.0, 3.0], real),
                                np.array(2, np.int32))]
    outs = [zeros(), zeros()]
    for side in (0, 1):
        site.call(side, lambda table: [x, table, *values], [outs[side], scratch_for(site, side, 3, plan.scratch_elements)])
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    site.close()

    # Dot (inner / norm): the summation orders differ, so within the precision.
    records = [stride.AffineRecord((30, 7), (7, 1), 0, (1, 30), 5), stride.AffineRecord((50,), (-2,), 400, (3,), 300)]
    words = stride.encode_layout(records, source_size=500, output_size=500)
    a, b = cuda(sample(rng, dtype, (4, 500))), cuda(sample(rng, dtype, (4, 500)))
    tolerance = 1e-6 if real == np.float32 else 1e-12
    for conjugate in (0, 1):
        site = Site(hosts, companion, "dot", words, dtype, conjugate_left=conjugate)
        plan = stride.Plan(_native.OP_DOT, site.words, element_bytes=np.dtype(dtype).itemsize)
        outs = [torch.zeros(4, dtype=_torch_dtype(dtype), device="cuda") for _ in (0, 1)]
        for side in (0, 1):
            site.call(side, lambda table: [a, b, table], [outs[side], scratch_for(site, side, 4, plan.scratch_elements)])
        expected, got = outs[0].cpu().numpy(), outs[1].cpu().numpy()
        magnitude = (a.abs() * b.abs()).sum(dim=1).cpu().numpy()
        assert np.all(np.abs(got - expected) <= tolerance * magnitude)
        site.close()


def _device_ms(call, repeats):
    torch = _torch()
    call()
    call()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        call()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / repeats


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [np.float32, np.complex64])
def test_u1_permute_workload_against_the_reference_companion(hosts, companion, dtype):
    """The U(1) four-leg permute + beta = 1 accumulate at degeneracy scale 40
    (151 M elements): the permute as an accumulation with unit coefficients,
    then the update, on both libraries; identical bits, and the device time per
    call of each (both on the default stream, after two warm-up calls)."""
    torch = _torch()
    from tensor0_b200.structure import U1Irrep, degeneracy_structure, hom, space
    from tensor0_b200.tensor_map import permute_plan
    v = space(U1Irrep, {q: int(round(40 * np.exp(-q * q / 8))) for q in range(-4, 5)})
    h = hom((v, v), (v, v))
    plan = permute_plan(h, (2, 0), (3, 1))
    n = degeneracy_structure(h).total_dim
    assert n == plan.output_size == 151162418
    x = cuda(sample(np.random.default_rng(7), dtype, (1, n)))
    z = cuda(sample(np.random.default_rng(8), dtype, (1, n)))
    real = np.float32
    one = cuda(np.array(1.0, real))
    item = np.dtype(dtype).itemsize
    rows = []

    permute = Site(hosts, companion, "accumulation", plan.words, dtype, coefficient_records=[])
    ours = stride.Plan(_native.OP_ACCUMULATION, permute.words, element_bytes=item, coefficient_records=[])
    ys = [torch.empty_like(x), torch.empty_like(x)]
    times = []
    for side in (0, 1):
        scratch = scratch_for(permute, side, 1, ours.scratch_elements)
        times.append(_device_ms(lambda: permute.call(side, lambda table: [x, table], [ys[side], scratch]), 3))
    assert np.array_equal(bits(ys[0]), bits(ys[1]))
    rows.append(("permute (accumulation)", 2 * n * item, times))
    permute.close()

    update = Site(hosts, companion, "update", plan.words, dtype)
    outs = [torch.empty_like(x), torch.empty_like(x)]
    times = []
    for side in (0, 1):
        times.append(_device_ms(lambda: update.call(side, lambda table: [ys[1], z, one, one, table], [outs[side]]), 3))
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    rows.append(("update (beta = 1)", 3 * n * item, times))
    update.close()

    for name, nbytes, (reference_ms, our_ms) in rows:
        print(f"\n{SUFFIX[dtype]} {name}: reference companion {reference_ms:.3f} ms "
              f"({nbytes / reference_ms / 1e6:.0f} GB/s), this library {our_ms:.3f} ms "
              f"({nbytes / our_ms / 1e6:.0f} GB/s), ratio {reference_ms / our_ms:.2f}")


@pytest.mark.gpu
def test_z2u1_trace_against_the_reference_companion(hosts, companion):
    """The partial trace of the Z2 x U(1) six-leg tensor (degeneracies 4 / 3,
    q in -3..3, 548,896,075 f64) over the leg pairs (1, 4) and (2, 5), through
    both libraries' reduction handlers: within 1e-12 of each other (the
    summation orders differ), and the time per call of each, taken with CUDA
    events around five back-to-back calls from this host (Python call frames
    included for both)."""
    torch = _torch()
    from tensor0_b200.structure import ProductSector, U1Irrep, Z2Irrep, degeneracy_structure, hom, space
    from tensor0_b200.tensor_map import trace_plan
    w = space(ProductSector(Z2Irrep, U1Irrep), {(p, q): (4, 3)[p] for p in (0, 1) for q in range(-3, 4)})
    h = hom((w, w, w), (w, w, w))
    n = degeneracy_structure(h).total_dim
    tp = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    assert n == 548896075 and set(np.asarray(tp.coefficients).tolist()) == {1.0}
    site = Site(hosts, companion, "reduction", tp.words, np.float64, coefficient_records=[])
    ours = stride.Plan(_native.OP_REDUCTION, site.words, element_bytes=8, coefficient_records=[])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    x = torch.randn((1, n), generator=gen, device="cuda", dtype=torch.float64)
    outs = [torch.full((1, ours.output_size), float("nan"), dtype=torch.float64, device="cuda") for _ in (0, 1)]
    times = []
    for side in (0, 1):
        scratch = scratch_for(site, side, 1, ours.scratch_elements)
        times.append(_device_ms(lambda: site.call(side, lambda table: [x, table], [outs[side], scratch]), 5))
    expected, got = outs[0].cpu().numpy(), outs[1].cpu().numpy()
    scale = max(float(np.max(np.abs(expected))), 1e-300)
    assert float(np.max(np.abs(got - expected))) / scale <= 1e-12
    site.close()
    print(f"\nf64 Z2xU1 trace: reference companion {times[0]:.3f} ms, this library {times[1]:.3f} ms per call "
          f"from this host, ratio {times[0] / times[1]:.1f}")
