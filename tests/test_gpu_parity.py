"""Parity of the sm_100a engine (called through the C ABI) with the oracle.

Bit-exact: copies, permutes (accumulation with unit coefficients) and real
or real-coefficient updates — the reference computes these with single IEEE
operations in a fixed order.  Within tolerance (rel. 1e-6 for f32 / c64,
1e-12 for f64 / c128, as the hot-path contract states): sums over reduction
axes, complex-coefficient scalings and GEMMs, whose summation order differs."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import stride_oracle as so
from random_layouts import random_layout
from tensor0_b200 import _native, stride
from tensor0_b200.structure import (ProductSector, U1Irrep, Z2Irrep, Z3Irrep, degeneracy_structure, hom,
                                    space)
from tensor0_b200.tensor_map import (TensorMap, add_transform, permute, permute_plan, tensorcontract,
                                     tensortrace, trace_plan)

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden.json").read_text())
TOL = {np.float32: 1e-6, np.complex64: 1e-6, np.float64: 1e-12, np.complex128: 1e-12}
TORCH = {np.float32: torch.float32, np.float64: torch.float64, np.complex64: torch.complex64,
         np.complex128: torch.complex128}


def cuda(array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def host(tensor):
    torch.cuda.synchronize()
    return tensor.cpu().numpy()


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def assert_close(actual, expected, dtype):
    scale = max(float(np.max(np.abs(expected))), 1e-300)
    error = float(np.max(np.abs(actual - expected))) / scale if expected.size else 0.0
    assert error <= TOL[dtype], f"relative error {error:.3e} > {TOL[dtype]:.0e}"


def digest(array):
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


@pytest.mark.parametrize("case", GOLDEN["copy"], ids=lambda c: c["name"])
def test_reference_copy_vectors(case):
    plan = stride.Plan(_native.OP_COPY, np.array(case["words"]), element_bytes=8)
    out = stride.execute_copy(cuda(np.array(case["source"], np.float64)), plan)
    assert host(out).tolist() == case["expected"]


def test_reference_packed_trace_vector():
    case = GOLDEN["packed_trace"]
    plan = stride.Plan(_native.OP_REDUCTION, np.array(case["words"]), element_bytes=8,
                       coefficient_records=case["coefficient_records"])
    out = stride.execute_reduction(cuda(np.array(case["source"])), plan,
                                   torch.tensor(case["coefficients"], dtype=torch.float64))
    np.testing.assert_allclose(host(out), case["expected"], rtol=1e-14, atol=1e-14)


def test_config_one_permute_and_add_transform_match_reference_bits():
    golden = GOLDEN["config_one"]
    v = space(U1Irrep, {-2: 4, -1: 8, 0: 12, 1: 8, 2: 4})
    h = hom((v, v), (v, v))
    n = degeneracy_structure(h).total_dim
    x = TensorMap(h, cuda(np.random.default_rng(1).standard_normal(n)))
    y = permute(x, ((1, 0), (3, 2)))
    assert digest(host(y.data)) == golden["permute_sha256"]
    base = TensorMap(y.space, cuda(np.random.default_rng(2).standard_normal(n)))
    z = add_transform(base, x, ((1, 0), (3, 2)), alpha=1.0, beta=0.5)
    assert digest(host(z.data)) == golden["add_transform_sha256"]
    # In place into the destination tensor (the reference's result aliases base).
    w = add_transform(base, x, ((1, 0), (3, 2)), alpha=1.0, beta=0.5, inplace=True)
    assert w.data.data_ptr() == base.data.data_ptr()
    assert digest(host(w.data)) == golden["add_transform_sha256"]


def sample(rng, dtype, shape):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    return rng.standard_normal(shape).astype(dtype)


DTYPES = [np.float32, np.float64, np.complex64, np.complex128]


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("dtype", DTYPES)
def test_random_layouts_bit_exact(seed, dtype):
    rng = np.random.default_rng(100 + seed)
    size_in, size_out = 3000, 4000
    records = random_layout(rng, size_in, size_out, 60, max_extent=40 if seed % 2 else 6)
    words = stride.encode_layout(records, source_size=size_in, output_size=size_out)
    x = sample(rng, dtype, (3, size_in))
    eb = np.dtype(dtype).itemsize
    copy_plan = stride.Plan(_native.OP_COPY, words, element_bytes=eb)
    assert np.array_equal(bits(host(stride.execute_copy(cuda(x), copy_plan))), bits(so.copy(words, x)))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = rng.choice([0.0, 1.0, -0.5, 2.0], size=len(records)).astype(real)
    acc_plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=eb,
                           coefficient_records=np.arange(len(records)), outputs_disjoint=True)
    got = host(stride.execute_accumulation(cuda(x), acc_plan, torch.from_numpy(coefficients)))
    assert np.array_equal(bits(got), bits(so.accumulation(words, x, list(coefficients), np.arange(len(records)))))
    # Without the producer's assertion the planner proves disjointness itself.
    proven = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=eb,
                         coefficient_records=np.arange(len(records)))
    got = host(stride.execute_accumulation(cuda(x), proven, torch.from_numpy(coefficients)))
    assert np.array_equal(bits(got), bits(so.accumulation(words, x, list(coefficients), np.arange(len(records)))))
    base = sample(rng, dtype, (3, size_out))
    update_plan = stride.Plan(_native.OP_UPDATE, words, element_bytes=eb)
    for alpha, beta in ((1.0, 0.0), (1.0, 0.5), (0.0, 1.0), (-2.0, 1.0), (0.0, 0.0), (1.0, 1.0)):
        got = host(stride.execute_update(cuda(x), cuda(base), alpha, beta, update_plan))
        expected = so.update(words, x, base, real(alpha), real(beta))
        assert np.array_equal(bits(got), bits(expected)), (alpha, beta)


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
def test_complex_coefficient_update_within_tolerance(dtype):
    rng = np.random.default_rng(7)
    records = random_layout(rng, 2000, 2500, 40)
    words = stride.encode_layout(records, source_size=2000, output_size=2500)
    x, base = sample(rng, dtype, (2, 2000)), sample(rng, dtype, (2, 2500))
    plan = stride.Plan(_native.OP_UPDATE, words, element_bytes=np.dtype(dtype).itemsize)
    alpha = torch.tensor([0.7 + 0.2j], dtype=TORCH[dtype])
    got = host(stride.execute_update(cuda(x), cuda(base), alpha, 1.0, plan))
    assert_close(got, so.update(words, x, base, np.array(0.7 + 0.2j, dtype), np.float64(1.0)), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_per_batch_coefficients(dtype):
    rng = np.random.default_rng(9)
    records = random_layout(rng, 500, 700, 10)
    words = stride.encode_layout(records, source_size=500, output_size=700)
    x = sample(rng, dtype, (4, 500))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = rng.choice([0.0, 1.0, 3.0], size=(len(records), 4)).astype(real)
    plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=np.arange(len(records)), outputs_disjoint=True)
    got = host(stride.execute_accumulation(cuda(x), plan, torch.from_numpy(coefficients)))
    for b in range(4):
        expected = so.accumulation(words, x[b:b + 1], list(coefficients[:, b]), np.arange(len(records)))
        assert np.array_equal(bits(got[b:b + 1]), bits(expected))


@pytest.mark.parametrize("dtype", DTYPES)
def test_overlapping_accumulation_and_fibers(dtype):
    """Records sharing outputs and zero-stride (summed) axes run in the reduce engine."""
    rng = np.random.default_rng(11)
    records = [
        stride.AffineRecord((4, 3), (3, 1), 0, (1, 0), 0),       # sums over the second axis
        stride.AffineRecord((4,), (1,), 12, (1,), 0),           # overlaps the first record's outputs
        stride.AffineRecord((2, 5), (5, 1), 20, (1, 0), 10),
        stride.AffineRecord((3,), (2,), 1, (1,), 2),            # partial overlap
        stride.AffineRecord((0, 3), (1, 1), 0, (1, 1), 0),      # empty
    ]
    words = stride.encode_layout(records, source_size=40, output_size=16)
    x = sample(rng, dtype, (2, 40))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = np.array([1.0, -2.0, 0.5, 0.0], real)
    plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=[0, 1, 2, 3])
    got = host(stride.execute_accumulation(cuda(x), plan, torch.from_numpy(coefficients)))
    assert_close(got, so.accumulation(words, x, list(coefficients), [0, 1, 2, 3]), dtype)


def z2u1_space(deg0, deg1, charges=range(-1, 2)):
    return space(ProductSector(Z2Irrep, U1Irrep), {(p, q): (deg0 if p == 0 else deg1) for p in (0, 1) for q in charges})


@pytest.mark.parametrize("dtype", DTYPES)
def test_partial_trace(dtype):
    w = z2u1_space(2, 1)
    h = hom((w, w, w), (w, w, w))
    plan = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    x = sample(np.random.default_rng(3), dtype, degeneracy_structure(h).total_dim)
    got = tensortrace(TensorMap(h, cuda(x)), axes=((1, 2), (4, 5)), output=((0,), (3,)))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    expected = so.reduction(plan.words, x, [real(c) for c in plan.coefficients], np.arange(plan.records))
    assert_close(host(got.data), expected, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_permute_and_accumulate_u1_four_leg(dtype):
    """The permute ((2, 0), (3, 1)) then beta = 1 accumulate, at reduced degeneracies."""
    degs = {q: max(1, round(16 * np.exp(-q * q / 8))) for q in range(-4, 5)}
    v = space(U1Irrep, degs)
    h = hom((v, v), (v, v))
    n = degeneracy_structure(h).total_dim
    x = sample(np.random.default_rng(21), dtype, n)
    t = TensorMap(h, cuda(x))
    y = permute(t, ((2, 0), (3, 1)))
    plan = permute_plan(h, (2, 0), (3, 1))
    records = np.arange(len(plan.transform.src))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    expected = so.accumulation(plan.words, x, [real(1)] * len(records), records)
    assert np.array_equal(bits(host(y.data)), bits(expected))
    base = sample(np.random.default_rng(22), dtype, plan.output_size)
    z = add_transform(TensorMap(y.space, cuda(base)), t, ((2, 0), (3, 1)), alpha=1.0, beta=1.0)
    assert np.array_equal(bits(host(z.data)), bits(so.update(plan.words, x, base, real(1), real(1))))
    # Round trip: the inverse permute restores every bit.
    back = permute(y, ((1, 3), (0, 2)))
    assert back.space == h and np.array_equal(bits(host(back.data)), bits(x))


@pytest.mark.parametrize("dtype", DTYPES)
def test_sector_gemm(dtype):
    rng = np.random.default_rng(31)
    shapes = [(70, 33, 129), (1, 1, 1), (64, 64, 64), (5, 100, 0), (130, 2, 17), (0, 4, 3)]
    spec, a_off, b_off, c_off = [], 0, 0, 0
    for m, n, k in shapes:
        spec.append((m, n, k, a_off, b_off, c_off))
        a_off, b_off, c_off = a_off + m * k, b_off + k * n, c_off + m * n
    left, right = sample(rng, dtype, a_off), sample(rng, dtype, b_off)
    plan = stride.GemmPlan(np.array(spec))
    out = torch.full((c_off,), 7, dtype=TORCH[dtype], device="cuda")
    got = host(stride.sector_gemm(plan, cuda(left), cuda(right), out))
    assert_close(got, so.sector_gemm(np.array(spec), left, right, c_off), dtype)


@pytest.mark.parametrize("dtype", [np.float32, np.complex64])
def test_sector_gemm_single_precision_long_k_on_tensor_cores(dtype):
    """F32 and C64 sectors run on tcgen05 (three-term TF32 split, K slices
    summed in FP32 registers; C64 as four real products with A negated for
    -Ai Bi): the error stays within the single-precision tolerance for K in
    the thousands, several 128 x 64 tiles per sector and ragged edges."""
    rng = np.random.default_rng(33)
    shapes = [(300, 200, 2048), (129, 65, 1000), (7, 3, 4097)]
    spec, a_off, b_off, c_off = [], 0, 0, 0
    for m, n, k in shapes:
        spec.append((m, n, k, a_off, b_off, c_off))
        a_off, b_off, c_off = a_off + m * k, b_off + k * n, c_off + m * n
    left, right = sample(rng, dtype, a_off), sample(rng, dtype, b_off)
    wide = np.complex128 if dtype == np.complex64 else np.float64
    plan = stride.GemmPlan(np.array(spec))
    for _ in range(2):
        out = torch.full((c_off,), float("nan"), dtype=TORCH[dtype], device="cuda")
        got = host(stride.sector_gemm(plan, cuda(left), cuda(right), out))
        expected = so.sector_gemm(np.array(spec), left.astype(wide), right.astype(wide), c_off)
        assert_close(got, expected, dtype)


@pytest.mark.parametrize("dtype", [np.float64, np.complex128])
def test_dmrg_contraction(dtype):
    """L . A with U1 sectors (the DMRG-style contraction, reduced bond dimension)."""
    chi = space(U1Irrep, {q: 6 + 2 * (2 - abs(q)) for q in range(-2, 3)})
    phys = space(U1Irrep, {0: 1, 1: 1})
    w = space(U1Irrep, {0: 3})
    a_space, l_space = hom((chi, phys), (chi,)), hom((chi,), (chi, w))
    rng = np.random.default_rng(41)
    a = sample(rng, dtype, degeneracy_structure(a_space).total_dim)
    l = sample(rng, dtype, degeneracy_structure(l_space).total_dim)
    out = tensorcontract(TensorMap(l_space, cuda(l)), TensorMap(a_space, cuda(a)), axes=((1,), (0,)),
                         output=(((0, 0), (1, 1)), ((0, 2), (1, 2))))
    from oracle import dense
    expected = dense.contract(dense.to_dense(l_space, l), dense.to_dense(a_space, a), (1,), (0,),
                              (((0, 0), (1, 1)), ((0, 2), (1, 2))))
    assert_close(dense.to_dense(out.space, host(out.data)), expected, dtype)


def test_tensormap_add():
    v = space(U1Irrep, {-1: 3, 0: 4, 1: 3})
    h = hom((v,), (v, v))
    n = degeneracy_structure(h).total_dim
    rng = np.random.default_rng(51)
    x, y = rng.standard_normal(n), rng.standard_normal(n)
    got = TensorMap(h, cuda(x)).add(TensorMap(h, cuda(y)), 1.0, 0.5)
    assert np.array_equal(host(got.data), x + 0.5 * y)
    xc = x + 1j * y
    got = TensorMap(h, cuda(xc)).add(TensorMap(h, cuda(xc)), 0.7 + 0.2j, 1.0)
    assert_close(host(got.data), (0.7 + 0.2j) * xc + xc, np.complex128)


def test_engine_launches_are_counted():
    before = stride.kernel_launches()
    test_config_one_permute_and_add_transform_match_reference_bits()
    assert stride.kernel_launches() >= before + 3


@pytest.mark.parametrize("dtype", DTYPES)
def test_rectangular_tiles_with_edges(dtype):
    """Transposes with unit strides on both sides and X / Y extents from 32 to
    130: the fixed-map rectangular tiles, including edge tiles along X (64 + 1,
    64 + 66), ragged Y and several Z slices per tile."""
    rng = np.random.default_rng(131)
    shapes = [(32, 32), (64, 64), (65, 40), (130, 33), (40, 3, 97), (33, 7, 50), (70, 2, 70)]
    records, src_off, dst_off = [], 0, 0
    for shape in shapes:
        # Source row-major, destination with the axis order reversed: the
        # source's innermost axis is the destination's outermost.
        dst = stride.contiguous_strides(tuple(reversed(shape)))[::-1]
        src = stride.contiguous_strides(shape)
        records.append(stride.AffineRecord(shape, tuple(src), src_off, tuple(dst), dst_off))
        count = int(np.prod(shape))
        src_off += count + 3
        dst_off += count + 1
    words = stride.encode_layout(records, source_size=src_off, output_size=dst_off)
    x, base = sample(rng, dtype, (2, src_off)), sample(rng, dtype, (2, dst_off))
    eb = np.dtype(dtype).itemsize
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    copy = stride.Plan(_native.OP_COPY, words, element_bytes=eb)
    assert np.array_equal(bits(host(stride.execute_copy(cuda(x), copy))), bits(so.copy(words, x)))
    coefficients = np.array([1.0, -0.5, 1.0, 2.0, 0.0, 1.0, 3.0], real)
    acc = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=eb, coefficient_records=np.arange(len(records)),
                      outputs_disjoint=True)
    got = host(stride.execute_accumulation(cuda(x), acc, torch.from_numpy(coefficients)))
    assert np.array_equal(bits(got), bits(so.accumulation(words, x, list(coefficients), np.arange(len(records)))))
    update = stride.Plan(_native.OP_UPDATE, words, element_bytes=eb)
    for alpha, beta in ((1.0, 1.0), (1.0, 0.0), (-2.0, 0.5), (0.0, 1.0)):
        got = host(stride.execute_update(cuda(x), cuda(base), alpha, beta, update))
        assert np.array_equal(bits(got), bits(so.update(words, x, base, real(alpha), real(beta)))), (alpha, beta)


def dot_layout(rng, size, records=12):
    out = []
    for _ in range(records):
        rank = int(rng.integers(1, 4))
        shape = tuple(int(n) for n in rng.integers(1, 40, size=rank))
        left = tuple(int(s) for s in rng.integers(-3, 4, size=rank))
        right = tuple(int(s) for s in rng.integers(-3, 4, size=rank))

        def origin(strides):
            low = sum((n - 1) * s for n, s in zip(shape, strides) if s < 0)
            high = sum((n - 1) * s for n, s in zip(shape, strides) if s > 0)
            return int(rng.integers(-low, size - high)) if size - high > -low else None

        lo, ro = origin(left), origin(right)
        if lo is not None and ro is not None:
            out.append(stride.AffineRecord(shape, left, lo, right, ro))
    return out


@pytest.mark.parametrize("dtype", DTYPES)
def test_dot_matches_oracle(dtype):
    """Dot over overlapping, broadcast and negative-stride records; the error
    is measured against the sum of |terms| (single precision sums accumulate
    in double precision)."""
    rng = np.random.default_rng(141)
    size = 5000
    records = dot_layout(rng, size)
    words = stride.encode_layout(records, source_size=size, output_size=size)
    a, b = sample(rng, dtype, (3, size)), sample(rng, dtype, (3, size))
    plan = stride.Plan(_native.OP_DOT, words, element_bytes=np.dtype(dtype).itemsize)
    for conjugate in (False, True):
        got = host(stride.execute_dot(cuda(a), cuda(b), plan, conjugate_left=conjugate))
        expected = so.dot(words, a, b, conjugate)
        magnitude = so.dot(words, np.abs(a), np.abs(b))
        assert np.all(np.abs(got - expected) <= TOL[dtype] * np.maximum(magnitude, 1e-300))


@pytest.mark.parametrize("dtype", DTYPES)
def test_tensormap_inner_and_norm(dtype):
    v = space(U1Irrep, {-1: 30, 0: 40, 1: 30})
    h = hom((v, v), (v,))
    n = degeneracy_structure(h).total_dim
    rng = np.random.default_rng(151)
    x, y = sample(rng, dtype, n), sample(rng, dtype, n)
    tx, ty = TensorMap(h, cuda(x)), TensorMap(h, cuda(y))
    got = host(tx.inner(ty))
    expected = np.vdot(x.astype(np.complex128), y.astype(np.complex128))
    assert abs(got - expected) <= TOL[dtype] * np.sum(np.abs(x) * np.abs(y))
    norm = float(host(tx.norm()))
    assert abs(norm - np.linalg.norm(x.astype(np.complex128))) <= TOL[dtype] * np.linalg.norm(x)
