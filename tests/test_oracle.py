"""The NumPy oracle pinned against the reference: golden vectors authored by the
reference's own tests, outputs of the compiled reference (oracle/_ref) stored
as fixtures, and — where oracle/_ref is present — randomized descriptors run
through both."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import ref, stride_oracle as so
from tensor0_b200 import stride
from random_layouts import random_reduction_layout
from tensor0_b200.structure import U1Irrep, degeneracy_structure, hom, space
from tensor0_b200.tensor_map import permute_plan

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden.json").read_text())
needs_ref = pytest.mark.skipif(not ref.available(), reason="compiled reference (oracle/_ref) not built")


def digest(array):
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


@pytest.mark.parametrize("case", GOLDEN["copy"], ids=lambda c: c["name"])
def test_copy_vectors(case):
    out = so.copy(np.array(case["words"]), np.array(case["source"], np.float64))
    assert out.tolist() == case["expected"]


def test_packed_trace_vector():
    case = GOLDEN["packed_trace"]
    out = so.reduction(np.array(case["words"]), np.array(case["source"]),
                       [np.float64(c) for c in case["coefficients"]], case["coefficient_records"])
    np.testing.assert_allclose(out, case["expected"], rtol=1e-14, atol=1e-14)


def config_one():
    v = space(U1Irrep, {-2: 4, -1: 8, 0: 12, 1: 8, 2: 4})
    h = hom((v, v), (v, v))
    plan = permute_plan(h, (1, 0), (3, 2))
    x = np.random.default_rng(1).standard_normal(degeneracy_structure(h).total_dim)
    y = np.random.default_rng(2).standard_normal(plan.output_size)
    return plan, x, y


def test_config_one_layout_and_outputs_match_reference_fixture():
    golden = GOLDEN["config_one"]
    plan, x, y = config_one()
    assert digest(plan.words) == golden["words_sha256"]
    n = len(plan.transform.src)
    permuted = so.accumulation(plan.words, x, [np.float64(1)] * n, np.arange(n))
    assert digest(permuted) == golden["permute_sha256"]
    updated = so.update(plan.words, x, y, np.float64(1.0), np.float64(0.5))
    assert digest(updated) == golden["add_transform_sha256"]


def random_layout(rng, source_size, output_size, records, max_rank=4):
    """Disjoint random records: permuted boxes carved from distinct output ranges."""
    out, cursor = [], 0
    for _ in range(records):
        rank = int(rng.integers(1, max_rank + 1))
        shape = tuple(int(n) for n in rng.integers(1, 6, size=rank))
        count = int(np.prod(shape))
        if cursor + count > output_size:
            break
        dst = stride.contiguous_strides(shape)
        perm = rng.permutation(rank)
        src_shape = tuple(shape[p] for p in perm)
        src_contig = stride.contiguous_strides(src_shape)
        sstr = [0] * rank
        for i, p in enumerate(perm):
            sstr[p] = src_contig[i]
        sign = rng.choice([-1, 1], size=rank)
        soff = int(rng.integers(0, source_size - count + 1))
        sstr = [int(s * g) for s, g in zip(sstr, sign)]
        soff += sum((n - 1) * (-s) for n, s in zip(shape, sstr) if s < 0)
        if soff + sum((n - 1) * s for n, s in zip(shape, sstr) if s > 0) >= source_size:
            continue
        out.append(stride.AffineRecord(shape, tuple(sstr), soff, dst, cursor))
        cursor += count + int(rng.integers(0, 3))
    return out


@needs_ref
@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.complex64, np.complex128])
def test_random_layouts_match_compiled_reference(seed, dtype):
    rng = np.random.default_rng(seed)
    records = random_layout(rng, 400, 600, 12)
    words = stride.encode_layout(records, source_size=400, output_size=600)
    x = rng.standard_normal(800).astype(dtype)[:400] if not np.iscomplexobj(np.zeros(1, dtype)) else \
        (rng.standard_normal(400) + 1j * rng.standard_normal(400)).astype(dtype)
    x = x.reshape(1, 400).repeat(2, axis=0)
    assert np.array_equal(so.copy(words, x).view(np.uint8), ref.copy(words, x, 600).view(np.uint8))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = [real(c) for c in rng.choice([0.0, 1.0, -0.5, 2.0], size=len(records))]
    a = so.accumulation(words, x, coefficients, np.arange(len(records)))
    b = ref.accumulation(words, x, 600, coefficients, np.arange(len(records)), outputs_disjoint=True)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    base = np.ascontiguousarray(np.roll(x, 1, axis=1)[:, :1].repeat(600, axis=1) * 0.25 + 1.0).astype(dtype)
    for alpha, beta in ((1.0, 0.0), (1.0, 0.5), (0.0, 1.0), (-2.0, 1.0), (0.0, 0.0)):
        u1 = so.update(words, x, base, real(alpha), real(beta))
        u2 = ref.update(words, x, base, real(alpha), real(beta))
        assert np.array_equal(u1.view(np.uint8), u2.view(np.uint8)), (alpha, beta)


@needs_ref
def test_reference_preparation_accepts_planner_words():
    plan, _, _ = config_one()
    prepared = ref.prepare_layout(3, plan.words)
    assert prepared[:4].tolist() == plan.words[:4].tolist()


def test_sector_gemm_oracle_is_blockwise_matmul():
    rng = np.random.default_rng(5)
    spec = np.array([[3, 4, 5, 0, 0, 0], [2, 2, 0, 0, 0, 12], [1, 3, 2, 15, 20, 16]])
    left, right = rng.standard_normal(20), rng.standard_normal(30)
    out = so.sector_gemm(spec, left, right, 19)
    np.testing.assert_allclose(out[:12].reshape(3, 4), left[:15].reshape(3, 5) @ right[:20].reshape(5, 4))
    assert np.all(out[12:16] == 0)
    np.testing.assert_allclose(out[16:19], (left[15:17].reshape(1, 2) @ right[20:26].reshape(2, 3)).reshape(-1))


@needs_ref
@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.complex64, np.complex128])
def test_random_reductions_match_compiled_reference(seed, dtype):
    rng = np.random.default_rng(200 + seed)
    records, shapes, roles, output_size = random_reduction_layout(rng, 300, 14)
    words = stride.encode_reduction_layout(records, output_shapes=shapes, reduction_axes=roles,
                                           source_size=300, output_size=output_size)
    complex_storage = np.iscomplexobj(np.zeros(1, dtype))
    x = rng.standard_normal((2, 300)) + (1j * rng.standard_normal((2, 300)) if complex_storage else 0)
    x = x.astype(dtype)
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = [real(c) for c in rng.choice([0.0, 1.0, -0.5, 2.0], size=len(records))]
    mine = so.reduction(words, x, coefficients, np.arange(len(records)))
    theirs = ref.reduction(words, x, output_size, coefficients, np.arange(len(records)))
    tolerance = 1e-6 if real == np.float32 else 1e-12
    scale = max(float(np.max(np.abs(theirs))), 1.0)
    assert float(np.max(np.abs(mine - theirs))) <= tolerance * scale


@needs_ref
@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.complex64, np.complex128])
def test_random_dots_match_compiled_reference(seed, dtype):
    """Dot records are only bounds-checked: sides may overlap or repeat."""
    rng = np.random.default_rng(300 + seed)
    records = []
    for _ in range(10):
        rank = int(rng.integers(1, 4))
        shape = tuple(int(n) for n in rng.integers(1, 5, size=rank))
        left = tuple(int(s) for s in rng.integers(-3, 4, size=rank))
        right = tuple(int(s) for s in rng.integers(-3, 4, size=rank))
        def origin(strides):
            low = sum((n - 1) * s for n, s in zip(shape, strides) if s < 0)
            high = sum((n - 1) * s for n, s in zip(shape, strides) if s > 0)
            return int(rng.integers(-low, 200 - high))
        records.append(stride.AffineRecord(shape, left, origin(left), right, origin(right)))
    words = stride.encode_layout(records, source_size=200, output_size=200)
    complex_storage = np.iscomplexobj(np.zeros(1, dtype))
    a = (rng.standard_normal((3, 200)) + (1j * rng.standard_normal((3, 200)) if complex_storage else 0)).astype(dtype)
    b = (rng.standard_normal((3, 200)) + (1j * rng.standard_normal((3, 200)) if complex_storage else 0)).astype(dtype)
    for conjugate in (False, True):
        mine = so.dot(words, a, b, conjugate)
        theirs = ref.dot(words, a, b, conjugate)
        tolerance = 1e-5 if dtype in (np.float32, np.complex64) else 1e-12
        assert np.max(np.abs(mine - theirs)) <= tolerance * max(1.0, float(np.max(np.abs(theirs))))
