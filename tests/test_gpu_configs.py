"""Parity of the sm_100a engine with the oracle at the benchmark workloads'
own sizes, and on the coefficient and offset paths the small cases leave out.

* U(1) 4-leg permute ((2, 0), (3, 1)) then beta = 1 accumulate at full size
  (N = 1,023,777,634), f32 and c64: bit-exact against the oracle, plus the
  size-independent round trip (the inverse permute restores every bit).
* The same workload at degeneracy scale 40 against the compiled reference's
  own executors, bit for bit (where oracle/_ref is built).
* Z2 x U(1) 6-leg partial trace at degeneracies 4 / 3, q in -3..3 (all
  298,592 sub-blocks), within 1e-12.
* The DMRG contraction L . A at chi = 2048 against dense tensordot, 1e-12.
* S32 coefficients, complex coefficients on accumulation and reduction,
  per-batch alpha / beta on update, and the 64-bit in-tile offset kernels.
"""

import numpy as np
import pytest
import torch

from oracle import dense, stride_oracle as so
from random_layouts import random_layout, random_reduction_layout
from tensor0_b200 import _native, stride
from tensor0_b200.structure import ProductSector, U1Irrep, Z2Irrep, degeneracy_structure, hom, space
from tensor0_b200.tensor_map import (TensorMap, add_transform, permute, permute_plan, tensorcontract,
                                     tensortrace, trace_plan)

pytestmark = pytest.mark.gpu

TOL = {np.float32: 1e-6, np.complex64: 1e-6, np.float64: 1e-12, np.complex128: 1e-12}
TORCH = {np.float32: torch.float32, np.float64: torch.float64, np.complex64: torch.complex64,
         np.complex128: torch.complex128}
DTYPES = [np.float32, np.float64, np.complex64, np.complex128]


def host(tensor):
    torch.cuda.synchronize()
    return tensor.cpu().numpy()


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def assert_close(actual, expected, dtype):
    scale = max(float(np.max(np.abs(expected))), 1e-300) if expected.size else 1.0
    error = float(np.max(np.abs(actual - expected))) / scale if expected.size else 0.0
    assert error <= TOL[dtype], f"relative error {error:.3e} > {TOL[dtype]:.0e}"


def sample(rng, dtype, shape):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    return rng.standard_normal(shape).astype(dtype)


def four_leg_space(scale):
    degs = {q: int(round(scale * np.exp(-q * q / 8))) for q in range(-4, 5)}
    v = space(U1Irrep, degs)
    return hom((v, v), (v, v))


def device_normal(n, dtype, seed):
    generator = torch.Generator(device="cuda")
    generator.manual_seed(seed)
    return torch.randn(n, generator=generator, device="cuda", dtype=TORCH[dtype])


@pytest.mark.parametrize("dtype", [np.float32, np.complex64])
def test_config_two_full_size_permute_and_accumulate(dtype):
    h = four_leg_space(64)
    plan = permute_plan(h, (2, 0), (3, 1))
    n = plan.source_size
    assert n == 1023777634 and len(plan.transform.src) == 489
    x = TensorMap(h, device_normal(n, dtype, 11))
    y = permute(x, ((2, 0), (3, 1)))
    base = device_normal(n, dtype, 12)
    z = add_transform(TensorMap(y.space, base.clone()), x, ((2, 0), (3, 1)), alpha=1.0, beta=1.0)
    # Size-independent: the inverse permute restores every bit of x.
    back = permute(y, ((1, 3), (0, 2)))
    torch.cuda.synchronize()
    assert back.space == h and torch.equal(back.data.view(torch.uint8), x.data.view(torch.uint8))
    del back
    x_host, y_host, base_host, z_host = host(x.data), host(y.data), host(base), host(z.data)
    del x, y, z, base
    torch.cuda.empty_cache()
    records = np.arange(len(plan.transform.src))
    real = np.float32
    expected = so.accumulation(plan.words, x_host, [real(1)] * len(records), records)
    assert np.array_equal(bits(y_host), bits(expected))
    del expected
    expected = so.update(plan.words, x_host, base_host, real(1), real(1))
    assert np.array_equal(bits(z_host), bits(expected))


def test_config_two_scale_forty_matches_compiled_reference_bits():
    from oracle import ref
    if not ref.available():
        pytest.skip("compiled reference (oracle/_ref) not built")
    h = four_leg_space(40)
    plan = permute_plan(h, (2, 0), (3, 1))
    n = plan.source_size
    x = TensorMap(h, device_normal(n, np.float32, 21))
    base = device_normal(n, np.float32, 22)
    y = permute(x, ((2, 0), (3, 1)))
    z = add_transform(TensorMap(y.space, base.clone()), x, ((2, 0), (3, 1)), alpha=1.0, beta=1.0)
    x_host, base_host = host(x.data), host(base)
    records = np.arange(len(plan.transform.src))
    threads = 8
    expected = ref.accumulation(plan.words, x_host, n, [np.float32(1)] * len(records), records,
                                outputs_disjoint=True, threads=threads)
    assert np.array_equal(bits(host(y.data)), bits(expected))
    expected = ref.update(plan.words, x_host, base_host, np.float32(1), np.float32(1), threads=threads)
    assert np.array_equal(bits(host(z.data)), bits(expected))


def test_config_three_scaled_partial_trace():
    w = space(ProductSector(Z2Irrep, U1Irrep), {(p, q): (4 if p == 0 else 3) for p in (0, 1) for q in range(-3, 4)})
    h = hom((w, w, w), (w, w, w))
    ds = degeneracy_structure(h)
    assert len(ds.offsets) == 298592
    x = device_normal(ds.total_dim, np.float64, 3)
    got = tensortrace(TensorMap(h, x), axes=((1, 2), (4, 5)), output=((0,), (3,)))
    tp = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    expected = so.reduction(tp.words, host(x), list(tp.coefficients), np.arange(tp.records))
    assert got.data.numel() == 175
    assert_close(host(got.data), expected, np.float64)


def test_config_four_dmrg_contraction_full_bond_dimension():
    degeneracies = [8, 18, 37, 68, 112, 166, 219, 259, 274, 259, 219, 166, 112, 68, 37, 18, 8]
    chi = space(U1Irrep, {q: d for q, d in zip(range(-8, 9), degeneracies)})
    assert chi.dim == 2048
    phys = space(U1Irrep, {0: 1, 1: 1})
    w = space(U1Irrep, {0: 5})
    a_space, l_space = hom((chi, phys), (chi,)), hom((chi,), (chi, w))
    a = device_normal(degeneracy_structure(a_space).total_dim, np.float64, 4)
    l = device_normal(degeneracy_structure(l_space).total_dim, np.float64, 5)
    output = (((0, 0), (1, 1)), ((0, 2), (1, 2)))
    out = tensorcontract(TensorMap(l_space, l), TensorMap(a_space, a), axes=((1,), (0,)), output=output)
    expected = dense.contract(dense.to_dense(l_space, host(l)), dense.to_dense(a_space, host(a)), (1,), (0,),
                              output)
    assert_close(dense.to_dense(out.space, host(out.data)), expected, np.float64)


@pytest.mark.parametrize("dtype", DTYPES)
def test_s32_coefficients(dtype):
    rng = np.random.default_rng(61)
    records = random_layout(rng, 1500, 2000, 30, max_extent=12)
    words = stride.encode_layout(records, source_size=1500, output_size=2000)
    x, base = sample(rng, dtype, (2, 1500)), sample(rng, dtype, (2, 2000))
    eb = np.dtype(dtype).itemsize
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = rng.choice([0, 1, -1, 3], size=len(records)).astype(np.int32)
    plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=eb,
                       coefficient_records=np.arange(len(records)), outputs_disjoint=True)
    got = host(stride.execute_accumulation(torch.from_numpy(x).cuda(), plan, torch.from_numpy(coefficients)))
    expected = so.accumulation(words, x, [real(c) for c in coefficients], np.arange(len(records)))
    assert np.array_equal(bits(got), bits(expected))
    update = stride.Plan(_native.OP_UPDATE, words, element_bytes=eb)
    for alpha, beta in ((1, 0), (2, -1), (0, 3)):
        got = host(stride.execute_update(torch.from_numpy(x).cuda(), torch.from_numpy(base).cuda(),
                                         torch.tensor([alpha], dtype=torch.int32),
                                         torch.tensor([beta], dtype=torch.int32), update))
        expected = so.update(words, x, base, real(alpha), real(beta))
        assert np.array_equal(bits(got), bits(expected)), (alpha, beta)


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
def test_complex_coefficients_on_accumulation_and_reduction(dtype):
    rng = np.random.default_rng(71)
    records = random_layout(rng, 1200, 1600, 25, max_extent=10)
    words = stride.encode_layout(records, source_size=1200, output_size=1600)
    x = sample(rng, dtype, (3, 1200))
    coefficients = sample(rng, dtype, len(records))
    coefficients[::5] = 0
    coefficients[1::5] = 1
    plan = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=np.arange(len(records)), outputs_disjoint=True)
    got = host(stride.execute_accumulation(torch.from_numpy(x).cuda(), plan, torch.from_numpy(coefficients)))
    assert_close(got, so.accumulation(words, x, list(coefficients), np.arange(len(records))), dtype)
    reduction, shapes, roles, output_size = random_reduction_layout(rng, 1200, 20)
    words = stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                           source_size=1200, output_size=output_size)
    coefficients = sample(rng, dtype, len(reduction))
    plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=np.arange(len(reduction)))
    got = host(stride.execute_reduction(torch.from_numpy(x).cuda(), plan, torch.from_numpy(coefficients)))
    assert_close(got, so.reduction(words, x, list(coefficients), np.arange(len(reduction))), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_random_reductions(dtype):
    rng = np.random.default_rng(81)
    for _ in range(3):
        reduction, shapes, roles, output_size = random_reduction_layout(rng, 800, 24)
        words = stride.encode_reduction_layout(reduction, output_shapes=shapes, reduction_axes=roles,
                                               source_size=800, output_size=output_size)
        x = sample(rng, dtype, (2, 800))
        real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
        coefficients = rng.choice([0.0, 1.0, -0.5, 2.0], size=len(reduction)).astype(real)
        plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=np.dtype(dtype).itemsize,
                           coefficient_records=np.arange(len(reduction)))
        got = host(stride.execute_reduction(torch.from_numpy(x).cuda(), plan, torch.from_numpy(coefficients)))
        assert_close(got, so.reduction(words, x, list(coefficients), np.arange(len(reduction))), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_per_batch_update_coefficients(dtype):
    rng = np.random.default_rng(91)
    records = random_layout(rng, 900, 1200, 20, max_extent=9)
    words = stride.encode_layout(records, source_size=900, output_size=1200)
    batches = 4
    x, base = sample(rng, dtype, (batches, 900)), sample(rng, dtype, (batches, 1200))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    alpha = np.array([1.0, 0.0, -2.0, 1.0], real)
    beta = np.array([0.0, 1.0, 0.5, 1.0], real)
    plan = stride.Plan(_native.OP_UPDATE, words, element_bytes=np.dtype(dtype).itemsize)
    got = host(stride.execute_update(torch.from_numpy(x).cuda(), torch.from_numpy(base).cuda(),
                                     torch.from_numpy(alpha), torch.from_numpy(beta), plan))
    for b in range(batches):
        expected = so.update(words, x[b:b + 1], base[b:b + 1], alpha[b], beta[b])
        assert np.array_equal(bits(got[b:b + 1]), bits(expected)), b


@pytest.mark.parametrize("dtype", DTYPES)
def test_wide_offset_kernels_bit_exact(dtype):
    """The 64-bit in-tile offset instantiation gives the same bits."""
    rng = np.random.default_rng(101)
    records = random_layout(rng, 4000, 5000, 50, max_extent=30)
    words = stride.encode_layout(records, source_size=4000, output_size=5000)
    x, base = sample(rng, dtype, (2, 4000)), sample(rng, dtype, (2, 5000))
    eb = np.dtype(dtype).itemsize
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    copy = stride.Plan(_native.OP_COPY, words, element_bytes=eb, wide_offsets=True)
    got = host(stride.execute_copy(torch.from_numpy(x).cuda(), copy))
    assert np.array_equal(bits(got), bits(so.copy(words, x)))
    coefficients = rng.choice([0.0, 1.0, -0.5], size=len(records)).astype(real)
    acc = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=eb, coefficient_records=np.arange(len(records)),
                      outputs_disjoint=True, wide_offsets=True)
    got = host(stride.execute_accumulation(torch.from_numpy(x).cuda(), acc, torch.from_numpy(coefficients)))
    assert np.array_equal(bits(got), bits(so.accumulation(words, x, list(coefficients), np.arange(len(records)))))
    update = stride.Plan(_native.OP_UPDATE, words, element_bytes=eb, wide_offsets=True)
    got = host(stride.execute_update(torch.from_numpy(x).cuda(), torch.from_numpy(base).cuda(), 1.0, 0.5, update))
    assert np.array_equal(bits(got), bits(so.update(words, x, base, real(1.0), real(0.5))))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sector_shards_gathered_equal_the_single_launch(world):
    """The multi-GPU split run on one GPU: each LPT shard's compacted source is
    scattered out of the packed tensor, permuted and accumulated by its own
    plans, the padded outputs are concatenated as an all-gather would and one
    engine copy unpacks them; the result equals the single launch bit for bit."""
    from tensor0_b200.sharding import gather_words, scatter_words, shard_capacity, shard_permute
    h = four_leg_space(24)
    plan = permute_plan(h, (2, 0), (3, 1))
    x = device_normal(plan.source_size, np.float32, 31)
    base = device_normal(plan.output_size, np.float32, 32)
    y = permute(TensorMap(h, x), ((2, 0), (3, 1)))
    z = add_transform(TensorMap(y.space, base.clone()), TensorMap(h, x), ((2, 0), (3, 1)), 1.0, 1.0)
    capacity = shard_capacity(plan, world, 4)
    gathered_y = torch.zeros(world * capacity, device="cuda")
    gathered_z = torch.zeros(world * capacity, device="cuda")
    one = torch.ones(1, device="cuda")
    for r in range(world):
        shard = shard_permute(plan, r, world, 4)
        scatter_x = stride.Plan(_native.OP_COPY, scatter_words(plan, r, world, 4), element_bytes=4)
        scatter_b = stride.Plan(_native.OP_COPY, scatter_words(plan, r, world, 4, source=False), element_bytes=4)
        xl = stride.execute_copy(x, scatter_x)
        bl = stride.execute_copy(base, scatter_b)
        acc = stride.Plan(_native.OP_ACCUMULATION, shard.words, element_bytes=4,
                          coefficient_records=np.arange(shard.records.size), outputs_disjoint=True)
        upd = stride.Plan(_native.OP_UPDATE, shard.words, element_bytes=4)
        stride.execute_accumulation(xl, acc, torch.ones(shard.records.size, device="cuda"),
                                    out=gathered_y[r * capacity: r * capacity + shard.local_output_size])
        stride.execute_update(xl, bl, one, one, upd, out=gathered_z[r * capacity: r * capacity + shard.local_output_size])
    unpack = stride.Plan(_native.OP_COPY, gather_words(plan, world, 4), element_bytes=4)
    torch.cuda.synchronize()
    assert torch.equal(stride.execute_copy(gathered_y, unpack).view(torch.int32), y.data.view(torch.int32))
    assert torch.equal(stride.execute_copy(gathered_z, unpack).view(torch.int32), z.data.view(torch.int32))


@pytest.mark.parametrize("dtype", DTYPES)
def test_long_fiber_reductions(dtype):
    """Records summing 100-300 elements each (lanes stride one record's fiber)
    beside short-fiber records (lanes take whole records)."""
    rng = np.random.default_rng(171)
    records = [stride.AffineRecord((8, 100), (100, 1), 0, (1, 0), 0),
               stride.AffineRecord((8, 300), (1, 8), 800, (1, 0), 0),
               stride.AffineRecord((8, 3), (3, 1), 3200, (1, 0), 8),
               stride.AffineRecord((8, 150), (150, 1), 0, (1, 0), 8)]
    words = stride.encode_reduction_layout(records, output_shapes=[(8, 1)] * 4, reduction_axes=[(False, True)] * 4,
                                           source_size=3300, output_size=16)
    x = sample(rng, dtype, (2, 3300))
    real = np.float32 if dtype in (np.float32, np.complex64) else np.float64
    coefficients = np.array([1.0, -0.5, 2.0, 1.0], real)
    plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=np.dtype(dtype).itemsize,
                       coefficient_records=np.arange(4))
    got = host(stride.execute_reduction(torch.from_numpy(x).cuda(), plan, torch.from_numpy(coefficients)))
    expected = so.reduction(words, x, list(coefficients), np.arange(4))
    magnitude = so.reduction(words, np.abs(x), [abs(c) for c in coefficients], np.arange(4))
    assert np.all(np.abs(got - expected) <= 4 * TOL[dtype] * np.maximum(np.abs(magnitude), 1e-300))
