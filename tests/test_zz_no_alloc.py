"""The allocation-free reduction entry point (t0b_reduction_static_scratch).

Some callers cannot allocate device memory: an XLA FFI handler, where XLA
owns every buffer, or an application whose device memory belongs to its own
pool.  The entry point keeps the reduce engine's partials in an array compiled
into the library.  It must give the same result as t0b_reduction with
caller-provided scratch, on consecutive calls that share that array.

This file is collected last, so a failure here comes after every other test
has run.  It passes on its own in a fresh process as well.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import stride_oracle as so
from tensor0_b200 import _native, stride
from tensor0_b200.structure import ProductSector, U1Irrep, Z2Irrep, degeneracy_structure, hom, space
from tensor0_b200.tensor_map import trace_plan

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-12   # f64, the tolerance of the other reduction parity tests


def call_static(plan, source, output, coefficients, coefficient_count=1):
    err = _native.error_buffer()
    status = _native.lib().t0b_reduction_static_scratch(
        plan._handle, _native.F64, source.data_ptr(), output.data_ptr(), source.shape[0] if source.ndim > 1 else 1,
        coefficients.data_ptr(), _native.F64, coefficient_count, plan.device_table(source.device).data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err, len(err))
    return status, err.value.decode()


def relative_error(actual, expected):
    return float(np.max(np.abs(actual - expected))) / max(float(np.max(np.abs(expected))), 1e-300)


def test_static_scratch_matches_caller_scratch_on_consecutive_calls():
    w = space(ProductSector(Z2Irrep, U1Irrep), {(p, q): 2 - p for p in (0, 1) for q in (-1, 0, 1)})
    h = hom((w, w, w), (w, w, w))
    tp = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    plan = tp.engine_plan(torch.float64)
    assert plan.scratch_elements > 0
    coefficients = torch.as_tensor(tp.coefficients, dtype=torch.float64, device="cuda")
    for seed in (1, 2):
        x_host = np.random.default_rng(seed).standard_normal(degeneracy_structure(h).total_dim)
        x = torch.from_numpy(x_host).cuda()
        expected = stride.execute_reduction(x, plan, coefficients)
        out = torch.full((plan.output_size,), float("nan"), dtype=torch.float64, device="cuda")
        status, message = call_static(plan, x, out, coefficients)
        assert status == 0, message
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert relative_error(got, expected.cpu().numpy()) <= TOLERANCE
        oracle = so.reduction(tp.words, x_host, list(tp.coefficients), np.arange(tp.records))
        assert relative_error(got, oracle) <= TOLERANCE


def test_static_scratch_batches_with_per_batch_coefficients():
    """Three batches index the shared array at their own scratch strides."""
    w = space(ProductSector(Z2Irrep, U1Irrep), {(p, q): 2 - p for p in (0, 1) for q in (-1, 0, 1)})
    h = hom((w, w, w), (w, w, w))
    tp = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    plan = tp.engine_plan(torch.float64)
    rng = np.random.default_rng(5)
    batches = 3
    per_batch = rng.choice([0.0, 1.0, -0.5, 2.0], size=(tp.records, batches))
    coefficients = torch.as_tensor(per_batch, dtype=torch.float64, device="cuda").contiguous()
    x_host = rng.standard_normal((batches, degeneracy_structure(h).total_dim))
    x = torch.from_numpy(x_host).cuda()
    expected = stride.execute_reduction(x, plan, coefficients).cpu().numpy()
    for _ in range(2):
        out = torch.full((batches, plan.output_size), float("nan"), dtype=torch.float64, device="cuda")
        status, message = call_static(plan, x, out, coefficients, coefficient_count=batches)
        assert status == 0, message
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert relative_error(got, expected) <= TOLERANCE
        for b in range(batches):
            oracle = so.reduction(tp.words, x_host[b:b + 1], list(per_batch[:, b]), np.arange(tp.records))
            assert relative_error(got[b:b + 1], oracle) <= TOLERANCE


def test_static_scratch_accepts_exactly_the_array_size():
    """A call whose scratch need equals the array size is accepted and correct."""
    record = stride.AffineRecord((8, 4), (4, 1), 0, (1, 0), 0)
    words = stride.encode_reduction_layout([record], output_shapes=[(8, 1)], reduction_axes=[(False, True)],
                                           source_size=32, output_size=8)
    plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=8, coefficient_records=[0])
    assert plan.scratch_elements == 8
    batches = (16 << 20) // (plan.scratch_elements * 8)
    x = torch.randn(batches, 32, dtype=torch.float64, device="cuda")
    coefficients = torch.tensor([0.5], dtype=torch.float64, device="cuda")
    out = torch.full((batches, 8), float("nan"), dtype=torch.float64, device="cuda")
    status, message = call_static(plan, x, out, coefficients)
    assert status == 0, message
    expected = 0.5 * x.reshape(batches, 8, 4).sum(dim=2)
    torch.cuda.synchronize()
    assert relative_error(out.cpu().numpy(), expected.cpu().numpy()) <= TOLERANCE
    bigger = torch.empty(batches + 1, 32, dtype=torch.float64, device="cuda")
    status, message = call_static(plan, bigger, torch.empty(batches + 1, 8, dtype=torch.float64, device="cuda"),
                                  coefficients)
    assert status == 1 and "static scratch holds" in message


def test_static_scratch_rejects_oversize_requests_before_any_work():
    v = space(U1Irrep, {-1: 2, 0: 2, 1: 1})
    h = hom((v, v), (v, v))
    plan = trace_plan(h, (1,), (3,), (0,), (2,)).engine_plan(torch.float64)
    per_batch_bytes = plan.scratch_elements * 8
    batches = (16 << 20) // per_batch_bytes + 1
    err = _native.error_buffer()
    status = _native.lib().t0b_reduction_static_scratch(plan._handle, _native.F64, None, None, batches, None,
                                                        _native.F64, 1, None, None, err, len(err))
    assert status == 1 and b"static scratch holds" in err.value
