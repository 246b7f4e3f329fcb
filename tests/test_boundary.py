"""The C-ABI library: it loads without a GPU, exports every symbol the header
declares, and its plan validation reproduces the reference's error classes and
messages (crates/tensor0-py/native/layout/descriptor.cc:14-165; errors map to
InvalidArgument = status 1, ffi/errors.h:12-24).  No compute call runs here."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from tensor0_b200 import _native, build, stride

HEADER = Path(__file__).resolve().parents[1] / "include" / "tensor0_b200.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _native.lib()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(t0b_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 17
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.SIGNATURES)


def test_version(lib):
    assert b"sm_100a" in lib.t0b_version()


def plan_error(operation, words, element_bytes=8, records=()):
    with pytest.raises(ValueError) as error:
        stride.Plan(operation, np.asarray(words, np.int64), element_bytes=element_bytes, coefficient_records=records)
    return str(error.value)


@pytest.mark.parametrize("words, message", [
    ([2, 1, 1, 0], "unsupported native layout version"),
    ([1, -1, 1, 0], "layout size or offset is negative"),
    ([1, 4, 4, 5], "layout record count exceeds descriptor length"),
    ([1, 4], "layout descriptor is truncated"),
    ([1, 4, 4, 1, 1, 0, 0], "layout rank exceeds descriptor length"),
    ([1, 4, 4, 1, 9, 0, 0, 1, 1, 1], "layout rank exceeds descriptor length"),
    ([1, 4, 4, 1, 1, 0, 0, 4, 1, 1, 7], "layout descriptor has trailing words"),
    ([1, 4, 4, 1, 1, 0, 0, 5, 1, 1], "source address exceeds storage"),
    ([1, 4, 4, 1, 1, 0, 0, 2, -1, 1], "source address precedes storage"),
    ([1, 4, 4, 1, 1, 0, 1, 4, 1, 1], "destination address exceeds storage"),
    ([1, 4, 4, 1, 2, 0, 0, 2, 2, 1, 1, 1, 1], "destination strides do not prove an injective view"),
])
def test_copy_descriptor_validation(lib, words, message):
    assert message in plan_error(_native.OP_COPY, words)
    from oracle import ref
    if ref.available():
        # The compiled reference rejects the same words with the same message.
        with pytest.raises(ref.ReferenceError) as error:
            ref.prepare_layout(0, words)
        assert error.value.status == 1 and message in str(error.value)


def test_accumulation_allows_zero_stride_fibers_but_not_collisions(lib):
    fiber = [1, 4, 2, 1, 2, 0, 0, 2, 2, 2, 1, 1, 0]
    plan = stride.Plan(_native.OP_ACCUMULATION, np.asarray(fiber), element_bytes=8)
    assert plan.output_size == 2
    colliding = [1, 4, 4, 1, 2, 0, 0, 2, 2, 1, 1, 1, 1]
    assert "accumulation cannot prove injective output owners" in plan_error(_native.OP_ACCUMULATION, colliding)


def test_coefficient_records_must_increase(lib):
    words = [1, 4, 4, 2, 1, 0, 0, 2, 1, 1, 1, 2, 2, 2, 1, 1]
    message = plan_error(_native.OP_ACCUMULATION, words, records=[1, 0])
    assert "CUDA accumulation coefficient records must be increasing valid record indices" in message
    assert "valid record indices" in plan_error(_native.OP_ACCUMULATION, words, records=[2])


def test_reduction_validation(lib):
    words = stride.encode_reduction_layout(
        [stride.AffineRecord((2, 2), (2, 1), 0, (1, 0), 0)], output_shapes=[(2, 1)],
        reduction_axes=[(False, True)], source_size=4, output_size=2)
    plan = stride.Plan(_native.OP_REDUCTION, words, element_bytes=8)
    assert plan.scratch_elements > 0
    bad = words.copy()
    bad[-1] = 2
    assert "reduction layout axis flag is not boolean" in plan_error(_native.OP_REDUCTION, bad)
    wrong = stride.encode_reduction_layout(
        [stride.AffineRecord((2, 2), (2, 1), 0, (1, 0), 0)], output_shapes=[(2, 2)],
        reduction_axes=[(False, True)], source_size=4, output_size=2)
    assert "reduction input/output shapes do not match axis roles" in plan_error(_native.OP_REDUCTION, wrong)


def test_plan_lifecycle_counters(lib):
    created = lib.t0b_plan_created_count()
    destroyed = lib.t0b_plan_destroyed_count()
    plan = stride.Plan(_native.OP_COPY, np.asarray([1, 4, 4, 1, 1, 0, 0, 4, 1, 1]), element_bytes=4)
    assert plan.info["full_coverage"] == 1
    assert lib.t0b_plan_created_count() == created + 1
    del plan
    assert lib.t0b_plan_destroyed_count() == destroyed + 1


def test_unknown_dtype_is_rejected_before_any_device_work(lib):
    plan = stride.Plan(_native.OP_COPY, np.asarray([1, 4, 4, 1, 1, 0, 0, 4, 1, 1]), element_bytes=4)
    err = _native.error_buffer()
    status = lib.t0b_copy(plan._handle, 9, None, None, 1, None, None, err, len(err))
    assert status == 1 and b"F32/F64/C64/C128" in err.value
    status = lib.t0b_copy(plan._handle, _native.F64, None, None, 1, None, None, err, len(err))
    assert status == 1 and b"element size" in err.value


def test_overlapping_buffers_are_rejected(lib):
    plan = stride.Plan(_native.OP_COPY, np.asarray([1, 4, 4, 1, 1, 0, 0, 4, 1, 1]), element_bytes=4)
    err = _native.error_buffer()
    table = ctypes.c_void_p(0x20000)
    status = lib.t0b_copy(plan._handle, _native.F32, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1008), 1,
                          table, None, err, len(err))
    assert status == 1 and b"overlap" in err.value


def test_misaligned_buffers_are_rejected(lib):
    """Storage buffers must be aligned to their element size (checked before any launch)."""
    words = np.asarray([1, 4, 4, 1, 1, 0, 0, 4, 1, 1])
    err = _native.error_buffer()
    table = ctypes.c_void_p(0x20000)
    copy = stride.Plan(_native.OP_COPY, words, element_bytes=4)
    status = lib.t0b_copy(copy._handle, _native.F32, ctypes.c_void_p(0x1002), ctypes.c_void_p(0x3000), 1,
                          table, None, err, len(err))
    assert status == 1 and b"source buffer is not aligned" in err.value
    wide = stride.Plan(_native.OP_COPY, words, element_bytes=16)
    status = lib.t0b_copy(wide._handle, _native.C128, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x3008), 1,
                          table, None, err, len(err))
    assert status == 1 and b"output buffer is not aligned" in err.value
    update = stride.Plan(_native.OP_UPDATE, words, element_bytes=8)
    alpha = ctypes.c_void_p(0x5000)
    status = lib.t0b_update(update._handle, _native.F64, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x3004),
                            ctypes.c_void_p(0x4000), 1, alpha, _native.F64, 1, alpha, _native.F64, 1,
                            table, None, err, len(err))
    assert status == 1 and b"base buffer is not aligned" in err.value


def test_map_tiling_covers_every_element(lib):
    """The packed table's tiles account for every element of every record."""
    from tensor0_b200.structure import U1Irrep, hom, space
    from tensor0_b200.tensor_map import permute_plan
    v = space(U1Irrep, {-2: 4, -1: 8, 0: 12, 1: 8, 2: 4})
    plan = permute_plan(hom((v, v), (v, v)), (1, 0), (3, 2))
    import torch
    engine = plan.engine_plan(_native.OP_ACCUMULATION, torch.float64)
    assert engine.info["full_coverage"] == 1
    assert engine.info["kernels_per_call"] == 1
    assert engine.info["records"] == 85


def gemm_call(lib, dtype, spec, left, left_size, right, right_size, output, output_size):
    plan = stride.GemmPlan(np.asarray(spec))
    err = _native.error_buffer()
    status = lib.t0b_sector_gemm(dtype, plan.sectors, plan.table.ctypes.data_as(_native.c_i64p),
                                 ctypes.c_void_p(0x90000), ctypes.c_void_p(left), left_size, ctypes.c_void_p(right),
                                 right_size, ctypes.c_void_p(output), output_size, None, err, len(err))
    return status, err.value


def test_sector_gemm_validates_operands_before_any_launch(lib):
    """Rows outside their operands, overlapping output blocks, misaligned or
    overlapping operands are rejected with status 1 and launch nothing."""
    launches = lib.t0b_kernel_launches()
    spec = [[4, 4, 4, 0, 0, 0]]
    status, message = gemm_call(lib, _native.F64, spec, 0x1000, 15, 0x2000, 16, 0x3000, 16)
    assert status == 1 and b"left block lies outside" in message
    status, message = gemm_call(lib, _native.F64, spec, 0x1000, 16, 0x2000, 12, 0x3000, 16)
    assert status == 1 and b"right block lies outside" in message
    status, message = gemm_call(lib, _native.F64, spec, 0x1000, 16, 0x2000, 16, 0x3000, 15)
    assert status == 1 and b"output block lies outside" in message
    status, message = gemm_call(lib, _native.F64, [[2, 2, 2, 0, 0, 0], [2, 2, 2, 0, 0, 3]],
                                0x1000, 4, 0x2000, 4, 0x3000, 8)
    assert status == 1 and b"output blocks overlap" in message
    status, message = gemm_call(lib, _native.C128, spec, 0x1000, 16, 0x2008, 16, 0x3000, 16)
    assert status == 1 and b"not aligned" in message
    status, message = gemm_call(lib, _native.F32, spec, 0x1000, 16, 0x2000, 16, 0x1020, 16)
    assert status == 1 and b"overlap" in message
    assert lib.t0b_kernel_launches() == launches


def test_gemm_table_carries_both_tile_prefixes(lib):
    """Row 6 counts 64 x 64 tiles (DMMA), row 7 128 x 64 tiles (tcgen05); a
    table whose prefixes disagree with its sizes is rejected before launch."""
    spec = np.array([[70, 33, 129, 0, 0, 0], [300, 200, 8, 0, 0, 2310], [0, 4, 3, 0, 0, 62310]])
    plan = stride.GemmPlan(spec)
    rows = plan.table.reshape(-1, 8)
    assert list(rows[:, 6]) == [0, 2, 2 + 5 * 4]
    assert list(rows[:, 7]) == [0, 1, 1 + 3 * 4]
    tampered = plan.table.copy()
    tampered[8 + 7] += 1
    err = _native.error_buffer()
    status = lib.t0b_sector_gemm(_native.F32, plan.sectors, tampered.ctypes.data_as(_native.c_i64p),
                                 ctypes.c_void_p(0x90000), ctypes.c_void_p(0x1000), 1 << 20, ctypes.c_void_p(0x400000),
                                 1 << 20, ctypes.c_void_p(0x800000), 1 << 20, None, err, len(err))
    assert status == 1 and b"tile prefix is inconsistent" in err.value


def test_disjointness_is_proven_for_large_packed_permutes(lib):
    """Without the producer's assertion the planner proves the full-size U(1)
    4-leg permute disjoint (1.02e9 outputs, beyond a bitmap's reach) by the
    block-row radix decomposition, so accumulation stays one map launch."""
    from tensor0_b200.structure import U1Irrep, hom, space
    from tensor0_b200.tensor_map import permute_plan
    degs = {q: int(round(64 * np.exp(-q * q / 8))) for q in range(-4, 5)}
    v = space(U1Irrep, degs)
    for p in (((2, 0), (3, 1)), ((1, 0), (3, 2)), ((3,), (0, 1, 2))):
        plan = permute_plan(hom((v, v), (v, v)), *p)
        engine = stride.Plan(_native.OP_ACCUMULATION, plan.words, element_bytes=4,
                             coefficient_records=np.arange(len(plan.transform.src)))
        assert engine.output_size > 1 << 28
        assert engine.info["kernels_per_call"] == 1 and engine.info["full_coverage"] == 1


def test_overlap_beyond_the_bitmap_reach_is_not_proven(lib):
    """Records that share an address over a span too large for the exact
    check run in record order (one reduce wave per record)."""
    big = 1 << 29
    records = [stride.AffineRecord((2,), (1,), 0, (big,), 0), stride.AffineRecord((2,), (1,), 2, (big,), big)]
    words = stride.encode_layout(records, source_size=4, output_size=2 * big + 1)
    engine = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=8, coefficient_records=[0, 1])
    assert engine.info["kernels_per_call"] == 4
    interleaved = [stride.AffineRecord((3, 2), (2, 1), 0, (big, 1), 0),
                   stride.AffineRecord((3, 2), (2, 1), 6, (big, 1), 2)]
    words = stride.encode_layout(interleaved, source_size=12, output_size=2 * big + 4)
    engine = stride.Plan(_native.OP_ACCUMULATION, words, element_bytes=8, coefficient_records=[0, 1])
    assert engine.info["kernels_per_call"] == 1
