"""Grouped transform (the non-abelian permute's pack -> basis matrix -> unpack,
_stride/_tensor_ops.py:119-203) in one launch.

CPU: the planner's validation (bounds, destination disjointness, the
reference's shape-consistency messages), its choice of tiled and element
groups, and the oracle on the reference's own fixture
(tests/stride/tensor_ops/test_grouped.py:57-62) against values worked out by
hand.  GPU: the kernel against the oracle on that fixture, on random groups
(repeated sources, zero and negative source strides, several batch shapes,
all four storage types, real and complex matrices) and on the 1 x 1
short-circuits.  Single-tree groups are bit-exact; multi-tree groups agree
within 1e-6 (f32/c64) and 1e-12 (f64/c128) of the output's scale.
"""

from types import SimpleNamespace

import numpy as np
import pytest

from oracle import stride_oracle as so
from tensor0_b200 import _native, stride

TOL = {np.float32: 1e-6, np.complex64: 1e-6, np.float64: 1e-12, np.complex128: 1e-12}
DTYPES = [np.float32, np.float64, np.complex64, np.complex128]


def block(shape, strides, offset):
    return SimpleNamespace(sizes=shape, strides=strides, offset=offset)


def fixture(complex_matrix=False):
    """The reference's fixture_layouts (test_grouped.py:57-62)."""
    sources = (block((2, 3), (3, -1), 2), block((2, 3), (0, 1), 3), block((2, 3), (3, 1), 0), block((0, 3), (3, 1), 6))
    destinations = tuple(block((3, 2), (6, 3), offset) for offset in range(3)) + (block((3, 0), (6, 3), 18),)
    matrix = np.asarray([[1, 2, -1], [-1, 0.5, 2]], dtype=np.complex64 if complex_matrix else np.float32)
    if complex_matrix:
        matrix[0, 1] += 1j
    groups = (SimpleNamespace(src_indices=(0, 1, 0), dst_indices=(2, 0), transform=matrix),
              SimpleNamespace(src_indices=(2,), dst_indices=(1,), transform=np.asarray([[-2]])),
              SimpleNamespace(src_indices=(3,), dst_indices=(3,), transform=np.asarray([[3]])))
    return (SimpleNamespace(subblockstructure=sources, total_dim=6),
            SimpleNamespace(subblockstructure=destinations, total_dim=18), groups)


def oracle(source, source_layout, destination_layout, permutation, groups):
    as_tuples = lambda blocks: [(tuple(b.sizes), tuple(b.strides), b.offset) for b in blocks]
    return so.grouped(source, as_tuples(source_layout.subblockstructure),
                      as_tuples(destination_layout.subblockstructure), destination_layout.total_dim, permutation,
                      [(g.src_indices, g.dst_indices, g.transform) for g in groups])


def plan_of(source_layout, destination_layout, permutation, groups, element_bytes=8, source_size=None):
    words, _ = stride.encode_grouped(source_layout.subblockstructure, destination_layout.subblockstructure,
                                     permutation, groups, source_size=source_size or source_layout.total_dim,
                                     output_size=destination_layout.total_dim)
    return stride.Plan(_native.OP_GROUPED, words, element_bytes=element_bytes)


def group_records(plan):
    """(rank, n_src, n_dst, tiled, tx, ty, tz) of each device group record."""
    table = plan.table
    count, offset, operands = int(table[14]), int(table[15]), int(table[16])
    per = (operands - offset) // count if count else 0
    out = []
    for g in range(count):
        words = table[offset + g * per: offset + (g + 1) * per]
        i32 = words[4:].view(np.int32)
        out.append(tuple(int(v) for v in i32[8:15]))
    return out


def test_oracle_on_the_reference_fixture():
    """Worked by hand: source block 0 reads [2, 1, 0, 5, 4, 3], block 1
    [3, 4, 5, 3, 4, 5]; destination 2 = 2 * block 1 and destination 0 =
    block 0 + block 1 / 2, each transposed into (3, 2) blocks of strides
    (6, 3); destination 1 = -2 * block 2 with -0 written as +0."""
    source_layout, destination_layout, groups = fixture()
    got = oracle(np.arange(6, dtype=np.float32), source_layout, destination_layout, (1, 0), groups)
    expected = np.asarray([3.5, 0, 6, 6.5, -6, 6, 3, -2, 8, 6, -8, 8, 2.5, -4, 10, 5.5, -10, 10], np.float32)
    assert np.array_equal(got, expected)
    assert not np.signbit(got[1])


def test_plan_counts_and_coverage():
    source_layout, destination_layout, groups = fixture()
    plan = plan_of(source_layout, destination_layout, (1, 0), groups, element_bytes=4)
    assert plan.matrix_elements == 6 + 1 + 1
    assert plan.info["records"] == 3
    assert plan.info["full_coverage"] == 1          # 12 + 6 + 0 destination elements cover all 18
    assert plan.info["kernels_per_call"] == 1
    assert plan.scratch_elements == 0


def test_tiled_and_element_groups():
    """A transposing permute of d^4 blocks is tiled 16 x 16 x 8 for one f64
    source (X = the destination's innermost axis, Y = the source's); an
    identity permute of contiguous blocks runs one element per thread."""
    shape = (16,) * 4
    for permutation, tiled in (((2, 0, 3, 1), (4, 1, 1, 1, 16, 16, 8)), ((0, 1, 2, 3), None)):
        logical = tuple(shape[p] for p in permutation)
        sources = (block(shape, stride.contiguous_strides(shape), 0),)
        destinations = (block(logical, stride.contiguous_strides(logical), 0),)
        groups = (SimpleNamespace(src_indices=(0,), dst_indices=(0,), transform=np.ones((1, 1))),)
        plan = plan_of(SimpleNamespace(subblockstructure=sources, total_dim=16 ** 4),
                       SimpleNamespace(subblockstructure=destinations, total_dim=16 ** 4), permutation, groups)
        record = group_records(plan)[0]
        if tiled:
            assert record == tiled
        else:
            assert record[:4] == (1, 1, 1, 0)        # contiguous on both sides: one fused axis, not tiled


@pytest.mark.parametrize("side", ["source", "destination"])
def test_shape_consistency_messages(side):
    """The reference's messages (_tensor_ops.py:151-152, 159-160)."""
    source_layout, destination_layout, groups = fixture()
    layout = source_layout if side == "source" else destination_layout
    blocks = list(layout.subblockstructure)
    index = 1 if side == "source" else 0
    blocks[index] = block((1, 6), blocks[index].strides, blocks[index].offset)
    layout.subblockstructure = tuple(blocks)
    with pytest.raises(ValueError, match=f"generic tree transform {side} subblock shapes are inconsistent"):
        plan_of(source_layout, destination_layout, (1, 0), groups)


def test_address_validation():
    """A source larger than the storage (test_grouped.py:206-210's case:
    five source elements) is rejected when the plan is built."""
    source_layout, destination_layout, groups = fixture()
    with pytest.raises(ValueError, match="(?i)(bounds|storage)"):
        plan_of(source_layout, destination_layout, (1, 0), groups, source_size=5)


def test_overlapping_destinations_are_rejected():
    source_layout, destination_layout, groups = fixture()
    blocks = list(destination_layout.subblockstructure)
    blocks[1] = block((3, 2), (6, 3), 0)            # the same addresses as destination 0
    destination_layout.subblockstructure = tuple(blocks)
    with pytest.raises(ValueError, match="not pairwise disjoint"):
        plan_of(source_layout, destination_layout, (1, 0), groups)


@pytest.mark.parametrize("words, message", [
    ([2, 0, 0, 0], "unsupported grouped descriptor version"),
    ([1, 4, 4, 1], "exceeds descriptor length"),
    ([1, 4, 4, 1, 1, 0, 1, 4, 0, 1, 0, 1], "at least one source"),
    ([1, 4, 4, 1, 1, 1, 1, 4, 0, 1, 0, 1, 7], "trailing words"),
    ([1, 4, 4, 1, 1, 1, 1, 4, 1, 1, 0, 1], "source address exceeds storage"),
    ([1, 4, 4, 1, 1, 1, 1, 4, 0, 1, 0, 0], "destination strides do not prove an injective view"),
])
def test_descriptor_errors(words, message):
    with pytest.raises(ValueError, match=message):
        stride.Plan(_native.OP_GROUPED, np.asarray(words, np.int64), element_bytes=8)


# ---------------------------------------------------------------------------
# GPU.

def _cuda(array):
    import torch
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def _host(tensor):
    import torch
    torch.cuda.synchronize()
    return tensor.cpu().numpy()


def _sample(rng, dtype, shape):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    return rng.standard_normal(shape).astype(dtype)


def _close(got, expected, dtype):
    scale = max(float(np.max(np.abs(expected))) if expected.size else 0.0, 1e-300)
    assert got.shape == expected.shape
    if expected.size:
        error = float(np.max(np.abs(got - expected))) / scale
        assert error <= TOL[dtype], f"relative error {error:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_shape", [(), (2,), (2, 0), (3, 2)])
def test_reference_fixture_on_gpu(dtype, batch_shape):
    complex_matrix = np.iscomplexobj(np.zeros(1, dtype))
    source_layout, destination_layout, groups = fixture(complex_matrix)
    rng = np.random.default_rng(2)
    x = _sample(rng, dtype, (*batch_shape, 6))
    got = _host(stride.grouped_transform(_cuda(x), source_layout, destination_layout, dtype, (1, 0), groups))
    expected = oracle(x, source_layout, destination_layout, (1, 0), groups)
    _close(got, expected, dtype)
    # The single-tree groups (destinations 1 and 3) are bit-exact.
    direct = np.asarray([1, 4, 7, 10, 13, 16])
    bits = lambda a: np.ascontiguousarray(a[..., direct]).view(np.uint8)
    assert np.array_equal(bits(got), bits(expected))


def random_groups(rng, permutation, shape, groups, max_trees=5, wide=False):
    """Random groups over one block shape: source blocks with permuted,
    negative or zero strides laid out in a source storage; destination blocks
    packed contiguously (so they cover the output)."""
    rank = len(shape)
    count = int(np.prod(shape))
    sources, destinations, data = [], [], []
    source_size = 0
    logical = tuple(shape[p] for p in permutation)
    out_cursor = 0
    for _ in range(groups):
        n_src = int(rng.integers(1, max_trees + 1)) if not wide else int(rng.integers(9, 14))
        n_dst = int(rng.integers(1, max_trees + 1))
        src_indices = []
        for _ in range(n_src):
            if sources and rng.random() < 0.2:
                src_indices.append(int(rng.integers(0, len(sources))))   # repeated source
                continue
            order = rng.permutation(rank)
            strides = [0] * rank
            step = 1
            for axis in order:
                strides[axis] = step
                step *= shape[axis]
            if rank and rng.random() < 0.3:
                axis = int(rng.integers(0, rank))
                strides[axis] = -strides[axis]
            if rank and rng.random() < 0.1:
                strides[int(rng.integers(0, rank))] = 0
            low = sum((n - 1) * s for n, s in zip(shape, strides) if s < 0)
            high = sum((n - 1) * s for n, s in zip(shape, strides) if s > 0)
            offset = source_size - low + int(rng.integers(0, 3))
            source_size = offset + high + 1
            sources.append(block(shape, tuple(strides), offset))
            src_indices.append(len(sources) - 1)
        dst_indices = []
        for _ in range(n_dst):
            destinations.append(block(logical, stride.contiguous_strides(logical), out_cursor))
            out_cursor += count
            dst_indices.append(len(destinations) - 1)
        data.append(SimpleNamespace(src_indices=tuple(src_indices), dst_indices=tuple(dst_indices),
                                    transform=rng.standard_normal((n_dst, n_src))))
    return (SimpleNamespace(subblockstructure=tuple(sources), total_dim=source_size),
            SimpleNamespace(subblockstructure=tuple(destinations), total_dim=out_cursor), data)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", [((3, 4, 5), (2, 0, 1)), ((7, 1, 33, 2), (1, 3, 2, 0)), ((300,), (0,)),
                                  ((2, 3, 2, 3, 2, 3), (5, 3, 1, 4, 2, 0)), ((40, 9, 13), (1, 2, 0))])
def test_random_groups(dtype, case):
    shape, permutation = case
    rng = np.random.default_rng(sum(shape))
    source_layout, destination_layout, groups = random_groups(rng, permutation, shape, 6)
    x = _sample(rng, dtype, (2, source_layout.total_dim))
    got = _host(stride.grouped_transform(_cuda(x), source_layout, destination_layout, dtype, permutation, groups))
    _close(got, oracle(x, source_layout, destination_layout, permutation, groups), dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [np.float64, np.complex64])
def test_wide_groups_and_complex_matrices(dtype):
    """More sources than the kernel keeps in registers, and (complex storage)
    complex basis matrices."""
    rng = np.random.default_rng(41)
    source_layout, destination_layout, groups = random_groups(rng, (1, 0), (16, 9), 3, wide=True)
    if np.iscomplexobj(np.zeros(1, dtype)):
        for g in groups:
            g.transform = g.transform + 1j * rng.standard_normal(g.transform.shape)
    x = _sample(rng, dtype, (3, source_layout.total_dim))
    got = _host(stride.grouped_transform(_cuda(x), source_layout, destination_layout, dtype, (1, 0), groups))
    _close(got, oracle(x, source_layout, destination_layout, (1, 0), groups), dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("factor", [0, 1])
def test_scalar_short_circuit(factor):
    """test_grouped.py:43-52: a zero factor writes 0 over NaN, a unit factor keeps NaN."""
    layout = SimpleNamespace(subblockstructure=(block((), (), 0),), total_dim=1)
    groups = (SimpleNamespace(src_indices=(0,), dst_indices=(0,), transform=np.asarray([[factor]])),)
    got = _host(stride.grouped_transform(_cuda(np.asarray([np.nan])), layout, layout, np.float64, (), groups))
    assert (got[0] == 0) if factor == 0 else np.isnan(got[0])


@pytest.mark.gpu
def test_uncovered_outputs_are_zero_and_no_groups():
    source_layout, destination_layout, groups = fixture()
    x = np.arange(6, dtype=np.float64)
    # Only the multi-tree group: destinations 1 and 3 are not written.
    got = _host(stride.grouped_transform(_cuda(x), source_layout, destination_layout, np.float64, (1, 0),
                                         groups[:1]))
    _close(got, oracle(x, source_layout, destination_layout, (1, 0), groups[:1]), np.float64)
    assert np.all(got[[1, 4, 7, 10, 13, 16]] == 0)
    empty = SimpleNamespace(subblockstructure=(), total_dim=0)
    assert _host(stride.grouped_transform(_cuda(np.zeros((2, 0))), empty, empty, np.float64, (), ())).shape == (2, 0)
