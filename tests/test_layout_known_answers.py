"""Planner layouts against the reference's Rust known answers
(crates/tensor0-core/tests/layout.rs).  U1 sectors there are given as twice
the charge (``u1(charge2)``); here ``space`` takes charges, so ``u1(1)`` is 0.5."""

import numpy as np

from tensor0_b200.structure import (U1Irrep, Z2Irrep, ProductSector, degeneracy_structure, hom,
                                    sector_structure, space)


def charges2(ss):
    return [int(s[0]) for s in ss.blocksectors]


def test_single_factor_order_dims_and_offsets():
    # layout.rs:315-345
    v = space(U1Irrep, {-0.5: 5, 0: 2, 0.5: 3})
    h = hom((v,), (v,))
    ss, ds = sector_structure(h), degeneracy_structure(h)
    assert charges2(ss) == [0, 1, -1]
    assert list(zip(ds.block_rows, ds.block_cols)) == [(2, 2), (3, 3), (5, 5)]
    assert ds.offsets.tolist() == [0, 4, 13]
    assert ds.sizes.tolist() == [[2, 2], [3, 3], [5, 5]]
    assert ds.strides.tolist() == [[2, 1], [3, 1], [5, 1]]


def test_single_factor_dual_order():
    # layout.rs:347-365: visible sectors of a dual space are the duals of the stored ones
    v = space(U1Irrep, {0.5: 3, -0.5: 5}, dual=True)
    h = hom((v,), (v,))
    ss, ds = sector_structure(h), degeneracy_structure(h)
    assert charges2(ss) == [1, -1]
    assert list(zip(ds.block_rows, ds.block_cols)) == [(5, 5), (3, 3)]


def test_two_factor_tree_order_and_row_major_subblocks():
    # layout.rs:368-405
    c = (space(U1Irrep, {-0.5: 5, 0: 2, 0.5: 3}), space(U1Irrep, {-0.5: 13, 0: 7, 0.5: 11}))
    d = (space(U1Irrep, {-0.5: 17, 0: 19, 0.5: 23}), space(U1Irrep, {-0.5: 29, 0: 31, 0.5: 37}))
    h = hom(c, d)
    ss, ds = sector_structure(h), degeneracy_structure(h)
    assert charges2(ss) == [0, 1, -1, 2, -2]
    assert list(zip(ds.block_rows, ds.block_cols)) == [(108, 1885), (43, 1416), (61, 1078), (33, 851), (65, 493)]
    assert ds.offsets[:9].tolist() == [0, 589, 1218, 26390, 26979, 27608, 130065, 130654, 131283]
    assert ds.sizes[0].tolist() == [2, 7, 19, 31] and ds.strides[0].tolist() == [13195, 1885, 31, 1]
    assert ds.sizes[4].tolist() == [5, 11, 17, 37] and ds.strides[4].tolist() == [20735, 1885, 37, 1]
    assert int(ds.offsets[4]) == 26979
    # layout.rs:236-263: uncoupled order of the first nine pairs (charge2 units)
    visible = [0, 1, -1]
    rows = [[visible[i] for i in r] for r in ss.pair_row[:9].tolist()]
    cols = [[visible[i] for i in c] for c in ss.pair_col[:9].tolist()]
    expected = [([0, 0], [0, 0]), ([0, 0], [-1, 1]), ([0, 0], [1, -1]), ([-1, 1], [0, 0]), ([-1, 1], [-1, 1]),
                ([-1, 1], [1, -1]), ([1, -1], [0, 0]), ([1, -1], [-1, 1]), ([1, -1], [1, -1])]
    assert list(zip(rows, cols)) == expected


def test_three_factor_one_sided_layouts():
    # layout.rs:407-435
    legs = (space(U1Irrep, {0.5: 2}), space(U1Irrep, {-1.5: 5}), space(U1Irrep, {1: 7}))
    for h, dims in ((hom(legs, ()), (70, 1)), (hom((), legs), (1, 70))):
        ss, ds = sector_structure(h), degeneracy_structure(h)
        assert charges2(ss) == [0]
        assert (int(ds.block_rows[0]), int(ds.block_cols[0])) == dims
        assert ds.sizes[0].tolist() == [2, 5, 7] and ds.strides[0].tolist() == [35, 7, 1]


def test_scalar_and_empty_spaces():
    assert degeneracy_structure(hom((), ())).total_dim == 1
    zero = space(U1Irrep, {})
    assert degeneracy_structure(hom((zero,), ())).total_dim == 0


def test_product_sector_order_is_manhattan():
    # product.rs:403-411: by the sum of component indices, then the indices.
    # Component indices: Z2 value; U1 0, 1, -1 -> 0, 3, 4 (u1.rs:123-130 on twice the charge).
    st = ProductSector(Z2Irrep, U1Irrep)
    v = space(st, {(p, q): 1 for p in (0, 1) for q in (-1, 0, 1)})
    stored = [tuple(s) for s in v.stored]
    assert stored == [(0, 0), (1, 0), (0, 2), (0, -2), (1, 2), (1, -2)]


def test_benchmark_space_sizes():
    # Sizes of the benchmark workloads (storage elements, blocks, sub-blocks).
    v = space(U1Irrep, {-2: 4, -1: 8, 0: 12, 1: 8, 2: 4})
    ds = degeneracy_structure(hom((v, v), (v, v)))
    assert (ds.total_dim, len(ds.block_start), len(ds.offsets)) == (283392, 9, 85)
    degs = {q: round(64 * np.exp(-q * q / 8)) for q in range(-4, 5)}
    assert list(degs.values()) == [9, 21, 39, 56, 64, 56, 39, 21, 9]
    w = space(U1Irrep, degs)
    ds = degeneracy_structure(hom((w, w), (w, w)))
    assert (ds.total_dim, len(ds.block_start), len(ds.offsets)) == (1023777634, 17, 489)


# ---------------------------------------------------------------------------
# Fermionic coefficients, twists, flips and traces
# (crates/tensor0-core/tests/transform.rs).

from tensor0_b200.structure import (FermionParity, flip_transform, trace_transformer, tree_permuter,  # noqa: E402
                                    twist_factors)


def fp(values):
    return space(FermionParity, values)


def test_fermion_parity_braid_coefficients():
    # transform.rs:432-484
    odd2, odd3, odd5, odd7 = fp({1: 2}), fp({1: 3}), fp({1: 5}), fp({1: 7})
    even = fp({0: 1})
    _, t = tree_permuter(hom((odd2, odd3), ()), (1, 0), ())
    assert t.coeff.tolist() == [-1.0]
    _, t = tree_permuter(hom((even, fp({1: 1})), (fp({1: 1}),)), (1, 0), (2,))
    assert t.coeff.tolist() == [1.0]
    number = ProductSector(U1Irrep, FermionParity)
    left, right = space(number, {(0.5, 1): 1}), space(number, {(-0.5, 1): 1})
    _, t = tree_permuter(hom((left, right), ()), (1, 0), ())
    assert t.coeff.tolist() == [-1.0]
    _, t = tree_permuter(hom((odd2,), (odd3,)), (1,), (0,))
    assert t.coeff.tolist() == [-1.0]
    _, t = tree_permuter(hom((odd2, odd3, odd5, odd7), ()), (1, 2, 0, 3), ())
    assert t.coeff.tolist() == [1.0]


def test_twist_factors_follow_pair_order():
    # transform.rs:835-871
    v = fp({0: 1, 1: 1})
    h = hom((v,), (v,))
    assert twist_factors(h, (0,)).tolist() == [1.0, -1.0]
    assert twist_factors(h, (1,)).tolist() == [1.0, -1.0]
    assert twist_factors(h, (0, 1)) is None
    assert twist_factors(h, (0,), inv=True).tolist() == [1.0, -1.0]
    odd, even = fp({1: 1}), fp({0: 1})
    h = hom((odd, odd), (even, even))
    assert twist_factors(h, (0,)).tolist() == [-1.0]
    assert twist_factors(h, (2,)) is None
    u = space(U1Irrep, {0: 1, 0.5: 1})
    assert twist_factors(hom((u,), (u,)), (0,)) is None


def test_flip_entries():
    # transform.rs:904-930, 961-970
    f = space(U1Irrep, {-0.5: 2, 0: 3, 0.5: 5})
    _, t = flip_transform(hom((f,), (f,)), (0, 1))
    assert t.coeff.tolist() == [1.0] * len(t.coeff) and t.dst.tolist() == list(range(len(t.dst)))
    g = space(U1Irrep, {-0.5: 1, 0.5: 1})
    _, t = flip_transform(hom((g, g), ()), (1,))
    assert list(zip(t.dst.tolist(), t.coeff.tolist())) == [(1, 1.0), (0, 1.0)]
    number = ProductSector(U1Irrep, FermionParity)
    odd = space(number, {(0.5, 1): 1})
    h = hom((odd,), (odd,))
    assert flip_transform(h, (0,))[1].coeff.tolist() == [1.0]
    assert flip_transform(h, (1,))[1].coeff.tolist() == [-1.0]


def test_fermion_trace_twists_only_nondual_tail_sectors():
    # transform.rs:723-740
    for dual, expected in ((False, -1.0), (True, 1.0)):
        odd = fp({1: 1}) if not dual else space(FermionParity, {1: 1}, dual=True)
        src = hom((odd,), (odd,))
        dst = hom((), ())
        canonical, basis = tree_permuter(src, (0,), (1,))
        t = trace_transformer(canonical, dst, basis)
        assert t.coeff.tolist() == [expected]
