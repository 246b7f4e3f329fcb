"""Planner records executed by the NumPy oracle satisfy the reference's dense
contracts: permute = transpose of to_dense (tests/test_transforms.py:685-692),
trace = dense trace (tests/test_contractions.py:669-726) and contraction =
tensordot (tests/test_contractions.py:374-391)."""

import numpy as np
import pytest

from oracle import dense, stride_oracle as so
from tensor0_b200.structure import (ProductSector, U1Irrep, Z2Irrep, Z3Irrep, degeneracy_structure, hom,
                                    space)
from oracle_steps import oracle_permute, oracle_permute_adjoint, sample
from tensor0_b200.tensor_map import _adjoint_axis, _compose_spec, contract_plan, permute_plan, trace_plan


def u1_space(dims):
    return space(U1Irrep, dims)


def z2u1_space(deg0, deg1, charges=range(-1, 2)):
    return space(ProductSector(Z2Irrep, U1Irrep), {(p, q): (deg0 if p == 0 else deg1) for p in (0, 1) for q in charges})


def z2z3u1_space(seed, charges=range(-1, 2), high=3):
    rng = np.random.default_rng(seed)
    st = ProductSector(Z2Irrep, Z3Irrep, U1Irrep)
    return space(st, {(a, b, q): int(rng.integers(1, high + 1)) for a in (0, 1) for b in range(3) for q in charges})


PERMUTES = [
    (lambda: hom((u1_space({-1: 2, 0: 3, 1: 2}),) * 2, (u1_space({-1: 2, 0: 3, 1: 2}),) * 2), ((1, 0), (3, 2))),
    (lambda: hom((u1_space({-1: 2, 0: 3, 1: 2}),) * 2, (u1_space({-1: 2, 0: 3, 1: 2}),) * 2), ((2, 0), (3, 1))),
    (lambda: hom((u1_space({-1: 2, 0: 3, 1: 2}), u1_space({0: 2, 1: 1})), (u1_space({-1: 1, 0: 2}),)),
     ((2,), (0, 1))),
    (lambda: hom((z2u1_space(2, 1),) * 2, (z2u1_space(1, 2),)), ((1, 2), (0,))),
    (lambda: hom((z2z3u1_space(1),) * 2, (z2z3u1_space(2),)), ((2, 0), (1,))),
]


@pytest.mark.parametrize("index", range(len(PERMUTES)))
def test_permute_records_are_a_dense_transpose(index):
    make, (pc, pd) = PERMUTES[index]
    h = make()
    plan = permute_plan(h, pc, pd)
    x = np.random.default_rng(index).standard_normal(degeneracy_structure(h).total_dim)
    n = len(plan.transform.src)
    y = so.accumulation(plan.words, x, [np.float64(1)] * n, np.arange(n))
    assert plan.outputs_disjoint
    assert np.array_equal(dense.to_dense(plan.dst, y), dense.permute(dense.to_dense(h, x), pc, pd))
    # Every destination element is written exactly once.
    assert sorted(plan.transform.dst.tolist()) == list(range(len(degeneracy_structure(plan.dst).offsets)))


def test_partial_trace_records_match_dense_trace():
    w = z2u1_space(2, 1)
    h = hom((w, w, w), (w, w, w))
    plan = trace_plan(h, (1, 2), (4, 5), (0,), (3,))
    x = np.random.default_rng(3).standard_normal(degeneracy_structure(h).total_dim)
    y = so.reduction(plan.words, x, list(plan.coefficients), np.arange(plan.records))
    expected = dense.trace(dense.to_dense(h, x), (1, 2), (4, 5), (0,), (3,))
    np.testing.assert_allclose(dense.to_dense(plan.dst, y), expected, rtol=1e-12, atol=1e-12)


def test_partial_trace_with_permuted_output():
    v = u1_space({-1: 2, 0: 2, 1: 1})
    h = hom((v, v), (v, v))
    plan = trace_plan(h, (1,), (3,), (0,), (2,))
    x = np.random.default_rng(4).standard_normal(degeneracy_structure(h).total_dim)
    y = so.reduction(plan.words, x, list(plan.coefficients), np.arange(plan.records))
    expected = dense.trace(dense.to_dense(h, x), (1,), (3,), (0,), (2,))
    np.testing.assert_allclose(dense.to_dense(plan.dst, y), expected, rtol=1e-12, atol=1e-12)


def run_contract(left_space, right_space, axes, output, seed, conjugate=(False, False), complex_values=False):
    plan = contract_plan(left_space, right_space, axes[0], axes[1], output, conjugate)
    rng = np.random.default_rng(seed)
    a = sample(rng, degeneracy_structure(left_space).total_dim, complex_values)
    b = sample(rng, degeneracy_structure(right_space).total_dim, complex_values)
    if plan.reversed_operands:
        first, second, fs, ss_ = b, a, right_space, left_space
    else:
        first, second, fs, ss_ = a, b, left_space, right_space

    def prepared(space_, data, p, conj):
        if not conj:
            return oracle_permute(space_, data, p)
        adjoint_space = hom(space_.domain, space_.codomain)
        parent = (tuple(_adjoint_axis(adjoint_space, x) for x in p[1]),
                  tuple(_adjoint_axis(adjoint_space, x) for x in p[0]))
        return oracle_permute_adjoint(space_, data, parent)

    ls, ld = prepared(fs, first, plan.left_p, plan.conjugate[0])
    rs, rd = prepared(ss_, second, plan.right_p, plan.conjugate[1])
    c = so.sector_gemm(plan.gemm.spec, ld, rd, degeneracy_structure(plan.canonical).total_dim)
    rs_, rd_ = oracle_permute(plan.canonical, c, plan.output_p)
    da, db = dense.to_dense(left_space, a), dense.to_dense(right_space, b)
    expected = dense.contract(np.conj(da) if conjugate[0] else da, np.conj(db) if conjugate[1] else db,
                              axes[0], axes[1], output)
    np.testing.assert_allclose(dense.to_dense(rs_, rd_), expected, rtol=1e-12, atol=1e-12)
    assert rs_ == plan.result


def test_contraction_matches_tensordot():
    v = u1_space({-1: 2, 0: 3, 1: 2})
    d = u1_space({0: 1, 1: 1})
    a_space = hom((v, d), (v,))
    b_space = hom((v,), (v, d))
    run_contract(a_space, b_space, ((2,), (0,)), (((0, 0), (0, 1)), ((1, 1), (1, 2))), 0)
    run_contract(a_space, b_space, ((0,), (1,)), (((0, 1), (1, 0)), ((0, 2), (1, 2))), 1)


def test_dmrg_style_environment_contraction():
    chi = u1_space({-1: 3, 0: 4, 1: 3})
    phys = u1_space({0: 1, 1: 1})
    w = u1_space({0: 2})
    A = hom((chi, phys), (chi,))
    L = hom((chi,), (chi, w))
    run_contract(L, A, ((1,), (0,)), (((0, 0), (1, 1)), ((0, 2), (1, 2))), 2)


def test_compose_spec_zero_blocks():
    v = u1_space({0: 2, 1: 1})
    u = u1_space({0: 1})
    left, right = hom((v,), (u,)), hom((u,), (v,))
    spec = _compose_spec(left, right, hom((v,), (v,)))
    assert spec.shape == (2, 6)
    assert spec[1, 2] == 0  # sector 1 is absent from the shared middle space: zero block


ADJOINTS = [
    (lambda: hom((u1_space({-1: 2, 0: 3, 1: 2}),) * 2, (u1_space({-1: 2, 0: 3, 1: 2}),) * 2), ((0, 1), (2, 3))),
    (lambda: hom((u1_space({-1: 2, 0: 3, 1: 2}),) * 2, (u1_space({-1: 2, 0: 3, 1: 2}),) * 2), ((2, 0), (3, 1))),
    (lambda: hom((z2z3u1_space(1),) * 2, (z2z3u1_space(2),)), ((2, 0), (1,))),
    (lambda: hom((z2z3u1_space(3),) * 3, (z2z3u1_space(4),) * 2), ((0, 1, 2), (3, 4))),
]


@pytest.mark.parametrize("index", range(len(ADJOINTS)))
def test_adjoint_destination_is_the_dense_conjugate_transpose(index):
    """adjoint(permute(t, p)) = conj of the permuted dense array with its
    domain legs first (tensor_map.py:503-515; transforms.py:190-259)."""
    make, (pc, pd) = ADJOINTS[index]
    h = make()
    x = sample(np.random.default_rng(index), degeneracy_structure(h).total_dim, True)
    dst, y = oracle_permute_adjoint(h, x, (pc, pd))
    assert dst == hom(h.permute(pc, pd).domain, h.permute(pc, pd).codomain)
    permuted = dense.permute(dense.to_dense(h, x), pc, pd)
    order = tuple(range(len(pc), len(pc) + len(pd))) + tuple(range(len(pc)))
    assert np.array_equal(dense.to_dense(dst, y), np.conj(np.transpose(permuted, order)))


def test_conjugated_contractions_match_tensordot_of_conjugates():
    v = u1_space({-1: 2, 0: 3, 1: 2})
    a_space = hom((v, v), (v,))
    run_contract(a_space, a_space, ((2,), (2,)), (((0, 0), (0, 1)), ((1, 0), (1, 1))), 5, (False, True), True)
    run_contract(a_space, a_space, ((0, 1), (0, 1)), (((0, 2),), ((1, 2),)), 6, (True, False), True)
    run_contract(a_space, a_space, ((2,), (0,)), (((0, 0), (1, 1)), ((0, 1), (1, 2))), 7, (True, True), True)


def test_configuration_five_chain_contraction_with_adjoint():
    """Z2 x Z3 x U(1) 5-leg tensor contracted with its adjoint over its two
    domain legs (the many-small-block chain's last step, scaled down)."""
    w = z2z3u1_space(11, charges=range(0, 2), high=2)
    h = hom((w, w, w), (w, w))
    output = (((0, 0), (0, 1), (0, 2)), ((1, 0), (1, 1), (1, 2)))
    run_contract(h, h, ((3, 4), (3, 4)), output, 8, (False, True), True)
