"""Oracle restatements of the TensorMap-level steps (permute, adjoint
destination, contraction) built from the planner's records, shared by the CPU
and GPU tests."""

import numpy as np

from oracle import stride_oracle as so
from tensor0_b200.structure import degeneracy_structure, hom
from tensor0_b200.tensor_map import _adjoint_axis, adjoint_plan, contract_plan, permute_plan


def sample(rng, n, complex_values):
    x = rng.standard_normal(n)
    return x + 1j * rng.standard_normal(n) if complex_values else x


def oracle_permute(space_, data, p):
    pp = permute_plan(space_, *p)
    if p == (tuple(range(space_.numout)), tuple(range(space_.numout, space_.numind))):
        return space_, data
    n = len(pp.transform.src)
    return pp.dst, so.accumulation(pp.words, data, list(pp.transform.coeff), np.arange(n))


def oracle_permute_adjoint(space_, data, p):
    """The adjoint-destination records applied by the oracle to conj(data)."""
    pp = adjoint_plan(space_, *p)
    n = len(pp.transform.src)
    return pp.dst, so.accumulation(pp.words, np.conj(data), list(pp.transform.coeff), np.arange(n))


def oracle_contract(left_space, right_space, a, b, axes, output, conjugate=(False, False)):
    """tensorcontract restated with the oracle: the planner's operand
    preparation, per-sector GEMMs in float64 / complex128, output permute."""
    plan = contract_plan(left_space, right_space, tuple(axes[0]), tuple(axes[1]), output, tuple(conjugate))
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

    _, ld = prepared(fs, first, plan.left_p, plan.conjugate[0])
    _, rd = prepared(ss_, second, plan.right_p, plan.conjugate[1])
    c = so.sector_gemm(plan.gemm.spec, ld, rd, degeneracy_structure(plan.canonical).total_dim)
    return oracle_permute(plan.canonical, c, plan.output_p)
