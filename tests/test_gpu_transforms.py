"""Parity of the conjugating, fermionic and reweighting transforms on the
sm_100a engine with the oracle, and the scaled many-small-block chain.

* adjoint / permute-to-adjoint: one conjugating accumulation, bit-exact with
  the oracle applied to the conjugated source (transforms.py:190-259);
* fermion-parity permutes, twists and flips: +-1 coefficients, bit-exact;
* the Z2 x Z3 x U(1) 5-leg complex128 chain — permute, add_transform with
  alpha = 0.7 + 0.2i and beta = 1, contraction with its own adjoint over the
  two domain legs — against the oracle (1e-12), and at a small size against
  dense arithmetic on to_dense.
"""

import numpy as np
import pytest
import torch

from oracle import dense, stride_oracle as so
from oracle_steps import oracle_contract, oracle_permute, oracle_permute_adjoint
from tensor0_b200.structure import (FermionParity, ProductSector, U1Irrep, Z2Irrep, Z3Irrep, degeneracy_structure,
                                    hom, space)
from tensor0_b200.tensor_map import (TensorMap, add_transform, adjoint, flip, flip_plan, permute, permute_adjoint,
                                     permute_plan, tensorcontract, twist, twist_plan)

pytestmark = pytest.mark.gpu

TORCH = {np.float32: torch.float32, np.float64: torch.float64, np.complex64: torch.complex64,
         np.complex128: torch.complex128}
DTYPES = [np.float32, np.float64, np.complex64, np.complex128]


def host(tensor):
    torch.cuda.synchronize()
    return tensor.cpu().numpy()


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def sample(rng, dtype, n):
    if np.iscomplexobj(np.zeros(1, dtype)):
        return (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(dtype)
    return rng.standard_normal(n).astype(dtype)


def relative_error(actual, expected):
    return float(np.max(np.abs(actual - expected))) / max(float(np.max(np.abs(expected))), 1e-300)


def z2z3u1(seed, charges, high):
    rng = np.random.default_rng(seed)
    st = ProductSector(Z2Irrep, Z3Irrep, U1Irrep)
    return space(st, {(a, b, q): int(rng.integers(1, high + 1)) for a in (0, 1) for b in range(3) for q in charges})


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("p", [((0, 1), (2, 3)), ((2, 0), (3, 1)), ((3,), (1, 0, 2))])
def test_permute_adjoint_bit_exact(dtype, p):
    v = space(U1Irrep, {-1: 5, 0: 9, 1: 4, 2: 3})
    h = hom((v, v), (v, v))
    x = sample(np.random.default_rng(1), dtype, degeneracy_structure(h).total_dim)
    got = permute_adjoint(TensorMap(h, torch.from_numpy(x).cuda()), p)
    dst, expected = oracle_permute_adjoint(h, x, p)
    assert got.space == dst
    assert np.array_equal(bits(host(got.data)), bits(expected.astype(dtype)))
    if p == ((0, 1), (2, 3)):
        again = adjoint(TensorMap(h, torch.from_numpy(x).cuda()))
        assert np.array_equal(bits(host(again.data)), bits(expected.astype(dtype)))


@pytest.mark.parametrize("dtype", DTYPES)
def test_fermionic_permute_twist_flip_bit_exact(dtype):
    st = ProductSector(FermionParity, U1Irrep)
    v = space(st, {(0, 0): 3, (1, 0): 2, (0, 1): 4, (1, 1): 5, (1, -1): 2})
    h = hom((v, v), (v, v))
    x = sample(np.random.default_rng(2), dtype, degeneracy_structure(h).total_dim)
    t = TensorMap(h, torch.from_numpy(x).cuda())
    for p in (((1, 0), (2, 3)), ((2, 0), (3, 1)), ((3, 1, 0), (2,))):
        plan = permute_plan(h, *p)
        assert np.any(plan.transform.coeff == -1.0)
        got = permute(t, p)
        dst, expected = oracle_permute(h, x, p)
        assert got.space == dst
        assert np.array_equal(bits(host(got.data)), bits(expected.astype(dtype)))
    plan = twist_plan(h, (0, 2))
    got = twist(t, (0, 2))
    n = len(plan.transform.src)
    expected = so.accumulation(plan.words, x, [x.real.dtype.type(c) for c in plan.transform.coeff], np.arange(n))
    assert np.array_equal(bits(host(got.data)), bits(expected))
    plan = flip_plan(h, (1, 3))
    got = flip(t, (1, 3))
    expected = so.accumulation(plan.words, x, [x.real.dtype.type(c) for c in plan.transform.coeff], np.arange(n))
    assert got.space == h.flip((1, 3))
    assert np.array_equal(bits(host(got.data)), bits(expected))


def test_config_five_chain_scaled():
    """Z2 x Z3 x U(1), complex128, degeneracies uniform in 1..3, q in -1..1."""
    w = z2z3u1(5, range(-1, 2), 3)
    h = hom((w, w, w), (w, w))
    rng = np.random.default_rng(5)
    n = degeneracy_structure(h).total_dim
    x = sample(rng, np.complex128, n)
    t = TensorMap(h, torch.from_numpy(x).cuda())
    p = ((2, 0, 4), (1, 3))
    y = permute(t, p)
    dst, expected = oracle_permute(h, x, p)
    assert np.array_equal(bits(host(y.data)), bits(expected))
    base = sample(rng, np.complex128, degeneracy_structure(dst).total_dim)
    alpha = 0.7 + 0.2j
    z = add_transform(TensorMap(dst, torch.from_numpy(base).cuda()), t, p, alpha, 1.0)
    plan = permute_plan(h, *p)
    expected_z = so.update(plan.words, x, base, np.complex128(alpha), np.float64(1.0))
    assert relative_error(host(z.data), expected_z) <= 1e-12
    output = (((0, 0), (0, 1), (0, 2)), ((1, 0), (1, 1), (1, 2)))
    r = tensorcontract(z, z, axes=((3, 4), (3, 4)), output=output, conjugate=(False, True))
    rs, expected_r = oracle_contract(dst, dst, host(z.data), host(z.data), ((3, 4), (3, 4)), output, (False, True))
    assert r.space == rs
    assert relative_error(host(r.data), expected_r) <= 1e-12


def test_config_five_chain_dense_small():
    w = z2z3u1(7, range(0, 2), 2)
    h = hom((w, w, w), (w, w))
    rng = np.random.default_rng(6)
    x = sample(rng, np.complex128, degeneracy_structure(h).total_dim)
    t = TensorMap(h, torch.from_numpy(x).cuda())
    p = ((2, 0, 4), (1, 3))
    y = permute(t, p)
    base = sample(rng, np.complex128, degeneracy_structure(y.space).total_dim)
    z = add_transform(TensorMap(y.space, torch.from_numpy(base).cuda()), t, p, 0.7 + 0.2j, 1.0)
    dz = (0.7 + 0.2j) * dense.permute(dense.to_dense(h, x), *p) + dense.to_dense(y.space, base)
    assert relative_error(dense.to_dense(z.space, host(z.data)), dz) <= 1e-12
    output = (((0, 0), (0, 1), (0, 2)), ((1, 0), (1, 1), (1, 2)))
    r = tensorcontract(z, z, axes=((3, 4), (3, 4)), output=output, conjugate=(False, True))
    expected = dense.contract(dz, np.conj(dz), (3, 4), (3, 4), output)
    assert relative_error(dense.to_dense(r.space, host(r.data)), expected) <= 1e-12
