"""TensorMap operations of the block-sparse hot path on the B200 engine.

Mirrors the reference's public operations for abelian sector families:

* ``permute`` — operations/transforms.py:32-63 and 165-187: one tree permuter,
  one record per sub-block pair (_stride/_tensor_ops.py:17-87), executed as a
  single accumulation with per-record coefficients and disjoint outputs;
* ``TensorMap.add`` — tensor/tensor_map.py:434-455 (alpha*self + beta*other);
* ``add_transform`` — the fused permute + alpha/beta accumulate: one update
  call with permuted source records (the reference's update_p,
  _stride/_ops.py:66-104, whose ``alpha`` scales the source and ``beta`` the
  destination);
* ``tensortrace`` — operations/contractions/primitives.py:463-588 with
  _tensor_ops.py:206-289: paired traced strides are summed and one reduction
  call evaluates every contribution;
* ``tensorcontract`` — primitives.py:307-430: operand permutes chosen by the
  reference's copy-cost rule (primitives.py:147-234), per-sector GEMMs
  (linalg.py:533-566) and the output permute; conjugated operands are
  prepared in one conjugating pass into their adjoint destination
  (primitives.py:288-304 with transforms.py:190-259), and the right operand's
  dual contracted legs are twisted (primitives.py:422-428) inside its permute;
* ``adjoint`` / ``permute_adjoint`` — tensor_map.py:503-515 and
  transforms.py:190-259: one conjugating accumulation into hom(domain,
  codomain);
* ``twist`` / ``flip`` — transforms.py:275-373: one accumulation with the
  per-sub-block +-1 factors.

Storage is a CUDA tensor ``[*batch, total_dim]``; every operation is computed
by the sm_100a engine.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache
from math import prod

import numpy as np
import torch

from . import stride
from . import _native
from .structure import (AbelianTransform, HomSpace, adjoint_transform, degeneracy_structure, flip_transform, hom,
                        sector_structure, trace_transformer, tree_permuter, twist_factors)

__all__ = ["TensorMap", "random_normal", "permute", "add_transform", "tensortrace", "tensorcontract",
           "adjoint", "permute_adjoint", "twist", "flip", "PermutePlan", "permute_plan", "adjoint_plan",
           "twist_plan", "flip_plan", "trace_plan", "contract_plan"]

_ELEMENT_BYTES = {torch.float32: 4, torch.float64: 8, torch.complex64: 8, torch.complex128: 16}


@dataclass
class TensorMap:
    space: HomSpace
    data: torch.Tensor

    def __post_init__(self):
        total = degeneracy_structure(self.space).total_dim
        if self.data.shape[-1] != total:
            raise ValueError(f"storage has {self.data.shape[-1]} elements; the space needs {total}")

    @property
    def numout(self) -> int:
        return self.space.numout

    @property
    def numin(self) -> int:
        return self.space.numin

    @property
    def numind(self) -> int:
        return self.space.numind

    def blocks(self):
        """(block sector, row_dim x col_dim view) per block (tensor_map.py:256-277)."""
        ds = degeneracy_structure(self.space)
        ss = sector_structure(self.space)
        out = []
        for b in range(len(ds.block_start)):
            start, r, c = int(ds.block_start[b]), int(ds.block_rows[b]), int(ds.block_cols[b])
            out.append((tuple(int(x) for x in ss.blocksectors[b]), self.data[..., start:start + r * c].reshape(
                *self.data.shape[:-1], r, c)))
        return tuple(out)

    def adjoint(self) -> "TensorMap":
        """hom(domain, codomain) with every block conjugate-transposed."""
        return adjoint(self)

    def inner(self, other: "TensorMap") -> torch.Tensor:
        """sum over blocks of vdot(self block, other block) (tensor_map.py:457-473;
        abelian quantum dimensions are 1): one Dot over the whole storage
        with the left side conjugated."""
        if self.space != other.space:
            raise ValueError("TensorMap spaces are not compatible for inner")
        dtype = torch.promote_types(self.data.dtype, other.data.dtype)
        return stride.execute_dot(self.data.to(dtype).contiguous(), other.data.to(dtype).contiguous(),
                                  _storage_dot_plan(self.space, _ELEMENT_BYTES[dtype]), conjugate_left=True)

    def dot(self, other: "TensorMap") -> torch.Tensor:
        return self.inner(other)

    def norm(self) -> torch.Tensor:
        """sqrt(real(inner(self, self))) (tensor_map.py:478-484)."""
        return torch.sqrt(torch.real(self.inner(self)))

    def add(self, other: "TensorMap", alpha=1, beta=1) -> "TensorMap":
        """alpha * self + beta * other (tensor_map.py:434-455)."""
        if self.space != other.space:
            raise ValueError("TensorMap spaces are not compatible for add")
        dtype = _result_dtype(self.data.dtype, other.data.dtype, alpha, beta)
        left = self.data.to(dtype)
        right = other.data.to(dtype)
        return TensorMap(self.space, stride.axpby(alpha, left.contiguous(), beta, right.contiguous()))


_DOT_PLANS: dict = {}


def _storage_dot_plan(space: HomSpace, element_bytes: int) -> stride.Plan:
    """A Dot plan of one contiguous record over a space's whole storage."""
    n = degeneracy_structure(space).total_dim
    key = (n, element_bytes)
    plan = _DOT_PLANS.get(key)
    if plan is None:
        words = stride.encode_layout([stride.AffineRecord((n,), (1,), 0, (1,), 0)], source_size=n, output_size=n)
        plan = stride.Plan(_native.OP_DOT, words, element_bytes=element_bytes)
        _DOT_PLANS[key] = plan
    return plan


def _result_dtype(left: torch.dtype, right: torch.dtype, *scalars) -> torch.dtype:
    dtype = torch.promote_types(left, right)
    if any(isinstance(s, complex) and complex(s).imag != 0 for s in scalars) and not dtype.is_complex:
        dtype = torch.complex128 if dtype == torch.float64 else torch.complex64
    return dtype


def random_normal(space: HomSpace, dtype: torch.dtype, seed: int, *, device="cuda",
                  batch: tuple[int, ...] = ()) -> TensorMap:
    """Seeded N(0, 1) storage in packed order; complex = normal + 1j * normal
    from the same generator."""
    n = degeneracy_structure(space).total_dim
    rng = np.random.default_rng(seed)
    shape = (*batch, n)
    if dtype.is_complex:
        real = rng.standard_normal(shape)
        values = real + 1j * rng.standard_normal(shape)
    else:
        values = rng.standard_normal(shape)
    numpy_dtype = {torch.float32: np.float32, torch.float64: np.float64,
                   torch.complex64: np.complex64, torch.complex128: np.complex128}[dtype]
    return TensorMap(space, torch.from_numpy(values.astype(numpy_dtype)).to(device))


# ---------------------------------------------------------------------------
# Permute.


@dataclass
class PermutePlan:
    """Records of one permute: layout words, coefficients and destination space."""

    src: HomSpace
    dst: HomSpace
    words: np.ndarray
    transform: AbelianTransform
    outputs_disjoint: bool
    shape: np.ndarray
    src_strides: np.ndarray
    src_offsets: np.ndarray
    dst_strides: np.ndarray
    dst_offsets: np.ndarray
    perm: tuple = ()
    conjugate: bool = False
    _plans: dict = None

    @property
    def source_size(self) -> int:
        return degeneracy_structure(self.src).total_dim

    @property
    def output_size(self) -> int:
        return degeneracy_structure(self.dst).total_dim

    def engine_plan(self, operation: int, dtype: torch.dtype) -> stride.Plan:
        key = (operation, _ELEMENT_BYTES[dtype], self.conjugate and dtype.is_complex)
        if self._plans is None:
            self._plans = {}
        plan = self._plans.get(key)
        if plan is None:
            records = np.arange(len(self.transform.src)) if operation == _native.OP_ACCUMULATION else ()
            plan = stride.Plan(operation, self.words, element_bytes=_ELEMENT_BYTES[dtype],
                               coefficient_records=records, outputs_disjoint=self.outputs_disjoint,
                               conjugate_source=self.conjugate and dtype.is_complex)
            self._plans[key] = plan
        return plan


def _affine_plan(src: HomSpace, dst: HomSpace, transform: AbelianTransform, perm: tuple[int, ...],
                 conjugate: bool = False) -> PermutePlan:
    """Affine records of an abelian transform (_tensor_ops.py:17-87), vectorised:
    source sub-block transform.src read along the source axes `perm`, written
    to destination sub-block transform.dst."""
    sd, dd = degeneracy_structure(src), degeneracy_structure(dst)
    perm = list(perm)
    count = len(transform.src)
    shape = sd.sizes[transform.src][:, perm] if perm else np.zeros((count, 0), np.int64)
    sstr = sd.strides[transform.src][:, perm] if perm else np.zeros((count, 0), np.int64)
    if not np.array_equal(shape, dd.sizes[transform.dst]):
        raise ValueError("Abelian tree transform subblock shapes are inconsistent")
    disjoint = np.unique(transform.dst).size == transform.dst.size
    words = stride.encode_layout_arrays(shape, sstr, sd.offsets[transform.src], dd.strides[transform.dst],
                                        dd.offsets[transform.dst], source_size=sd.total_dim,
                                        output_size=dd.total_dim)
    return PermutePlan(src, dst, words, transform, bool(disjoint), shape, sstr, sd.offsets[transform.src],
                       dd.strides[transform.dst], dd.offsets[transform.dst], tuple(perm), conjugate=conjugate)


@lru_cache(maxsize=256)
def permute_plan(src: HomSpace, p_codomain: tuple[int, ...], p_domain: tuple[int, ...]) -> PermutePlan:
    """Tree permuter + affine records (_tensor_ops.py:17-87)."""
    dst, transform = tree_permuter(src, p_codomain, p_domain)
    return _affine_plan(src, dst, transform, tuple(p_codomain + p_domain))


@lru_cache(maxsize=256)
def adjoint_plan(src: HomSpace, p_codomain: tuple[int, ...], p_domain: tuple[int, ...]) -> PermutePlan:
    """The permutation's adjoint destination (transforms.py:190-259): conjugated
    source, destination hom(parent.domain, parent.codomain), coefficients the
    conjugated (real) tree coefficients."""
    dst, transform, axes = adjoint_transform(src, p_codomain, p_domain)
    return _affine_plan(src, dst, transform, axes, conjugate=True)


@lru_cache(maxsize=256)
def twist_plan(src: HomSpace, indices: tuple[int, ...], inv: bool = False) -> PermutePlan | None:
    """Per-sub-block twist factors (transforms.py:275-322), or None when trivial."""
    factors = twist_factors(src, indices, inv)
    if factors is None:
        return None
    n = len(factors)
    transform = AbelianTransform(np.arange(n, dtype=np.int64), np.arange(n, dtype=np.int64), factors)
    return _affine_plan(src, src, transform, tuple(range(src.numind)))


@lru_cache(maxsize=256)
def flip_plan(src: HomSpace, indices: tuple[int, ...], inv: bool = False) -> PermutePlan:
    """Flip of the selected visible legs (transforms.py:325-373)."""
    dst, transform = flip_transform(src, indices, inv)
    return _affine_plan(src, dst, transform, tuple(range(src.numind)))


def _normalize_p(space: HomSpace, p) -> tuple[tuple[int, ...], tuple[int, ...]]:
    p_codomain, p_domain = (tuple(int(i) for i in p[0]), tuple(int(i) for i in p[1]))
    if sorted(p_codomain + p_domain) != list(range(space.numind)):
        raise ValueError("permute() permutation must contain each visible index exactly once")
    return p_codomain, p_domain


def _run(tensor: TensorMap, plan: PermutePlan, coefficients=None) -> TensorMap:
    """One accumulation of the plan's records over the tensor's storage."""
    engine = plan.engine_plan(_native.OP_ACCUMULATION, tensor.data.dtype)
    real = torch.float32 if tensor.data.dtype in (torch.float32, torch.complex64) else torch.float64
    values = plan.transform.coeff if coefficients is None else coefficients
    out = stride.execute_accumulation(tensor.data.contiguous(), engine, _device_constant(values, real, tensor.data.device))
    return TensorMap(plan.dst, out)


def _is_identity_p(space: HomSpace, p_codomain, p_domain) -> bool:
    return tuple(p_codomain) == tuple(range(space.numout)) and tuple(p_domain) == tuple(range(space.numout, space.numind))


def permute(tensor: TensorMap, p) -> TensorMap:
    """permute(t, ((1, 0), (3, 2))) — one accumulation call (transforms.py:32-63)."""
    p_codomain, p_domain = _normalize_p(tensor.space, p)
    if _is_identity_p(tensor.space, p_codomain, p_domain):
        return tensor
    return _run(tensor, permute_plan(tensor.space, p_codomain, p_domain))


def permute_adjoint(tensor: TensorMap, p) -> TensorMap:
    """adjoint(permute(t, p)) in one conjugating accumulation
    (transforms.py:190-259, _permute_to_adjoint_destination)."""
    p_codomain, p_domain = _normalize_p(tensor.space, p)
    return _run(tensor, adjoint_plan(tensor.space, p_codomain, p_domain))


def adjoint(tensor: TensorMap) -> TensorMap:
    """t† in hom(domain, codomain): every block conjugate-transposed
    (tensor/tensor_map.py:503-515)."""
    return permute_adjoint(tensor, (tuple(range(tensor.numout)), tuple(range(tensor.numout, tensor.numind))))


def twist(tensor: TensorMap, indices, inv: bool = False) -> TensorMap:
    """twist(t, indices) (transforms.py:275-322): the selected legs' twists per sub-block."""
    if not isinstance(inv, bool):
        raise TypeError("twist() requires inv to be a bool")
    chosen = (indices,) if isinstance(indices, int) else tuple(int(i) for i in indices)
    plan = twist_plan(tensor.space, chosen, inv)
    return tensor if plan is None else _run(tensor, plan)


def flip(tensor: TensorMap, indices, inv: bool = False) -> TensorMap:
    """flip(t, indices) (transforms.py:325-373)."""
    if not isinstance(inv, bool):
        raise TypeError("flip() requires inv to be a bool")
    chosen = (indices,) if isinstance(indices, int) else tuple(int(i) for i in indices)
    if not chosen:
        return tensor
    return _run(tensor, flip_plan(tensor.space, chosen, inv))


def add_transform(destination: TensorMap, source: TensorMap, p, alpha=1, beta=1, *,
                  inplace: bool = False) -> TensorMap:
    """alpha * permute(source, p) + beta * destination in one fused update call."""
    p_codomain, p_domain = _normalize_p(source.space, p)
    plan = permute_plan(source.space, p_codomain, p_domain)
    if plan.dst != destination.space:
        raise ValueError("destination space does not match the permuted source space")
    engine = plan.engine_plan(_native.OP_UPDATE, destination.data.dtype)
    if source.data.dtype != destination.data.dtype:
        raise ValueError("add_transform operands must share a dtype")
    out = destination.data if inplace else None
    result = stride.execute_update(source.data.contiguous(), destination.data.contiguous(),
                                   _coefficient(alpha, destination.data), _coefficient(beta, destination.data),
                                   engine, out=out)
    return TensorMap(destination.space, result)


_CONSTANTS: dict = {}


def _device_constant(values, dtype: torch.dtype, device) -> torch.Tensor:
    """Device copy of small host constants (coefficient rows), made once per
    value, dtype and device so that repeated calls issue no host copies."""
    array = np.ascontiguousarray(np.asarray(values))
    key = (array.tobytes(), array.shape, str(array.dtype), dtype, str(device))
    tensor = _CONSTANTS.get(key)
    if tensor is None:
        if len(_CONSTANTS) > 4096:
            _CONSTANTS.clear()
        tensor = torch.as_tensor(array).to(dtype=dtype, device=device)
        _CONSTANTS[key] = tensor
    return tensor


def _coefficient(value, storage: torch.Tensor) -> torch.Tensor:
    real = torch.float32 if storage.dtype in (torch.float32, torch.complex64) else torch.float64
    if isinstance(value, complex) and value.imag != 0:
        if not storage.is_complex():
            raise ValueError("complex coefficient on real storage")
        return _device_constant([value], storage.dtype, storage.device)
    return _device_constant([complex(value).real if isinstance(value, complex) else value], real, storage.device)


# ---------------------------------------------------------------------------
# Partial trace.


@dataclass
class TracePlan:
    dst: HomSpace
    words: np.ndarray
    coefficients: np.ndarray
    records: int
    _plans: dict = None

    def engine_plan(self, dtype: torch.dtype) -> stride.Plan:
        key = _ELEMENT_BYTES[dtype]
        if self._plans is None:
            self._plans = {}
        if key not in self._plans:
            self._plans[key] = stride.Plan(_native.OP_REDUCTION, self.words, element_bytes=key,
                                           coefficient_records=np.arange(self.records))
        return self._plans[key]


@lru_cache(maxsize=128)
def trace_plan(space: HomSpace, trace_left: tuple[int, ...], trace_right: tuple[int, ...],
               out_codomain: tuple[int, ...], out_domain: tuple[int, ...]) -> TracePlan:
    """Canonical permute + trace transformer + reduction records
    (primitives.py:463-588, _tensor_ops.py:206-289)."""
    rank = space.numind
    partition = trace_left + trace_right + out_codomain + out_domain
    if sorted(partition) != list(range(rank)) or len(trace_left) != len(trace_right):
        raise ValueError("each original axis must appear exactly once")
    for left, right in zip(trace_left, trace_right):
        if space[left].dual() != space[right]:
            raise ValueError("paired trace axes must be dual-compatible")
    p_codomain = out_codomain + trace_left
    p_domain = out_domain + trace_right
    canonical, basis = tree_permuter(space, p_codomain, p_domain)
    no, ni, tc = len(out_codomain), len(out_domain), len(trace_left)
    dst = HomSpace(canonical.codomain[:no], canonical.domain[:ni])
    transform = trace_transformer(canonical, dst, basis)
    sd, dd = degeneracy_structure(space), degeneracy_structure(dst)
    perm = list(p_codomain + p_domain)
    sizes = sd.sizes[transform.src][:, perm]
    strides = sd.strides[transform.src][:, perm]
    open_axes = list(range(no)) + list(range(no + tc, no + tc + ni))
    shape = sizes[:, open_axes]
    sstr = strides[:, open_axes]
    traced_shape, traced_strides = [], []
    for t in range(tc):
        left, right = no + t, no + tc + ni + t
        if not np.array_equal(sizes[:, left], sizes[:, right]):
            raise ValueError("trace source subblock axes have inconsistent sizes")
        traced_shape.append(sizes[:, left])
        traced_strides.append(strides[:, left] + strides[:, right])
    count = len(transform.src)
    logical = np.concatenate([shape, np.stack(traced_shape, 1) if tc else np.zeros((count, 0), np.int64)], 1)
    src_strides = np.concatenate([sstr, np.stack(traced_strides, 1) if tc else np.zeros((count, 0), np.int64)], 1)
    dst_sizes = dd.sizes[transform.dst]
    if not np.array_equal(shape, dst_sizes):
        raise ValueError("trace destination subblock shape is inconsistent")
    dst_strides = np.concatenate([dd.strides[transform.dst], np.ones((count, tc), np.int64)], 1)
    rank_r = no + ni + tc
    # Reduction protocol words (_descriptor.py:41-76), vectorised.
    body = np.empty((count, 3 + 5 * rank_r), np.int64)
    body[:, 0] = rank_r
    body[:, 1] = sd.offsets[transform.src]
    body[:, 2] = dd.offsets[transform.dst]
    body[:, 3:3 + rank_r] = logical
    body[:, 3 + rank_r:3 + 2 * rank_r] = src_strides
    body[:, 3 + 2 * rank_r:3 + 3 * rank_r] = np.concatenate([dst_sizes, np.ones((count, tc), np.int64)], 1)
    body[:, 3 + 3 * rank_r:3 + 4 * rank_r] = dst_strides
    body[:, 3 + 4 * rank_r:] = np.array([0] * (no + ni) + [1] * tc, np.int64)
    words = np.concatenate([np.array([1, sd.total_dim, dd.total_dim, count], np.int64), body.reshape(-1)])
    return TracePlan(dst, words, transform.coeff, count)


def tensortrace(tensor: TensorMap, *, axes, output) -> TensorMap:
    """tensortrace(t, axes=((1, 2), (4, 5)), output=((0,), (3,)))."""
    left, right = tuple(int(a) for a in axes[0]), tuple(int(a) for a in axes[1])
    out_codomain, out_domain = tuple(int(a) for a in output[0]), tuple(int(a) for a in output[1])
    if not left:
        return permute(tensor, (out_codomain, out_domain))
    plan = trace_plan(tensor.space, left, right, out_codomain, out_domain)
    engine = plan.engine_plan(tensor.data.dtype)
    real = torch.float32 if tensor.data.dtype in (torch.float32, torch.complex64) else torch.float64
    coefficients = _device_constant(plan.coefficients, real, tensor.data.device)
    out = stride.execute_reduction(tensor.data.contiguous(), engine, coefficients)
    return TensorMap(plan.dst, out)


# ---------------------------------------------------------------------------
# Contraction.


@dataclass
class ContractPlan:
    left_p: tuple
    right_p: tuple
    output_p: tuple
    reversed_operands: bool
    canonical: HomSpace
    gemm: stride.GemmPlan
    result: HomSpace
    conjugate: tuple = (False, False)        # per operand, after any reversal
    right_twist: tuple = ()                  # right canonical codomain legs to twist


def _storage_dim(space: HomSpace) -> int:
    return degeneracy_structure(space).total_dim


def _copy_cost(space: HomSpace, p) -> int:
    return 0 if _is_identity_p(space, *p) else _storage_dim(space)


def _compose_spec(left: HomSpace, right: HomSpace, result: HomSpace) -> np.ndarray:
    """Per result block: {m, n, k, a_off, b_off, c_off} (linalg.py:551-566)."""
    ls, rs, res = sector_structure(left), sector_structure(right), sector_structure(result)
    ld, rd, resd = degeneracy_structure(left), degeneracy_structure(right), degeneracy_structure(result)
    lmap = {tuple(s): i for i, s in enumerate(ls.blocksectors.tolist())}
    rmap = {tuple(s): i for i, s in enumerate(rs.blocksectors.tolist())}
    rows = []
    for b, sector in enumerate(res.blocksectors.tolist()):
        m, n = int(resd.block_rows[b]), int(resd.block_cols[b])
        li, ri = lmap.get(tuple(sector)), rmap.get(tuple(sector))
        if li is None or ri is None:
            rows.append((m, n, 0, 0, 0, int(resd.block_start[b])))
            continue
        k = int(ld.block_cols[li])
        rows.append((m, n, k, int(ld.block_start[li]), int(rd.block_start[ri]), int(resd.block_start[b])))
    return np.array(rows, np.int64).reshape(-1, 6)


def _adjoint_axis(space: HomSpace, axis: int) -> int:
    """A visible axis of `space` as an axis of hom(domain, codomain) (primitives.py:141-144)."""
    return space.numin + axis if axis < space.numout else axis - space.numout


# Families with the reference's "symmetric boson" contraction options
# (primitives.py:399-406): reversed operand order and fused adjoint preparation.
_SYMMETRIC_BOSONS = frozenset(("U1Irrep", "Z2Irrep", "Z3Irrep", "Z4Irrep"))


def _symmetric_boson(space: HomSpace) -> bool:
    return space.sector_type.name in _SYMMETRIC_BOSONS


@lru_cache(maxsize=128)
def contract_plan(left: HomSpace, right: HomSpace, left_axes: tuple, right_axes: tuple,
                  output: tuple, conjugate: tuple = (False, False)) -> ContractPlan:
    """Operand permutations, sector GEMM table and result space of one
    contraction (primitives.py:307-430); conjugated operands are seen as their
    adjoints hom(domain, codomain)."""
    ranks = (left.numind, right.numind)
    spaces = tuple(hom(s.domain, s.codomain) if c else s for s, c in zip((left, right), conjugate))

    def mapped(operand, axis):
        return _adjoint_axis((left, right)[operand], axis) if conjugate[operand] else axis

    m_left = tuple(mapped(0, a) for a in left_axes)
    m_right = tuple(mapped(1, a) for a in right_axes)
    for la, ra in zip(m_left, m_right):
        if spaces[0][la].dual() != spaces[1][ra]:
            raise ValueError("contracted axes must be dual-compatible")
    open_left = tuple(a for a in range(ranks[0]) if a not in left_axes)
    open_right = tuple(a for a in range(ranks[1]) if a not in right_axes)
    m_open_left = tuple(mapped(0, a) for a in open_left)
    m_open_right = tuple(mapped(1, a) for a in open_right)
    canonical_refs = tuple((0, a) for a in open_left) + tuple((1, a) for a in open_right)
    position = {ref: i for i, ref in enumerate(canonical_refs)}
    output_p = (tuple(position[r] for r in output[0]), tuple(position[r] for r in output[1]))
    symmetric_boson = _symmetric_boson(spaces[0])

    def candidate(sort_position, reversed_operands):
        pairs = sorted(zip(m_left, m_right), key=lambda pair: pair[sort_position])
        lc, rc = tuple(p[0] for p in pairs), tuple(p[1] for p in pairs)
        if reversed_operands:
            lp, rp = (m_open_right, rc), (lc, m_open_left)
            ls, rs = spaces[1], spaces[0]
            nl, nr = len(m_open_left), len(m_open_right)
            op = tuple(tuple(a + nr if a < nl else a - nl for a in part) for part in output_p)
        else:
            lp, rp = (m_open_left, lc), (rc, m_open_right)
            ls, rs = spaces
            op = output_p
        cost = _copy_cost(ls, lp) + _copy_cost(rs, rp)
        canonical = HomSpace(ls.permute(*lp).codomain, rs.permute(*rp).domain)
        cost += _copy_cost(canonical, op)
        return cost, lp, rp, op, reversed_operands, canonical, ls, rs

    options = [candidate(s, r) for r in ((False, True) if symmetric_boson else (False,))
               for s in ((0, 1) if len(left_axes) > 1 else (0,))]
    cost, lp, rp, op, rev, canonical, ls, rs = min(options, key=lambda c: c[0])
    lspace, rspace = ls.permute(*lp), rs.permute(*rp)
    spec = _compose_spec(lspace, rspace, canonical)
    result = canonical.permute(*op)
    flags = tuple(conjugate[::-1]) if rev else tuple(conjugate)
    right_twist = tuple(a for a in range(len(rp[0])) if rspace[a].is_dual) if not rspace.sector_type.bosonic else ()
    return ContractPlan(lp, rp, op, rev, canonical, stride.GemmPlan(spec), result, flags, right_twist)


def _prepare_operand(value: TensorMap, permutation: tuple, conjugate: bool) -> TensorMap:
    """The canonical operand (primitives.py:288-304): a permute, or for a
    conjugated operand the permuted adjoint, computed in one conjugating pass
    into the adjoint destination (exact, so equal to the reference's
    adjoint-then-permute for the families without its fused path)."""
    if not conjugate:
        return permute(value, permutation)
    adjoint_space = hom(value.space.domain, value.space.codomain)
    parent = (tuple(_adjoint_axis(adjoint_space, a) for a in permutation[1]),
              tuple(_adjoint_axis(adjoint_space, a) for a in permutation[0]))
    return permute_adjoint(value, parent)


def tensorcontract(left: TensorMap, right: TensorMap, *, axes, output,
                   conjugate: tuple[bool, bool] = (False, False)) -> TensorMap:
    """tensorcontract(A, B, axes=((2,), (0,)), output=(((0, 0), (1, 1)), ((0, 1),)),
    conjugate=(False, True)) (primitives.py:307-430)."""
    left_axes, right_axes = tuple(int(a) for a in axes[0]), tuple(int(a) for a in axes[1])
    output = (tuple((int(o), int(a)) for o, a in output[0]), tuple((int(o), int(a)) for o, a in output[1]))
    flags = (bool(conjugate[0]), bool(conjugate[1]))
    plan = contract_plan(left.space, right.space, left_axes, right_axes, output, flags)
    if plan.reversed_operands:
        left, right = right, left
    lcan = _prepare_operand(left, plan.left_p, plan.conjugate[0])
    rcan = _prepare_operand(right, plan.right_p, plan.conjugate[1])
    if plan.right_twist:
        rcan = twist(rcan, plan.right_twist)
    dtype = torch.promote_types(lcan.data.dtype, rcan.data.dtype)
    out = torch.empty(_storage_dim(plan.canonical), dtype=dtype, device=lcan.data.device)
    stride.sector_gemm(plan.gemm, lcan.data.to(dtype).contiguous(), rcan.data.to(dtype).contiguous(), out)
    result = TensorMap(plan.canonical, out)
    return permute(result, plan.output_p)
