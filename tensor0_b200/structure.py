"""Abelian sector structures, packed layouts and tree transformers.

Host-side planner for the block-sparse stride path, restating the reference's
Rust metadata planner for UniqueFusion sector families (Rust is not part of
this build; the planner is vectorised over numpy arrays so million-sub-block
spaces plan in seconds):

* sectors and their canonical order — crates/tensor0-core/src/sector/
  u1.rs:98-130 (U1 order 0, 1, -1, 2, -2, ...), zn.rs:100-106,
  fermion_parity.rs:90-96, product.rs:265-268 and 403-411 (product order:
  sum of component indices, then the indices);
* graded spaces — space/graded.rs:40-60 (sectors stored sorted, zero
  degeneracies dropped) and 100-125 (visible sectors of a dual space are the
  duals of the stored ones, in stored order);
* fusion-tree order — space/product.rs:229-320: the last factor varies
  slowest and the first factor's sector is fixed by the coupled sector;
* block sectors — layout/sector_structure.rs:199-232 and space/product.rs:202-227;
* the packed layout — layout/degeneracy.rs:54-183: blocks in block-sector
  order, each a row-major row_dim x col_dim matrix; sub-block (row tree,
  column tree) has sizes = row leg dims ++ column leg dims, column strides
  row-major with innermost 1, row strides scaled by col_dim, offset = block
  start + row_offset * col_dim + col_offset;
* HomSpace.permute — space/hom.rs:202-231 (legs moving sides are dualised);
* abelian tree braiding — transform/tree_transformers.rs:216-242 with
  fusion_tree/braiding_ops.rs:18-46 and 129-189: a pair maps to the pair with
  the permuted uncoupled sectors.  The coefficient is the product of
  R-symbols over the inversions of the linearized permutation
  (fusion_tree/auxiliary.rs:82-141: codomain legs, then the domain legs in
  reverse); the repartition factors (duality_ops.rs:23-50, 372-382) are 1 for
  these families, whose F-, B-symbols and Frobenius-Schur phases are 1.  R is
  -1 exactly when both sectors have odd fermion parity
  (sector/fermion_parity.rs:79-88), so bosonic families have coefficient 1;
* twist factors — transform/reweighting.rs:60-99 (product of the twists of
  the selected legs' uncoupled sectors, theta = -1 for odd parity);
* flip — space/graded.rs:89-100, space/hom.rs:156-200 and
  fusion_tree/braiding_ops.rs:84-127;
* trace transformer — transform/trace_transformers.rs:57-84 and 214-246,
  with the coefficient of trace_coefficient (the twists of the non-dual
  traced legs; the tail tree's first sector is the open head's coupled one).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from functools import cached_property
from math import prod

import numpy as np

__all__ = [
    "SectorType", "U1Irrep", "Z2Irrep", "Z3Irrep", "Z4Irrep", "ZNIrrep", "FermionParity",
    "ProductSector", "GradedSpace", "HomSpace", "space", "hom", "SectorStructure",
    "DegeneracyStructure", "sector_structure", "degeneracy_structure", "tree_permuter",
    "trace_transformer", "AbelianTransform", "twist_factors", "flip_transform", "adjoint_transform",
]


# ---------------------------------------------------------------------------
# Sector families.


@dataclass(frozen=True)
class SectorType:
    """An abelian (UniqueFusion) sector family: a product of U1 / Zn / fermion parity.

    A sector value is a tuple of ints, one per component: twice the charge for
    U1 (so half-integer charges are representable, as in the reference's
    ``U1Irrep::charge2``), the residue for Zn, the parity for fermion parity.
    """

    components: tuple[tuple[str, int], ...]
    name: str = ""

    @property
    def width(self) -> int:
        return len(self.components)

    @property
    def bosonic(self) -> bool:
        return all(kind != "FP" for kind, _ in self.components)

    def unit(self) -> tuple[int, ...]:
        return (0,) * self.width

    def normalize(self, value) -> tuple[int, ...]:
        """User sector (int, half-int or tuple of those) -> internal tuple."""
        parts = value if isinstance(value, tuple) else (value,)
        if len(parts) != self.width:
            raise ValueError(f"{self.name} sectors have {self.width} components")
        out = []
        for (kind, n), part in zip(self.components, parts):
            if kind == "U1":
                twice = part * 2
                if twice != int(twice):
                    raise ValueError("U1 charges must be integers or half-integers")
                out.append(int(twice))
            elif kind == "Z":
                out.append(int(part) % n)
            else:
                out.append(int(part) % 2)
        return tuple(out)

    def display(self, sector: tuple[int, ...]):
        parts = []
        for (kind, _), value in zip(self.components, sector):
            parts.append(value // 2 if kind == "U1" and value % 2 == 0 else (value / 2 if kind == "U1" else value))
        return parts[0] if self.width == 1 else tuple(parts)

    # Vectorised group operations on arrays [..., width].
    def fuse(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        out = np.asarray(a, dtype=np.int64) + np.asarray(b, dtype=np.int64)
        return self._reduce(out)

    def dual(self, a: np.ndarray) -> np.ndarray:
        return self._reduce(-np.asarray(a, dtype=np.int64))

    def _reduce(self, values: np.ndarray) -> np.ndarray:
        values = values.copy()
        for c, (kind, n) in enumerate(self.components):
            if kind == "Z":
                values[..., c] %= n
            elif kind == "FP":
                values[..., c] %= 2
        return values

    def parity(self, a: np.ndarray) -> np.ndarray:
        """Per fermion-parity component, whether the sector is odd: [..., n_fp] bools."""
        a = np.asarray(a, dtype=np.int64)
        columns = [c for c, (kind, _) in enumerate(self.components) if kind == "FP"]
        if not columns:
            return np.zeros((*a.shape[:-1], 0), bool)
        return (a[..., columns] % 2) == 1

    def twist(self, a: np.ndarray) -> np.ndarray:
        """Sector twists theta (product over components; -1 for odd parity)."""
        odd = self.parity(a)
        return np.where(odd.sum(axis=-1) % 2 == 1, -1.0, 1.0)

    def sort_index(self, a: np.ndarray) -> np.ndarray:
        """Per-component canonical indices (u1.rs:123-130; zn / parity: value)."""
        a = np.asarray(a, dtype=np.int64)
        out = a.copy()
        for c, (kind, _) in enumerate(self.components):
            if kind == "U1":
                v = a[..., c]
                out[..., c] = np.where(v > 0, 2 * v - 1, -2 * v)
        return out

    def sort_keys(self, a: np.ndarray) -> np.ndarray:
        """Lexicographic sort keys [..., k]: product families prepend the index sum."""
        idx = self.sort_index(a)
        if self.width == 1:
            return idx
        return np.concatenate([idx.sum(axis=-1, keepdims=True), idx], axis=-1)

    def order(self, a: np.ndarray) -> np.ndarray:
        """Stable argsort of sectors [n, width] in canonical order."""
        keys = self.sort_keys(np.asarray(a, dtype=np.int64).reshape(-1, self.width))
        return np.lexsort(keys.T[::-1], axis=0) if len(keys) else np.zeros(0, dtype=np.int64)


U1Irrep = SectorType((("U1", 0),), "U1Irrep")
Z2Irrep = SectorType((("Z", 2),), "Z2Irrep")
Z3Irrep = SectorType((("Z", 3),), "Z3Irrep")
Z4Irrep = SectorType((("Z", 4),), "Z4Irrep")
FermionParity = SectorType((("FP", 2),), "FermionParity")


def ZNIrrep(n: int) -> SectorType:
    return SectorType((("Z", n),), f"Z{n}Irrep")


def ProductSector(*families: SectorType) -> SectorType:
    components = tuple(c for family in families for c in family.components)
    return SectorType(components, "×".join(f.name for f in families))


# ---------------------------------------------------------------------------
# Spaces.


@dataclass(frozen=True)
class GradedSpace:
    """Graded vector space: stored sectors (canonical order) with degeneracies."""

    sector_type: SectorType
    stored: tuple[tuple[int, ...], ...]
    dims: tuple[int, ...]
    is_dual: bool = False

    @staticmethod
    def from_dict(sector_type: SectorType, sector_dims, dual: bool = False) -> "GradedSpace":
        items = [(sector_type.normalize(s), int(d)) for s, d in dict(sector_dims).items() if int(d) != 0]
        if any(d < 0 for _, d in items):
            raise ValueError("degeneracies must be nonnegative")
        sectors = np.array([s for s, _ in items], dtype=np.int64).reshape(-1, sector_type.width)
        order = sector_type.order(sectors)
        stored = tuple(tuple(int(v) for v in sectors[i]) for i in order)
        if len(set(stored)) != len(stored):
            raise ValueError("sector appears multiple times")
        dims = tuple(items[i][1] for i in order)
        return GradedSpace(sector_type, stored, dims, dual)

    def dual(self) -> "GradedSpace":
        return GradedSpace(self.sector_type, self.stored, self.dims, not self.is_dual)

    def flip(self) -> "GradedSpace":
        """Stored sectors dualised and re-sorted, duality toggled: the visible
        sectors stay the same (space/graded.rs:89-100)."""
        st = self.sector_type
        if not self.stored:
            return GradedSpace(st, self.stored, self.dims, not self.is_dual)
        duals = st.dual(np.array(self.stored, dtype=np.int64).reshape(-1, st.width))
        order = st.order(duals)
        return GradedSpace(st, tuple(tuple(int(v) for v in duals[i]) for i in order),
                           tuple(self.dims[i] for i in order), not self.is_dual)

    @cached_property
    def visible(self) -> np.ndarray:
        stored = np.array(self.stored, dtype=np.int64).reshape(-1, self.sector_type.width)
        return self.sector_type.dual(stored) if self.is_dual else stored

    @cached_property
    def dim_array(self) -> np.ndarray:
        return np.array(self.dims, dtype=np.int64)

    @property
    def dim(self) -> int:
        return int(sum(self.dims))

    @cached_property
    def offsets(self) -> np.ndarray:
        """Dense index offset of each stored sector (sectors in stored order)."""
        return np.concatenate([[0], np.cumsum(self.dim_array)[:-1]]).astype(np.int64) if self.dims else np.zeros(0, np.int64)


def space(sector_type: SectorType, sector_dims, *, dual: bool = False) -> GradedSpace:
    """``space(U1Irrep, {-1: 2, 0: 3, 1: 2})`` (structure/spaces.py:69-78)."""
    return GradedSpace.from_dict(sector_type, sector_dims, dual)


@dataclass(frozen=True)
class HomSpace:
    codomain: tuple[GradedSpace, ...]
    domain: tuple[GradedSpace, ...]

    def __post_init__(self):
        types = {leg.sector_type for leg in (*self.codomain, *self.domain)}
        if len(types) > 1:
            raise ValueError("all legs of a HomSpace must use the same sector family")

    @property
    def sector_type(self) -> SectorType:
        legs = (*self.codomain, *self.domain)
        return legs[0].sector_type if legs else U1Irrep

    @property
    def numout(self) -> int:
        return len(self.codomain)

    @property
    def numin(self) -> int:
        return len(self.domain)

    @property
    def numind(self) -> int:
        return self.numout + self.numin

    def __getitem__(self, index: int) -> GradedSpace:
        """Visible leg (hom.rs:68-82): domain legs are seen dualised."""
        if index < self.numout:
            return self.codomain[index]
        return self.domain[index - self.numout].dual()

    def permute(self, p_codomain, p_domain) -> "HomSpace":
        p_codomain, p_domain = tuple(p_codomain), tuple(p_domain)
        if sorted(p_codomain + p_domain) != list(range(self.numind)):
            raise ValueError("transform permutation must contain each visible index exactly once")

        def leg(index: int, to_domain: bool) -> GradedSpace:
            if index < self.numout:
                factor = self.codomain[index]
                return factor.dual() if to_domain else factor
            factor = self.domain[index - self.numout]
            return factor if to_domain else factor.dual()

        return HomSpace(tuple(leg(i, False) for i in p_codomain), tuple(leg(i, True) for i in p_domain))

    @property
    def dims(self) -> tuple[int, ...]:
        return tuple(leg.dim for leg in (*self.codomain, *self.domain))

    def flip(self, indices) -> "HomSpace":
        """The selected visible legs flipped (space/hom.rs:156-200)."""
        chosen = set(_normalize_indices(indices, self.numind, "flip"))
        codomain = tuple(leg.flip() if i in chosen else leg for i, leg in enumerate(self.codomain))
        domain = tuple(leg.flip() if self.numout + j in chosen else leg for j, leg in enumerate(self.domain))
        return HomSpace(codomain, domain)


def _normalize_indices(indices, rank: int, what: str) -> tuple[int, ...]:
    values = (indices,) if isinstance(indices, int) else tuple(indices)
    out = []
    for index in values:
        index = int(index)
        if not 0 <= index < rank:
            raise ValueError(f"{what} visible index {index} is out of range for rank {rank}")
        if index in out:
            raise ValueError(f"{what} visible indices must be unique")
        out.append(index)
    return tuple(out)


def hom(codomain, domain) -> HomSpace:
    """``hom((v, v), (v, v))`` — a morphism space codomain <- domain."""
    def as_tuple(value):
        if isinstance(value, GradedSpace):
            return (value,)
        return tuple(value)
    return HomSpace(as_tuple(codomain), as_tuple(domain))


# ---------------------------------------------------------------------------
# Fusion trees and sector structures.


def _trees(sector_type: SectorType, legs: tuple[GradedSpace, ...]):
    """All fusion trees of a product space: (leg sector indices [T, k], coupled [T, width]).

    Rows are ordered as the reference enumerates them for each coupled sector:
    the last leg varies slowest, the first leg's sector is determined.
    """
    width = sector_type.width
    k = len(legs)
    if k == 0:
        return np.zeros((1, 0), np.int64), np.zeros((1, width), np.int64)
    counts = [len(leg.stored) for leg in legs]
    if 0 in counts:
        return np.zeros((0, k), np.int64), np.zeros((0, width), np.int64)
    # C order over (leg k-1, ..., leg 0): the first leg varies fastest.
    grids = np.indices(tuple(reversed(counts))).reshape(k, -1)[::-1].T  # [T, k], column i = leg i
    coupled = np.zeros((grids.shape[0], width), np.int64)
    for i, leg in enumerate(legs):
        coupled = sector_type.fuse(coupled, leg.visible[grids[:, i]])
    return grids.astype(np.int64), coupled


def _encode(sectors: np.ndarray, sector_type: SectorType) -> np.ndarray:
    """Map sector rows to int64 ids preserving identity (not order)."""
    sectors = np.asarray(sectors, np.int64).reshape(-1, sector_type.width)
    if sectors.shape[0] == 0:
        return np.zeros(0, np.int64)
    shifted = sectors - sectors.min(axis=0)
    span = shifted.max(axis=0) + 1
    ids = np.zeros(sectors.shape[0], np.int64)
    for c in range(sector_type.width):
        ids = ids * int(span[c]) + shifted[:, c]
    return ids


@dataclass
class SectorStructure:
    """Block sectors and fusion-tree pairs (layout/sector_structure.rs:128-171)."""

    blocksectors: np.ndarray          # [B, width] canonical order
    pair_block: np.ndarray            # [P] block index of each pair
    pair_row: np.ndarray              # [P, numout] leg sector indices of the row tree
    pair_col: np.ndarray              # [P, numin] leg sector indices of the column tree
    row_trees: list = field(default_factory=list)    # per block: [R, numout]
    col_trees: list = field(default_factory=list)    # per block: [C, numin]

    @property
    def pair_count(self) -> int:
        return int(self.pair_block.shape[0])


_STRUCTURE_CACHE: dict = {}


def _space_key(space: HomSpace):
    return (tuple((leg.stored, leg.dims, leg.is_dual) for leg in space.codomain),
            tuple((leg.stored, leg.dims, leg.is_dual) for leg in space.domain),
            space.sector_type)


def sector_structure(space: HomSpace) -> SectorStructure:
    key = ("sectors", _space_key(space))
    if key in _STRUCTURE_CACHE:
        return _STRUCTURE_CACHE[key]
    st = space.sector_type
    width = st.width
    if space.numout == 0 and space.numin == 0:
        result = SectorStructure(np.zeros((1, width), np.int64), np.zeros(1, np.int64),
                                 np.zeros((1, 0), np.int64), np.zeros((1, 0), np.int64),
                                 [np.zeros((1, 0), np.int64)], [np.zeros((1, 0), np.int64)])
        _STRUCTURE_CACHE[key] = result
        return result
    rows, row_coupled = _trees(st, space.codomain)
    cols, col_coupled = _trees(st, space.domain)
    row_ids, col_ids = _encode(row_coupled, st), _encode(col_coupled, st)
    # Block sectors: coupled sectors reachable on both sides, in canonical order.
    both = np.concatenate([row_coupled, col_coupled]) if len(row_coupled) + len(col_coupled) else np.zeros((0, width), np.int64)
    all_ids = _encode(both, st)
    common = np.intersect1d(all_ids[: len(row_coupled)], all_ids[len(row_coupled):])
    row_ids = all_ids[: len(row_coupled)]
    col_ids = all_ids[len(row_coupled):]
    if common.size:
        first = {int(i): j for j, i in reversed(list(enumerate(all_ids)))}
        sectors = np.array([both[first[int(i)]] for i in common], np.int64).reshape(-1, width)
        order = st.order(sectors)
        blocksectors = sectors[order]
        block_ids = common[order]
    else:
        blocksectors = np.zeros((0, width), np.int64)
        block_ids = np.zeros(0, np.int64)
    row_trees, col_trees, pair_block, pair_row, pair_col = [], [], [], [], []
    for b, bid in enumerate(block_ids):
        r = rows[row_ids == bid]
        c = cols[col_ids == bid]
        row_trees.append(r)
        col_trees.append(c)
        pair_block.append(np.full(len(r) * len(c), b, np.int64))
        pair_row.append(np.repeat(r, len(c), axis=0))
        pair_col.append(np.tile(c, (len(r), 1)))
    result = SectorStructure(
        blocksectors,
        np.concatenate(pair_block) if pair_block else np.zeros(0, np.int64),
        np.concatenate(pair_row) if pair_row else np.zeros((0, space.numout), np.int64),
        np.concatenate(pair_col) if pair_col else np.zeros((0, space.numin), np.int64),
        row_trees, col_trees)
    _STRUCTURE_CACHE[key] = result
    return result


@dataclass
class DegeneracyStructure:
    """Packed layout (layout/degeneracy.rs:8-28)."""

    total_dim: int
    block_rows: np.ndarray     # [B] row_dim
    block_cols: np.ndarray     # [B] col_dim
    block_start: np.ndarray    # [B]
    sizes: np.ndarray          # [P, rank]
    strides: np.ndarray        # [P, rank]
    offsets: np.ndarray        # [P]

    @property
    def block_stop(self) -> np.ndarray:
        return self.block_start + self.block_rows * self.block_cols


def _row_major(dims: np.ndarray) -> np.ndarray:
    """Row-major strides of each row of dims [T, k] (innermost 1)."""
    strides = np.ones_like(dims)
    for i in range(dims.shape[1] - 2, -1, -1):
        strides[:, i] = strides[:, i + 1] * dims[:, i + 1]
    return strides


def degeneracy_structure(space: HomSpace) -> DegeneracyStructure:
    key = ("degeneracy", _space_key(space))
    if key in _STRUCTURE_CACHE:
        return _STRUCTURE_CACHE[key]
    ss = sector_structure(space)
    rank = space.numind
    cod_dims = [leg.dim_array for leg in space.codomain]
    dom_dims = [leg.dim_array for leg in space.domain]
    sizes, strides, offsets = [], [], []
    rows_out, cols_out, starts = [], [], []
    start = 0
    for r, c in zip(ss.row_trees, ss.col_trees):
        rd = np.stack([cod_dims[i][r[:, i]] for i in range(space.numout)], axis=1) if space.numout else np.ones((len(r), 0), np.int64)
        cd = np.stack([dom_dims[j][c[:, j]] for j in range(space.numin)], axis=1) if space.numin else np.ones((len(c), 0), np.int64)
        row_size = rd.prod(axis=1) if rd.shape[1] else np.ones(len(r), np.int64)
        col_size = cd.prod(axis=1) if cd.shape[1] else np.ones(len(c), np.int64)
        row_dim, col_dim = int(row_size.sum()), int(col_size.sum())
        row_off = np.concatenate([[0], np.cumsum(row_size)[:-1]]).astype(np.int64)
        col_off = np.concatenate([[0], np.cumsum(col_size)[:-1]]).astype(np.int64)
        nr, nc = len(r), len(c)
        offsets.append(start + (row_off[:, None] * col_dim + col_off[None, :]).reshape(-1))
        s = np.empty((nr, nc, rank), np.int64)
        z = np.empty((nr, nc, rank), np.int64)
        if space.numout:
            s[:, :, : space.numout] = rd[:, None, :]
            z[:, :, : space.numout] = (_row_major(rd) * col_dim)[:, None, :]
        if space.numin:
            s[:, :, space.numout:] = cd[None, :, :]
            z[:, :, space.numout:] = _row_major(cd)[None, :, :]
        sizes.append(s.reshape(nr * nc, rank))
        strides.append(z.reshape(nr * nc, rank))
        rows_out.append(row_dim)
        cols_out.append(col_dim)
        starts.append(start)
        start += row_dim * col_dim
    result = DegeneracyStructure(
        start, np.array(rows_out, np.int64), np.array(cols_out, np.int64), np.array(starts, np.int64),
        np.concatenate(sizes) if sizes else np.zeros((0, rank), np.int64),
        np.concatenate(strides) if strides else np.zeros((0, rank), np.int64),
        np.concatenate(offsets) if offsets else np.zeros(0, np.int64))
    _STRUCTURE_CACHE[key] = result
    return result


# ---------------------------------------------------------------------------
# Tree transformers.


@dataclass
class AbelianTransform:
    """(src, dst, coeff) per sub-block pair (tree_transformers.rs:18-40)."""

    src: np.ndarray
    dst: np.ndarray
    coeff: np.ndarray

    @property
    def has_only_unit_coefficients(self) -> bool:
        return bool(np.all(self.coeff == 1.0))


def _pair_keys(rows: np.ndarray, cols: np.ndarray, counts: list[int]) -> np.ndarray:
    legs = np.concatenate([rows, cols], axis=1) if rows.size or cols.size else np.zeros((len(rows), 0), np.int64)
    keys = np.zeros(legs.shape[0], np.int64)
    for i, n in enumerate(counts):
        keys = keys * max(n, 1) + legs[:, i]
    return keys


def _lookup(dst: HomSpace, rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    ss = sector_structure(dst)
    counts = [len(leg.stored) for leg in (*dst.codomain, *dst.domain)]
    table = _pair_keys(ss.pair_row, ss.pair_col, counts)
    order = np.argsort(table, kind="stable")
    wanted = _pair_keys(rows, cols, counts)
    pos = np.searchsorted(table[order], wanted)
    pos = np.minimum(pos, max(len(order) - 1, 0))
    found = order[pos] if len(order) else np.zeros(len(wanted), np.int64)
    if len(wanted) and (len(order) == 0 or np.any(table[found] != wanted)):
        raise ValueError("transform destination fusion tree pair was not found")
    return found


def _pair_sectors(space: HomSpace, ss: SectorStructure) -> np.ndarray:
    """Uncoupled (visible) sectors of every pair: [P, numind, width], codomain
    legs then domain legs."""
    legs = (*space.codomain, *space.domain)
    width = space.sector_type.width
    indices = np.concatenate([ss.pair_row, ss.pair_col], axis=1)
    if not legs:
        return np.zeros((ss.pair_count, 0, width), np.int64)
    return np.stack([leg.visible[indices[:, i]] for i, leg in enumerate(legs)], axis=1)


def _braid_signs(space: HomSpace, ss: SectorStructure, p_codomain, p_domain) -> np.ndarray:
    """Product of R-symbols over the inversions of the linearized permutation
    (braiding_ops.rs:129-189): -1 per inverted pair of legs whose sectors are
    both odd in a fermion-parity component."""
    n1, n2 = space.numout, space.numin
    count = ss.pair_count
    if space.sector_type.bosonic:
        return np.ones(count, np.float64)

    def linear(index: int) -> int:
        return index if index < n1 else n1 + n2 - 1 - (index - n1)

    permutation = [linear(i) for i in (*p_codomain, *reversed(p_domain))]
    # The full outgoing tree lists the codomain legs, then the domain legs in reverse.
    visible = _pair_sectors(space, ss)
    order = list(range(n1)) + [n1 + n2 - 1 - k for k in range(n2)]
    odd = space.sector_type.parity(visible[:, order, :]) if count else np.zeros((0, n1 + n2, 0), bool)
    flips = np.zeros(count, np.int64)
    for i in range(len(permutation)):
        for j in range(i):
            if permutation[j] > permutation[i]:
                both = odd[:, permutation[j], :] & odd[:, permutation[i], :]
                flips += both.sum(axis=1)
    return np.where(flips % 2 == 1, -1.0, 1.0)


def tree_permuter(src: HomSpace, p_codomain, p_domain) -> tuple[HomSpace, AbelianTransform]:
    """Abelian tree permuter (tree_transformers.rs:95-173 via braid_pair).

    The destination pair of a source pair carries the same per-leg sector
    positions, permuted (a leg moving sides keeps its position in the dualised
    space's visible list).  The coefficient is +-1: the fermionic braid sign.
    """
    p_codomain, p_domain = tuple(p_codomain), tuple(p_domain)
    dst = src.permute(p_codomain, p_domain)
    ss = sector_structure(src)
    legs = np.concatenate([ss.pair_row, ss.pair_col], axis=1)
    rows = legs[:, list(p_codomain)] if p_codomain else np.zeros((len(legs), 0), np.int64)
    cols = legs[:, list(p_domain)] if p_domain else np.zeros((len(legs), 0), np.int64)
    dst_index = _lookup(dst, rows, cols)
    n = ss.pair_count
    return dst, AbelianTransform(np.arange(n, dtype=np.int64), dst_index,
                                 _braid_signs(src, ss, p_codomain, p_domain))


def twist_factors(space: HomSpace, indices, inv: bool = False) -> np.ndarray | None:
    """Per-pair twist factors for the selected visible legs, or None when all
    are 1 (reweighting.rs:60-99).  Abelian twists are +-1, their own inverse."""
    chosen = _normalize_indices(indices, space.numind, "twist")
    del inv
    if not chosen or space.sector_type.bosonic:
        return None
    ss = sector_structure(space)
    visible = _pair_sectors(space, ss)
    factors = np.ones(ss.pair_count, np.float64)
    for index in chosen:
        factors *= space.sector_type.twist(visible[:, index, :])
    return None if np.all(factors == 1.0) else factors


def flip_transform(src: HomSpace, indices, inv: bool = False) -> tuple[HomSpace, AbelianTransform]:
    """Flip the selected visible legs (braiding_ops.rs:84-127): every pair maps
    to the pair with the same visible sectors in the flipped space; a codomain
    leg contributes theta when its duality differs from `inv`, a domain leg when
    it equals `inv` (the Frobenius-Schur phases are 1 for these families)."""
    chosen = _normalize_indices(indices, src.numind, "flip")
    dst = src.flip(chosen)
    ss = sector_structure(src)
    legs_src = (*src.codomain, *src.domain)
    legs_dst = (*dst.codomain, *dst.domain)
    indices_src = np.concatenate([ss.pair_row, ss.pair_col], axis=1)
    mapped = indices_src.copy()
    visible = _pair_sectors(src, ss)
    factors = np.ones(ss.pair_count, np.float64)
    st = src.sector_type
    for index in chosen:
        # Position of the same visible sector in the flipped leg's stored order.
        target = {tuple(int(v) for v in sector): k for k, sector in enumerate(legs_dst[index].visible)}
        mapped[:, index] = [target[tuple(int(v) for v in sector)] for sector in legs_src[index].visible[indices_src[:, index]]]
        was_dual = legs_src[index].is_dual
        applies = (was_dual != inv) if index < src.numout else (was_dual == inv)
        if applies:
            factors *= st.twist(visible[:, index, :])
    dst_index = _lookup(dst, mapped[:, :src.numout], mapped[:, src.numout:])
    return dst, AbelianTransform(np.arange(ss.pair_count, dtype=np.int64), dst_index, factors)


def adjoint_transform(src: HomSpace, p_codomain, p_domain) -> tuple[HomSpace, AbelianTransform, tuple[int, ...]]:
    """The adjoint destination of a permutation (operations/transforms.py:190-259):
    the parent space permute(src, p), the destination hom(parent.domain,
    parent.codomain), and every source pair sent to the swapped parent pair.
    Returns the destination, the transform (coefficients of the permutation,
    real, so equal to their conjugates) and the source axis order of the
    destination's legs."""
    parent, transform = tree_permuter(src, p_codomain, p_domain)
    dst = HomSpace(parent.domain, parent.codomain)
    ps = sector_structure(parent)
    rows = ps.pair_col[transform.dst]
    cols = ps.pair_row[transform.dst]
    dst_index = _lookup(dst, rows, cols)
    axes = tuple(p_codomain) + tuple(p_domain)
    axes = axes[len(p_codomain):] + axes[:len(p_codomain)]
    return dst, AbelianTransform(transform.src, dst_index, transform.coeff), axes


def trace_transformer(canonical: HomSpace, dst: HomSpace, basis: AbelianTransform) -> AbelianTransform:
    """Abelian trace transformer (trace_transformers.rs:57-84, 214-246).

    A canonical pair contributes when its row and column trees agree on the
    traced tail: equal sectors on every traced leg and an equal coupled sector
    of the open heads.  The destination pair is (row head, column head); the
    bosonic coefficient is 1.
    """
    st = canonical.sector_type
    ss = sector_structure(canonical)
    no, ni = dst.numout, dst.numin
    rows = ss.pair_row[basis.dst]
    cols = ss.pair_col[basis.dst]
    head_r, tail_r = rows[:, :no], rows[:, no:]
    head_c, tail_c = cols[:, :ni], cols[:, ni:]
    keep = np.all(tail_r == tail_c, axis=1)

    def coupled(legs, idx):
        out = np.zeros((idx.shape[0], st.width), np.int64)
        for i, leg in enumerate(legs):
            out = st.fuse(out, leg.visible[idx[:, i]])
        return out

    cr = coupled(canonical.codomain[:no], head_r)
    cc = coupled(canonical.domain[:ni], head_c)
    keep &= np.all(cr == cc, axis=1)
    dst_index = _lookup(dst, head_r[keep], head_c[keep])
    coefficient = basis.coeff[keep].copy()
    # trace_coefficient: the tail tree (split, basic_ops) starts with the open
    # head's coupled sector, then the traced legs; every traced leg that is
    # not dual contributes its twist (quantum dimensions are 1).
    for k in range(tail_r.shape[1]):
        leg = canonical.codomain[no + k]
        if not leg.is_dual:
            coefficient *= st.twist(leg.visible[tail_r[keep][:, k]])
    return AbelianTransform(basis.src[keep], dst_index, coefficient)
