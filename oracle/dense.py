"""Test infrastructure: dense-tensor contracts of the block-sparse operations.

The reference's own TensorMap tests check every hot-path operation against
dense arithmetic on ``to_dense``: permute against a transpose
(tests/test_transforms.py:99, 685-692), trace against an explicit dense trace
(tests/test_contractions.py:669-726) and contraction against tensordot
(tests/test_contractions.py:374-391, 436-461).  This module restates
``to_dense`` for abelian spaces (every sub-block placed at its legs' sector
offsets) so the same contracts can be checked here.
"""

from __future__ import annotations

import numpy as np


def to_dense(space, storage: np.ndarray) -> np.ndarray:
    """Dense array [leg dims...] of packed storage for ``space``."""
    from tensor0_b200.structure import degeneracy_structure, sector_structure

    ss, ds = sector_structure(space), degeneracy_structure(space)
    legs = (*space.codomain, *space.domain)
    dense = np.zeros(tuple(leg.dim for leg in legs), dtype=storage.dtype)
    legs_idx = np.concatenate([ss.pair_row, ss.pair_col], axis=1)
    for p in range(ss.pair_count):
        sizes, strides, offset = ds.sizes[p], ds.strides[p], int(ds.offsets[p])
        index = np.full(tuple(sizes), offset, dtype=np.int64)
        for axis, (n, s) in enumerate(zip(sizes, strides)):
            view = [1] * len(sizes)
            view[axis] = n
            index = index + np.arange(n).reshape(view) * s
        slices = tuple(slice(int(leg.offsets[i]), int(leg.offsets[i]) + int(n))
                       for leg, i, n in zip(legs, legs_idx[p], sizes))
        dense[slices] = storage[index] if len(sizes) else storage[offset]
    return dense


def permute(dense: np.ndarray, p_codomain, p_domain) -> np.ndarray:
    return np.transpose(dense, tuple(p_codomain) + tuple(p_domain))


def trace(dense: np.ndarray, left, right, out_codomain, out_domain) -> np.ndarray:
    """Sum over paired axes (left[i], right[i]); result axes in output order."""
    rank = dense.ndim
    letters = [chr(ord("a") + i) for i in range(rank)]
    for l_axis, r_axis in zip(left, right):
        letters[r_axis] = letters[l_axis]
    result = "".join(letters[a] for a in (*out_codomain, *out_domain))
    return np.einsum("".join(letters) + "->" + result, dense)


def contract(a: np.ndarray, b: np.ndarray, left_axes, right_axes, output) -> np.ndarray:
    """tensordot over paired axes, open axes placed as ``output`` refs (operand, axis)."""
    rest = np.tensordot(a, b, axes=(tuple(left_axes), tuple(right_axes)))
    open_a = [x for x in range(a.ndim) if x not in left_axes]
    open_b = [x for x in range(b.ndim) if x not in right_axes]
    position = {(0, x): i for i, x in enumerate(open_a)}
    position.update({(1, x): len(open_a) + i for i, x in enumerate(open_b)})
    order = [position[r] for r in (*output[0], *output[1])]
    return np.transpose(rest, order)
