"""Test infrastructure: a NumPy restatement of the reference's stride
primitives, used only as the checker of the CUDA engine.

Each function states the reference semantics it follows.  Address arithmetic
is exact (integer index arrays); floating-point results are bit-identical to
the reference's CPU executors for copies, real scalings and real sums whose
contributions do not collide.  Complex scalings use NumPy's complex product
(no fused multiply-add), so they match to rounding only.
"""

from __future__ import annotations

import numpy as np


def decode_layout(words):
    """Records of v1 layout words (src/tensor0/_stride/_ffi/_descriptor.py:8-32)."""
    w = [int(x) for x in np.asarray(words, dtype=np.int64)]
    assert w[0] == 1, "unsupported layout version"
    source_size, output_size, count = w[1], w[2], w[3]
    records, at = [], 4
    for _ in range(count):
        rank, src_off, dst_off = w[at], w[at + 1], w[at + 2]
        at += 3
        shape = w[at:at + rank]; at += rank
        sstr = w[at:at + rank]; at += rank
        dstr = w[at:at + rank]; at += rank
        records.append((tuple(shape), tuple(sstr), src_off, tuple(dstr), dst_off))
    return source_size, output_size, records


def decode_reduction_layout(words):
    """Records and reduction roles of reduction words (_descriptor.py:41-76)."""
    w = np.asarray(words, dtype=np.int64).view(np.uint64)
    w = [int(x) for x in w]

    def signed(x):
        return x - (1 << 64) if x >= 1 << 63 else x

    assert w[0] == 1, "unsupported reduction layout version"
    source_size, output_size, count = w[1], w[2], w[3]
    records, at = [], 4
    for _ in range(count):
        rank, src_off, dst_off = w[at], w[at + 1], w[at + 2]
        at += 3
        shape = w[at:at + rank]; at += rank
        sstr = [signed(x) for x in w[at:at + rank]]; at += rank
        at += rank  # output shape (implied by roles)
        dstr = [signed(x) for x in w[at:at + rank]]; at += rank
        roles = [bool(x) for x in w[at:at + rank]]; at += rank
        dstr = [0 if r else d for d, r in zip(dstr, roles)]
        records.append((tuple(shape), tuple(sstr), src_off, tuple(dstr), dst_off, tuple(roles)))
    return source_size, output_size, records


def addresses(shape, strides, offset) -> np.ndarray:
    """Flat addresses of a strided box in C order of its logical index."""
    index = np.full(tuple(shape), offset, dtype=np.int64)
    for axis, (size, stride) in enumerate(zip(shape, strides)):
        view = (1,) * axis + (size,) + (1,) * (len(shape) - axis - 1)
        index = index + np.arange(size, dtype=np.int64).reshape(view) * stride
    return index.reshape(-1)


def _view(array: np.ndarray, offset: int, shape, strides) -> np.ndarray:
    """The strided box (offset, shape, element strides) of the last axis of
    ``array`` as a numpy view, batch axes first.  The layout was validated, so
    every address of the box lies inside the array."""
    item = array.itemsize
    batch_shape = array.shape[:-1]
    batch_strides = array.strides[:-1]
    flat = array.reshape(-1, array.shape[-1]) if batch_shape else array.reshape(1, -1)
    base = flat[:, offset:] if array.shape[-1] else flat
    return np.lib.stride_tricks.as_strided(
        base, shape=(*batch_shape, *shape), strides=(*batch_strides, *(int(s) * item for s in strides)))


def _injective(shape, strides) -> bool:
    """No axis of extent > 1 with stride 0 (a validated record is then injective)."""
    return all(n < 2 or s != 0 for n, s in zip(shape, strides))


def _zero_plus(values: np.ndarray) -> np.ndarray:
    """0 + x, elementwise (turns -0 into +0)."""
    return np.zeros_like(values) + values


def copy(words, source: np.ndarray) -> np.ndarray:
    """Copy: zero output, then out[dst] = src[src] bit for bit
    (crates/tensor0-py/native/execute/copy.h:28-46, 119-134)."""
    _, output_size, records = decode_layout(words)
    view = source.view(np.uint8).reshape(*source.shape[:-1], source.shape[-1], source.itemsize)
    out = np.zeros((*source.shape[:-1], output_size, source.itemsize), np.uint8)
    for shape, sstr, so, dstr, do in records:
        if int(np.prod(shape)) == 0:
            continue
        out[..., addresses(shape, dstr, do), :] = view[..., addresses(shape, sstr, so), :]
    return out.reshape(*source.shape[:-1], output_size * source.itemsize).view(source.dtype)


def _factor(coefficient, batch_shape):
    c = np.asarray(coefficient)
    if c.ndim == 0 or c.shape == (1,):
        return c.reshape(()), True
    return c.reshape(*batch_shape, 1), False


def accumulation(words, source: np.ndarray, coefficients=(), coefficient_records=()) -> np.ndarray:
    """Accumulation: out = 0; per record in order out[dst] += c * src[src];
    a zero coefficient skips the record, a unit one the product
    (ffi/reduction_impl.h:99-118; execute/reduction.h:18-94)."""
    _, output_size, records = decode_layout(words)
    factors = dict(zip((int(r) for r in coefficient_records), coefficients))
    batch_shape = source.shape[:-1]
    out = np.zeros((*batch_shape, output_size), source.dtype)
    for index, (shape, sstr, so, dstr, do) in enumerate(records):
        if int(np.prod(shape)) == 0:
            continue
        fast = _injective(shape, dstr)
        values = _view(source, so, shape, sstr) if fast else source[..., addresses(shape, sstr, so)]
        if index in factors:
            c, shared = _factor(factors[index], batch_shape)
            if shared and c == 0:
                continue
            if not (shared and c == 1):
                if fast and not shared:
                    c = c.reshape(*batch_shape, *([1] * len(shape)))
                values = _scale(c, values, source.dtype)
                if not shared:
                    values = np.where(c == 0, np.zeros_like(values), values)
        if fast:
            # Records run in order; within one, destinations are distinct.
            target = _view(out, do, shape, dstr)
            target += values
        else:
            _scatter_add(out, addresses(shape, dstr, do), values)
    return out


def _scale(c, values, dtype):
    c = np.asarray(c)
    if np.iscomplexobj(values) and not np.iscomplexobj(c):
        real = values.real.dtype
        c = c.astype(real)
        return (c * values.real + 1j * (c * values.imag)).astype(dtype)
    return (c.astype(dtype) * values).astype(dtype)


def _scatter_add(out, dst, values):
    """out[..., dst] += values, summing repeated destinations in order."""
    unique = np.unique(dst).size == dst.size
    if unique:
        out[..., dst] = out[..., dst] + values
    else:
        flat = out.reshape(-1, out.shape[-1])
        vals = values.reshape(-1, values.shape[-1])
        for b in range(flat.shape[0]):
            np.add.at(flat[b], dst, vals[b])


def update(words, source: np.ndarray, base: np.ndarray, alpha, beta) -> np.ndarray:
    """Update: out = base; out[dst] = a*src + b*base[dst] with zero/one
    short-circuits (execute/update.h:28-77; map_reduce_policies.cuh:30-69)."""
    _, _, records = decode_layout(words)
    out = base.copy()
    batch_shape = base.shape[:-1]
    a, _ = _factor(alpha, batch_shape)
    b, _ = _factor(beta, batch_shape)
    rank_a, rank_b = np.ndim(a), np.ndim(b)
    for shape, sstr, so, dstr, do in records:
        if int(np.prod(shape)) == 0:
            continue
        s = _view(source, so, shape, sstr)
        o = _view(base, do, shape, dstr)
        ar = a.reshape(*a.shape, *([1] * (len(shape) - 1))) if rank_a else a
        br = b.reshape(*b.shape, *([1] * (len(shape) - 1))) if rank_b else b
        a0, a1 = np.all(a == 0), np.all(a == 1)
        b0, b1 = np.all(b == 0), np.all(b == 1)
        if a0:
            value = np.zeros_like(o) if b0 else (o if b1 else _scale(br, o, base.dtype))
        else:
            st = s if a1 else _scale(ar, s, base.dtype)
            value = st if b0 else (st + (o if b1 else _scale(br, o, base.dtype))).astype(base.dtype)
        _view(out, do, shape, dstr)[...] = value
    return out


def reduction(words, source: np.ndarray, coefficients=(), coefficient_records=()) -> np.ndarray:
    """Reduction (partial trace): out = 0; per record out[owner] +=
    c * sum over reduction axes (ffi/reduction_impl.h:29-150)."""
    _, output_size, records = decode_reduction_layout(words)
    factors = dict(zip((int(r) for r in coefficient_records), coefficients))
    batch_shape = source.shape[:-1]
    out = np.zeros((*batch_shape, output_size), source.dtype)
    for index, (shape, sstr, so, dstr, do, roles) in enumerate(records):
        if int(np.prod(shape)) == 0:
            continue
        values = source[..., addresses(shape, sstr, so)]
        if index in factors:
            c, shared = _factor(factors[index], batch_shape)
            if shared and c == 0:
                continue
            if not (shared and c == 1):
                values = _scale(c, values, source.dtype)
        _scatter_add(out, addresses(shape, dstr, do), values)
    return out


def sector_gemm(spec, left: np.ndarray, right: np.ndarray, output_size: int) -> np.ndarray:
    """C_g = A_g @ B_g per sector row {m, n, k, a_off, b_off, c_off}, computed
    in float64 / complex128 (stand-in for the XLA dot of linalg.py:560)."""
    wide = np.complex128 if np.iscomplexobj(left) else np.float64
    out = np.zeros(output_size, wide)
    for m, n, k, a, b, c in np.asarray(spec, np.int64).reshape(-1, 6):
        if m * n == 0:
            continue
        if k == 0:
            out[c:c + m * n] = 0
            continue
        A = left[a:a + m * k].reshape(m, k).astype(wide)
        B = right[b:b + k * n].reshape(k, n).astype(wide)
        out[c:c + m * n] = (A @ B).reshape(-1)
    return out


def dot(words, left: np.ndarray, right: np.ndarray, conjugate_left: bool = False) -> np.ndarray:
    """Dot: sum over records and elements of conj?(left[src]) * right[dst],
    per batch (execute/dot.h:21-56; map_reduce_policies.cuh:103-121)."""
    _, _, records = decode_layout(words)
    wide = np.complex128 if np.iscomplexobj(left) else np.float64
    out = np.zeros(left.shape[:-1], wide)
    for shape, sstr, so, dstr, do in records:
        if int(np.prod(shape)) == 0:
            continue
        a = left[..., addresses(shape, sstr, so)].astype(wide)
        b = right[..., addresses(shape, dstr, do)].astype(wide)
        out = out + np.sum((np.conj(a) if conjugate_left else a) * b, axis=-1)
    return out


def grouped(source: np.ndarray, source_blocks, destination_blocks, output_size: int, permutation, groups):
    """Grouped transform (_strided_grouped_transform, _tensor_ops.py:119-203;
    restated after the reference's own checker,
    tests/stride/support/oracles/grouped.py:13-35).

    ``*_blocks`` are (shape, strides, offset) sub-blocks; ``groups`` are
    (src_indices, dst_indices, matrix).  Output starts at zero.  A 1 x 1 group
    is the direct accumulation into zeros (factor 0 gives zeros, 1 the source
    values, others a scaling; -0 becomes +0); a larger one multiplies its
    [n_dst, n_src] matrix into the stacked source rows (products and sums in
    double / complex double, rounded to the storage type once).  Each
    destination row, reshaped to the source block shape and transposed by
    ``permutation``, is written to its destination block.  Real storage uses
    a matrix's real part."""
    dtype = source.dtype
    batch_shape = source.shape[:-1]
    out = np.zeros((*batch_shape, output_size), dtype)
    complex_storage = np.iscomplexobj(source)
    for src_indices, dst_indices, matrix in groups:
        shape = tuple(source_blocks[src_indices[0]][0])
        rows = np.stack([source[..., addresses(*source_blocks[i])] for i in src_indices], axis=-2)
        m = np.asarray(matrix)
        if not complex_storage:
            m = m.real
        if m.shape == (1, 1):
            # The reference runs these as accumulation records into zeros
            # (_tensor_ops.py:168-176): 0 + c * x.
            factor = m.reshape(())
            mapped = (np.zeros_like(rows) if factor == 0 else _zero_plus(rows) if factor == 1
                      else _zero_plus(_scale(factor, rows, dtype)))
        else:
            wide = np.complex128 if complex_storage else np.float64
            mapped = np.einsum("ji,...ik->...jk", m.astype(wide), rows.astype(wide)).astype(dtype)
        for row, index in enumerate(dst_indices):
            shaped = mapped[..., row, :].reshape((*batch_shape, *shape))
            axes = (*range(len(batch_shape)), *(len(batch_shape) + axis for axis in permutation))
            values = np.transpose(shaped, axes).reshape((*batch_shape, int(np.prod(shape))))
            out[..., addresses(*destination_blocks[index])] = values
    return out
