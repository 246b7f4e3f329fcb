"""Seeded random stride layouts shared by the CPU and GPU tests."""

import numpy as np

from tensor0_b200 import stride


def random_reduction_layout(rng, source_size, records):
    """Random reduction records: a permuted strided box of the source per
    record, some axes summed; outputs either a fresh contiguous region or the
    region of an earlier record with the same open shape (contributions add)."""
    out, shapes, roles, regions, cursor = [], [], [], [], 0
    for _ in range(records):
        rank = int(rng.integers(1, 5))
        shape = tuple(int(n) for n in rng.integers(1, 5, size=rank))
        role = tuple(bool(r) for r in rng.integers(0, 2, size=rank))
        count = int(np.prod(shape))
        if count > source_size:
            continue
        perm = rng.permutation(rank)
        src_contig = stride.contiguous_strides(tuple(shape[p] for p in perm))
        sstr = [0] * rank
        for i, p in enumerate(perm):
            sstr[p] = src_contig[i]
        sign = rng.choice([-1, 1], size=rank)
        sstr = [int(s * g) for s, g in zip(sstr, sign)]
        soff = int(rng.integers(0, source_size - count + 1))
        soff += sum((n - 1) * (-s) for n, s in zip(shape, sstr) if s < 0)
        if soff + sum((n - 1) * s for n, s in zip(shape, sstr) if s > 0) >= source_size:
            continue
        open_shape = tuple(n for n, r in zip(shape, role) if not r)
        reuse = [d for s, d in regions if s == open_shape]
        if reuse and rng.random() < 0.5:
            dst_off = int(rng.choice(reuse))
        else:
            dst_off = cursor
            regions.append((open_shape, cursor))
            cursor += int(np.prod(open_shape)) + int(rng.integers(0, 2))
        open_strides = iter(stride.contiguous_strides(open_shape))
        dstr = tuple(1 if r else next(open_strides) for r in role)
        out.append(stride.AffineRecord(shape, tuple(sstr), soff, dstr, dst_off))
        shapes.append(tuple(1 if r else n for n, r in zip(shape, role)))
        roles.append(role)
    return out, shapes, roles, max(cursor, 1)


def random_layout(rng, source_size, output_size, records, max_rank=4, max_extent=6):
    """Disjoint random records: permuted strided boxes of the source (some
    strides negative) written to consecutive output ranges with small gaps."""
    out, cursor = [], 0
    for _ in range(records):
        rank = int(rng.integers(1, max_rank + 1))
        shape = tuple(int(n) for n in rng.integers(1, max_extent, size=rank))
        count = int(np.prod(shape))
        if cursor + count > output_size:
            break
        if count > source_size:
            continue
        dst = stride.contiguous_strides(shape)
        perm = rng.permutation(rank)
        src_shape = tuple(shape[p] for p in perm)
        src_contig = stride.contiguous_strides(src_shape)
        sstr = [0] * rank
        for i, p in enumerate(perm):
            sstr[p] = src_contig[i]
        sign = rng.choice([-1, 1], size=rank)
        sstr = [int(s * g) for s, g in zip(sstr, sign)]
        soff = int(rng.integers(0, source_size - count + 1))
        soff += sum((n - 1) * (-s) for n, s in zip(shape, sstr) if s < 0)
        if soff + sum((n - 1) * s for n, s in zip(shape, sstr) if s > 0) >= source_size:
            continue
        out.append(stride.AffineRecord(shape, tuple(sstr), soff, dst, cursor))
        cursor += count + int(rng.integers(0, 3))
    return out
