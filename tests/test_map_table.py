"""The packed map-engine table, decoded the way the map kernel decodes it.

Each MapRecord (tensor0_b200/csrc/plan.h) carries division constants computed
on the host; the kernel splits a tile index with them and derives the tile's
box (edge tiles are smaller) and origin.  These tests restate that decode in
NumPy and check, for planner-built tables, that the boxes of all tiles cover
every element of every record exactly once, at the record's source and
destination offsets.  No GPU is involved.
"""

import numpy as np
import pytest
import torch

from tensor0_b200 import _native, stride
from tensor0_b200.structure import U1Irrep, ZNIrrep, hom, space
from tensor0_b200.tensor_map import permute_plan

WORDS = 42          # MapRecord is 336 bytes
HEADER = 16


def records(table):
    count, tiles, offset = int(table[1]), int(table[2]), int(table[3])
    out = []
    for i in range(count):
        w = table[offset + i * WORDS: offset + (i + 1) * WORDS]
        i32, u32 = w[19:].view(np.int32), w[19:].view(np.uint32)
        out.append(dict(src=int(w[0]), dst=int(w[1]), begin=int(w[2]), s=w[3:11].astype(np.int64),
                        d=w[11:19].astype(np.int64), n=i32[0:8].astype(np.int64), t=i32[8:11].astype(np.int64),
                        c=i32[11:14].astype(np.int64), nouter=int(i32[14]), edge=i32[34:36].astype(np.int64),
                        div_tiles=[(int(u32[18 + 2 * k]), int(u32[19 + 2 * k])) for k in range(8)],
                        div_extent=[(int(u32[36 + 2 * k]), int(u32[37 + 2 * k])) for k in range(4)]))
    return out, tiles


def divide(n, constants):
    """(umulhi(n, magic) + n) >> shift, the kernel's division (n < 2^31)."""
    magic, shift = constants
    n = np.asarray(n, dtype=np.uint64)
    return (((n * np.uint64(magic)) >> np.uint64(32)) + n) >> np.uint64(shift)


def covered(table, source_size, output_size):
    """Per output element: how often a tile writes it, and the source offset it reads."""
    recs, tiles = records(table)
    hits = np.zeros(output_size, np.int64)
    source_of = np.full(output_size, -1, np.int64)
    begins = np.array([r["begin"] for r in recs])
    for local in range(tiles):
        r = recs[int(np.searchsorted(begins, local, side="right")) - 1]
        q = local - r["begin"]
        chunk = []
        for i in range(3):
            nxt = int(divide(q, r["div_tiles"][i]))
            assert nxt == q // r["c"][i]
            chunk.append(q - nxt * int(r["c"][i]))
            q = nxt
        so, do = r["src"], r["dst"]
        for i in range(r["nouter"]):
            extent = int(r["n"][3 + i])
            nxt = int(divide(q, r["div_tiles"][3 + i]))
            assert nxt == q // extent
            so += (q - nxt * extent) * int(r["s"][3 + i])
            do += (q - nxt * extent) * int(r["d"][3 + i])
            q = nxt
        assert q == 0
        last = [chunk[i] == r["c"][i] - 1 for i in range(2)]
        ex = int(r["edge"][0]) if last[0] else int(r["t"][0])
        ey = int(r["edge"][1]) if last[1] else int(r["t"][1])
        z0 = chunk[2] * int(r["t"][2])
        ez = min(int(r["t"][2]), int(r["n"][2]) - z0)
        for k, extent in ((0, ex), (1, ey)):
            assert extent == min(int(r["t"][k]), int(r["n"][k]) - chunk[k] * int(r["t"][k])) > 0
            assert int(divide(extent, r["div_extent"][2 * k + int(last[k])])) == 1
        origin = np.array([chunk[0] * r["t"][0], chunk[1] * r["t"][1], z0])
        x, y, z = np.meshgrid(np.arange(ex), np.arange(ey), np.arange(ez), indexing="ij")
        idx = np.stack([x.ravel(), y.ravel(), z.ravel()]) + origin[:, None]
        src = so + (idx * r["s"][:3, None]).sum(0)
        dst = do + (idx * r["d"][:3, None]).sum(0)
        assert src.min() >= 0 and src.max() < source_size and dst.min() >= 0 and dst.max() < output_size
        np.add.at(hits, dst, 1)
        source_of[dst] = src
    return hits, source_of


def expected_sources(layout_records, output_size):
    out = np.full(output_size, -1, np.int64)
    for rec in layout_records:
        idx = np.indices(rec.logical_shape).reshape(len(rec.logical_shape), -1)
        src = rec.source_offset + sum(idx[k] * rec.source_strides[k] for k in range(len(rec.logical_shape)))
        dst = rec.destination_offset + sum(idx[k] * rec.destination_strides[k] for k in range(len(rec.logical_shape)))
        out[dst] = src
    return out


@pytest.mark.parametrize("element_bytes", [4, 16])
@pytest.mark.parametrize("op", [_native.OP_ACCUMULATION, _native.OP_UPDATE, _native.OP_COPY])
def test_permute_table_covers_each_output_once(op, element_bytes):
    v = space(U1Irrep, {-2: 30, -1: 70, 0: 90, 1: 70, 2: 30})
    plan = permute_plan(hom((v, v), (v,)), (2, 0), (1,))
    records_ = np.arange(len(plan.transform.src)) if op == _native.OP_ACCUMULATION else ()
    engine = stride.Plan(op, plan.words, element_bytes=element_bytes, coefficient_records=records_,
                         outputs_disjoint=plan.outputs_disjoint)
    hits, source_of = covered(engine.table, engine.source_size, engine.output_size)
    assert (hits == 1).all()
    src = np.arange(plan.source_size, dtype=np.float64)
    from oracle import stride_oracle
    assert np.array_equal(source_of.astype(np.float64), stride_oracle.copy(plan.words, src))


def test_random_layouts_with_outer_axes_and_negative_strides():
    rng = np.random.default_rng(7)
    for trial in range(6):
        size = 40_000
        layout, cursor = [], 0
        for _ in range(8):
            rank = int(rng.integers(1, 6))
            shape = tuple(int(n) for n in rng.integers(1, 40 if rank <= 3 else 9, size=rank))
            count = int(np.prod(shape))
            if cursor + count > size:
                break
            perm = rng.permutation(rank)
            src_contig = stride.contiguous_strides(tuple(shape[p] for p in perm))
            sstr = [0] * rank
            for i, p in enumerate(perm):
                sstr[p] = src_contig[i]
            sign = rng.choice([-1, 1], size=rank)
            sstr = [int(a * b) for a, b in zip(sstr, sign)]
            soff = int(rng.integers(0, size - count + 1)) + sum((n - 1) * -s for n, s in zip(shape, sstr) if s < 0)
            if soff + sum((n - 1) * s for n, s in zip(shape, sstr) if s > 0) >= size:
                continue
            layout.append(stride.AffineRecord(shape, tuple(sstr), soff, stride.contiguous_strides(shape), cursor))
            cursor += count + int(rng.integers(0, 3))
        words = stride.encode_layout(layout, source_size=size, output_size=size)
        engine = stride.Plan(_native.OP_COPY, words, element_bytes=8)
        hits, source_of = covered(engine.table, size, size)
        want = expected_sources(layout, size)
        assert np.array_equal(hits, (want >= 0).astype(np.int64))
        assert np.array_equal(source_of[want >= 0], want[want >= 0])


def test_three_by_three_z3_sectors_with_outer_axes():
    v = space(ZNIrrep(3), {0: 5, 1: 4, 2: 3})
    plan = permute_plan(hom((v, v, v), (v, v)), (4, 2, 0), (3, 1))
    engine = plan.engine_plan(_native.OP_ACCUMULATION, torch.float32)
    hits, _ = covered(engine.table, engine.source_size, engine.output_size)
    assert (hits == 1).all()
