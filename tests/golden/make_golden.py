"""Generate the golden fixtures in this directory (run where the compiled
reference, oracle/_ref, is available):

    python tests/golden/make_golden.py

Fixtures (golden.json):

* reference-authored vectors, restated as layouts with their expected values:
  - copy layouts of tests/stride/native/cpp/copy_execution_test.cc:70-99
    (a transposing permutation with a negative stride, a reversal and a
    strided copy with holes), expected values as that test computes them;
  - the packed trace of tests/stride/support/oracles/trace.py:20-43, expected
    values from its explicit index formula (reference_trace);
* outputs of the compiled reference on the U1 dim-36 workload (f64, seed 1):
  permute ((1, 0), (3, 2)) and add_transform(alpha=1, beta=0.5) into a second
  seeded tensor (seed 2), stored as SHA-256 digests of the output bytes plus
  sampled values.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import ref  # noqa: E402
from tensor0_b200 import stride  # noqa: E402
from tensor0_b200.structure import U1Irrep, degeneracy_structure, hom, space  # noqa: E402
from tensor0_b200.tensor_map import permute_plan  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.json"


def copy_vectors():
    cases = []
    source = [float(i + 1) for i in range(6)]
    layouts = {
        "permutation": stride.AffineRecord((2, 3), (3, 1), 0, (3, -1), 2),
        "reverse": stride.AffineRecord((6,), (1,), 0, (-1,), 5),
        "holes": stride.AffineRecord((3,), (2,), 0, (2,), 0),
    }
    for name, record in layouts.items():
        expected = []
        for i in range(6):
            if name == "permutation":
                expected.append(source[(i // 3) * 3 + (2 - i % 3)])
            elif name == "reverse":
                expected.append(source[5 - i])
            else:
                expected.append(source[i] if i % 2 == 0 else 0.0)
        words = stride.encode_layout((record,), source_size=6, output_size=6)
        computed = ref.copy(words, np.array(source, np.float64), 6)
        assert computed.tolist() == expected, (name, computed, expected)
        cases.append({"name": name, "words": words.tolist(), "source": source, "expected": expected})
    return cases


def packed_trace_vector():
    """tests/stride/support/oracles/trace.py:20-43 restated as one reduction layout."""
    subblocks = [((2, 0, 0), (1, 1, 1), 12), ((2, 2, 2), (4, 2, 1), 0), ((2, 2, 2), (0, -2, -1), 3)]
    destinations = [((2,), (1,), 1), ((2,), (-1,), 3)]
    entries = [(0, 0, None), (1, 0, None), (2, 1, 3.0), (1, 1, -2.0)]
    records, shapes, roles, coefficients, coefficient_records = [], [], [], [], []
    for index, (s, d, factor) in enumerate(entries):
        sizes, strides, offset = subblocks[s]
        dsizes, dstrides, doffset = destinations[d]
        records.append(stride.AffineRecord((sizes[0], sizes[1]), (strides[0], strides[1] + strides[2]), offset,
                                           (dstrides[0], 1), doffset))
        shapes.append((dsizes[0], 1))
        roles.append((False, True))
        if factor is not None:
            coefficients.append(factor)
            coefficient_records.append(index)
    words = stride.encode_reduction_layout(records, output_shapes=shapes, reduction_axes=roles,
                                           source_size=13, output_size=5)
    rng = np.random.default_rng(11)
    source = rng.standard_normal(13)
    factor, second = 3.0, -2.0
    first = source[np.array([[0, 3], [4, 7]])]
    broadcast = source[np.array([[3, 0], [3, 0]])]
    expected = np.zeros(5)
    expected[1:3] += first.sum(axis=-1)
    contribution = (broadcast * factor).sum(axis=-1) + (first * second).sum(axis=-1)
    np.add.at(expected, np.array([3, 2]), contribution)
    computed = ref.reduction(words, source, 5, [np.float64(c) for c in coefficients], coefficient_records)
    assert np.allclose(computed, expected, rtol=1e-14, atol=1e-14), (computed, expected)
    return {"words": words.tolist(), "source": source.tolist(), "coefficients": coefficients,
            "coefficient_records": coefficient_records, "expected": expected.tolist()}


def digest(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def config_one():
    v = space(U1Irrep, {-2: 4, -1: 8, 0: 12, 1: 8, 2: 4})
    h = hom((v, v), (v, v))
    plan = permute_plan(h, (1, 0), (3, 2))
    n = degeneracy_structure(h).total_dim
    x = np.random.default_rng(1).standard_normal(n)
    y = np.random.default_rng(2).standard_normal(plan.output_size)
    records = np.arange(len(plan.transform.src))
    permuted = ref.accumulation(plan.words, x, plan.output_size, [np.float64(1.0)] * len(records), records,
                                outputs_disjoint=True, threads=4)
    updated = ref.update(plan.words, x, y, np.float64(1.0), np.float64(0.5), threads=4)
    samples = np.random.default_rng(0).choice(plan.output_size, 64, replace=False)
    return {
        "space": {"U1": {"-2": 4, "-1": 8, "0": 12, "1": 8, "2": 4}, "codomain": 2, "domain": 2},
        "total_dim": int(n), "records": int(len(records)), "words_sha256": digest(plan.words),
        "permute_sha256": digest(permuted), "add_transform_sha256": digest(updated),
        "samples": samples.tolist(), "permute_samples": permuted[samples].tolist(),
        "add_transform_samples": updated[samples].tolist(),
    }


def main():
    fixtures = {"copy": copy_vectors(), "packed_trace": packed_trace_vector(), "config_one": config_one()}
    OUT.write_text(json.dumps(fixtures, indent=1))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
