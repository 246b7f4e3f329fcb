"""Sector (record) sharding across GPUs with longest-processing-time balancing.

Charge sectors are independent: every record of a permute reads one source
sub-block and writes one destination sub-block.  A shard owns a set of
records, holds their source sub-blocks compacted in its own HBM (input
sharding by record) and writes their destination sub-blocks compacted, so the
timed kernels need no communication.  Collectives are used only to gather (or
reshard) outputs whose ownership changes, outside the kernels' timed region.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np

from . import stride


def lpt_partition(costs, parts: int) -> list[np.ndarray]:
    """Greedy LPT: largest cost first, each to the least-loaded part (ties to
    the lowest part index).  Deterministic; returns sorted index arrays."""
    costs = np.asarray(costs, dtype=np.float64)
    if parts < 1:
        raise ValueError("parts must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, p) for p in range(parts)]
    owned: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        load, p = heapq.heappop(heap)
        owned[p].append(i)
        heapq.heappush(heap, (load + costs[i], p))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


def _row_major(shape: np.ndarray) -> np.ndarray:
    strides = np.ones_like(shape)
    for axis in range(shape.shape[1] - 2, -1, -1):
        strides[:, axis] = strides[:, axis + 1] * shape[:, axis + 1]
    return strides


@dataclass
class PermuteShard:
    """One rank's part of a permute: owned records and their compacted layout."""

    rank: int
    world: int
    records: np.ndarray          # global record indices (ascending)
    src_sizes: np.ndarray        # [R, rank] source sub-block sizes (source axis order)
    src_strides: np.ndarray      # [R, rank] global source strides
    src_offsets: np.ndarray      # [R] global source offsets
    dst_sizes: np.ndarray        # [R, rank] destination sub-block sizes
    dst_strides: np.ndarray      # [R, rank] global destination strides
    dst_offsets: np.ndarray      # [R] global destination offsets
    local_src_offsets: np.ndarray
    local_dst_offsets: np.ndarray
    local_source_size: int
    local_output_size: int
    words: np.ndarray            # local layout words

    @property
    def bytes_per_element_pair(self) -> int:
        return int(np.prod(self.dst_sizes, axis=1).sum())

    def _addresses(self, sizes, strides, offset):
        index = np.full(tuple(sizes), offset, dtype=np.int64)
        for axis, (n, s) in enumerate(zip(sizes, strides)):
            view = [1] * len(sizes)
            view[axis] = n
            index = index + np.arange(n, dtype=np.int64).reshape(view) * s
        return index.reshape(-1)

    def source_index(self) -> np.ndarray:
        """Global source address of every local source element, in local order."""
        parts = [self._addresses(s, t, o) for s, t, o in zip(self.src_sizes, self.src_strides, self.src_offsets)]
        return np.concatenate(parts) if parts else np.zeros(0, np.int64)

    def output_index(self) -> np.ndarray:
        """Global destination address of every local output element, in local order."""
        parts = [self._addresses(s, t, o) for s, t, o in zip(self.dst_sizes, self.dst_strides, self.dst_offsets)]
        return np.concatenate(parts) if parts else np.zeros(0, np.int64)


def shard_permute(plan, rank: int, world: int, element_bytes: int = 8) -> PermuteShard:
    """LPT-partition a permute's records (cost = bytes moved) and build the
    compacted local layout of shard ``rank``."""
    from .structure import degeneracy_structure

    sd = degeneracy_structure(plan.src)
    counts = np.prod(plan.shape, axis=1) if plan.shape.size else np.ones(len(plan.transform.src), np.int64)
    owned = lpt_partition(2 * counts * element_bytes, world)[rank]
    src_idx = plan.transform.src[owned]
    src_sizes = sd.sizes[src_idx]
    src_strides = sd.strides[src_idx]
    dst_sizes = plan.shape[owned]
    local_counts = np.prod(dst_sizes, axis=1) if len(owned) else np.zeros(0, np.int64)
    local_offsets = np.concatenate([[0], np.cumsum(local_counts)[:-1]]).astype(np.int64) if len(owned) else \
        np.zeros(0, np.int64)
    total = int(local_counts.sum())
    # Local source sub-blocks are compact row-major in source axis order; the
    # record reads them through the permutation.
    perm = list(plan.perm)
    compact_src = _row_major(src_sizes) if len(owned) else np.zeros((0, src_sizes.shape[1]), np.int64)
    local_src_strides = compact_src[:, perm] if len(owned) else compact_src
    local_dst_strides = _row_major(dst_sizes) if len(owned) else np.zeros_like(dst_sizes)
    words = stride.encode_layout_arrays(dst_sizes, local_src_strides, local_offsets, local_dst_strides,
                                        local_offsets, source_size=total, output_size=total)
    return PermuteShard(rank, world, owned, src_sizes, src_strides, sd.offsets[src_idx], dst_sizes,
                        plan.dst_strides[owned], plan.dst_offsets[owned], local_offsets, local_offsets, total, total,
                        words)


def shard_capacity(plan, world: int, element_bytes: int = 8) -> int:
    """Largest local output (elements) over the shards: the padded size of
    one rank's part of an all-gather."""
    return max(shard_permute(plan, r, world, element_bytes).local_output_size for r in range(world))


def gather_words(plan, world: int, element_bytes: int = 8) -> np.ndarray:
    """Copy layout words that unpack an all-gathered buffer — shard r's
    compacted destination sub-blocks at r * capacity — into the packed
    destination layout of the whole tensor (one engine copy)."""
    from .structure import degeneracy_structure

    capacity = shard_capacity(plan, world, element_bytes)
    shapes, src_strides, src_offsets, dst_strides, dst_offsets = [], [], [], [], []
    for r in range(world):
        shard = shard_permute(plan, r, world, element_bytes)
        if not shard.records.size:
            continue
        shapes.append(shard.dst_sizes)
        src_strides.append(_row_major(shard.dst_sizes))
        src_offsets.append(r * capacity + shard.local_dst_offsets)
        dst_strides.append(shard.dst_strides)
        dst_offsets.append(shard.dst_offsets)
    return stride.encode_layout_arrays(np.concatenate(shapes), np.concatenate(src_strides),
                                       np.concatenate(src_offsets), np.concatenate(dst_strides),
                                       np.concatenate(dst_offsets), source_size=world * capacity,
                                       output_size=degeneracy_structure(plan.dst).total_dim)


def scatter_words(plan, rank: int, world: int, element_bytes: int = 8, *, source: bool = True) -> np.ndarray:
    """Copy layout words that extract shard `rank`'s sub-blocks from the packed
    layout of the whole tensor into its compacted local buffer: the source
    sub-blocks (`source`, for distributing inputs) or the destination
    sub-blocks (for a shard's share of an existing output)."""
    shard = shard_permute(plan, rank, world, element_bytes)
    from .structure import degeneracy_structure

    if source:
        sizes, strides, offsets = shard.src_sizes, shard.src_strides, shard.src_offsets
        local, total = shard.local_src_offsets, shard.local_source_size
        whole = degeneracy_structure(plan.src).total_dim
    else:
        sizes, strides, offsets = shard.dst_sizes, shard.dst_strides, shard.dst_offsets
        local, total = shard.local_dst_offsets, shard.local_output_size
        whole = degeneracy_structure(plan.dst).total_dim
    compact = _row_major(sizes) if len(sizes) else np.zeros_like(sizes)
    return stride.encode_layout_arrays(sizes, strides, offsets, compact, local, source_size=whole, output_size=total)
