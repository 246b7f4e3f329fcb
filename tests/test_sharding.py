"""LPT sector sharding: balance, coverage, and a two-rank gloo run whose
gathered output equals the single-process permute bit for bit."""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import stride_oracle as so
from tensor0_b200 import _native, stride
from tensor0_b200.sharding import lpt_partition, shard_permute
from tensor0_b200.structure import U1Irrep, degeneracy_structure, hom, space
from tensor0_b200.tensor_map import permute_plan


def test_lpt_partition_is_balanced_and_complete():
    rng = np.random.default_rng(0)
    costs = rng.integers(1, 1000, size=489)
    for parts in (1, 2, 4, 8):
        shards = lpt_partition(costs, parts)
        assert sorted(np.concatenate(shards).tolist()) == list(range(489))
        loads = [costs[s].sum() for s in shards]
        # LPT is within 4/3 of optimal; the average load bounds the optimum from below.
        assert max(loads) <= (4 / 3) * max(costs.sum() / parts, costs.max()) + 1
    assert all(np.array_equal(a, b) for a, b in zip(lpt_partition(costs, 4), lpt_partition(costs, 4)))


def benchmark_plan(scale=16):
    degs = {q: max(1, int(round(scale * np.exp(-q * q / 8)))) for q in range(-4, 5)}
    v = space(U1Irrep, degs)
    return permute_plan(hom((v, v), (v, v)), (2, 0), (3, 1))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_every_record_and_validate(world):
    plan = benchmark_plan()
    shards = [shard_permute(plan, r, world, 4) for r in range(world)]
    assert sorted(np.concatenate([s.records for s in shards]).tolist()) == list(range(len(plan.transform.src)))
    for shard in shards:
        if shard.records.size:
            engine = stride.Plan(_native.OP_ACCUMULATION, shard.words, element_bytes=4,
                                 coefficient_records=np.arange(shard.records.size), outputs_disjoint=True)
            assert engine.info["full_coverage"] == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        plan = benchmark_plan(8)
        n = degeneracy_structure(plan.src).total_dim
        x = np.random.default_rng(5).standard_normal(n)
        shard = shard_permute(plan, rank, world, 8)
        local_source = x[shard.source_index()]
        local = so.accumulation(shard.words, local_source, [1.0] * shard.records.size, np.arange(shard.records.size))
        # Gather the variable-size shards (padded) and their global output addresses.
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([local.size], dtype=torch.int64))
        width = int(max(s.item() for s in sizes))
        values = torch.zeros(width, dtype=torch.float64)
        values[:local.size] = torch.from_numpy(local)
        index = torch.full((width,), -1, dtype=torch.int64)
        index[:local.size] = torch.from_numpy(shard.output_index())
        all_values = [torch.zeros(width, dtype=torch.float64) for _ in range(world)]
        all_index = [torch.zeros(width, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(all_values, values)
        dist.all_gather(all_index, index)
        if rank == 0:
            out = np.full(plan.output_size, np.nan)
            for v, i in zip(all_values, all_index):
                keep = i >= 0
                out[i[keep].numpy()] = v[keep].numpy()
            records = np.arange(len(plan.transform.src))
            expected = so.accumulation(plan.words, x, [1.0] * records.size, records)
            ok = np.array_equal(out.view(np.uint64), expected.view(np.uint64))
            with open(os.path.join(result_dir, "ok"), "w") as f:
                f.write("1" if ok else "0")
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharded_permute_equals_single_process():
    with tempfile.TemporaryDirectory() as result_dir:
        mp.start_processes(_worker, args=(2, _free_port(), result_dir), nprocs=2, join=True, start_method="spawn")
        assert open(os.path.join(result_dir, "ok")).read() == "1"
