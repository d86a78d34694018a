"""The multi-GPU host logic on CPU: row shards, and a world_size-2 gloo group running the per-rank protocol
(shard -> sample each shard independently -> gather ids, max over ranks of a timing).

Rows are independent in the reference (TalkerGenerator.cs:366-385), so ids sampled shard by shard and gathered
in rank order must equal the ids of the whole batch.  The per-shard sampler here is the CPU oracle (no GPU in
this suite); the GPU path takes the same shards.
"""

import json
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from voxwerk_b200 import workloads
from voxwerk_b200.shard import shard_bounds


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_the_batch_in_order(world):
    costs = [(1024, 16384.0), (15360, 4096.0)]   # config 3: talker rows, then sub-talker rows
    seen = {0: [], 1: []}
    loads = []
    for r in range(world):
        load = 0.0
        for s, a, b in shard_bounds(costs, r, world):
            seen[s].append((a, b))
            load += (b - a) * costs[s][1]
        loads.append(load)
    for s, (n, _) in enumerate(costs):
        ranges = seen[s]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(ranges[i][1] == ranges[i + 1][0] for i in range(len(ranges) - 1))
    total = sum(n * c for n, c in costs)
    assert max(loads) - min(loads) <= 2 * max(c for _, c in costs) + 1e-6 * total


def test_workload_shards_rebuild_the_workload():
    w = workloads.make(3, 6)
    parts = [w.shard(r, 2) for r in range(2)]
    assert sum(p.n_rows for p in parts) == w.n_rows
    logits = np.concatenate([s.logits for p in parts for s in p.segments if s.kind == 0])
    assert np.array_equal(logits, w.segments[0].logits)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import oracle
        from voxwerk_b200.shard import gather_ids, max_over_ranks
        w = workloads.make(3, 4)   # 4 talker rows + 60 sub-talker rows, bf16
        part = w.shard(rank, world)
        local = [oracle.sample_segment(s, w.options, threads=1) for s in part.segments]
        ids = np.concatenate(local) if local else np.zeros(0, np.int32)
        all_ids = gather_ids(ids)
        slowest = max_over_ranks(1.5 * (rank + 1))
        if rank == 0:
            np.save(os.path.join(out_dir, "ids.npy"), all_ids)
            with open(os.path.join(out_dir, "max.json"), "w") as f:
                json.dump({"max": slowest, "rows": [int(ids.size)]}, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_sample_and_gather(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    from oracle import oracle
    w = workloads.make(3, 4)
    whole = np.concatenate([oracle.sample_segment(s, w.options, threads=1) for s in w.segments])
    got = np.load(tmp_path / "ids.npy")
    assert np.array_equal(got, whole)
    assert json.load(open(tmp_path / "max.json"))["max"] == 3.0
