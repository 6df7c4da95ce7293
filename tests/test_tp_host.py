"""Host side of tensor parallelism on CPU, two gloo ranks (127.0.0.1): the
shard plan of every weight role tiles the full matrix exactly once across
ranks (row splits for q/k/v/gate/up/lm_head, column splits for o/down,
replicas for embeddings and norms), and the benchmark's rank plumbing
(barrier, max over ranks, broadcast of the NCCL unique id) agrees on all
ranks."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from starlight_b200.engine import LLAMA2_70B, LLAMA3_8B, ROLES, SHARDING, full_shape, shard_plan


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    d = bench.Dist(world)
    try:
        plans = {}
        for name, cfg in (("8b", LLAMA3_8B), ("70b", LLAMA2_70B)):
            plans[name] = {r: shard_plan(cfg, r, rank, world) for r in ROLES}
        gathered = [None] * world
        dist.all_gather_object(gathered, plans)
        uid = d.broadcast_bytes(bytes(range(128)) if rank == 0 else None, 128)
        mx = d.max(float(rank) + 0.5)
        d.barrier()
        q.put((rank, gathered, uid, mx))
    finally:
        d.close()


@pytest.mark.parametrize("world", [2])
def test_shard_plans_and_rank_plumbing(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, uid, mx in results:
        assert uid == bytes(range(128))
        assert mx == world - 1 + 0.5
        assert gathered == results[0][1]
    plans = results[0][1]
    for name, cfg in (("8b", LLAMA3_8B), ("70b", LLAMA2_70B)):
        for role in ROLES:
            fr, fc = full_shape(cfg, role)
            shards = [plans[r][name][role] for r in range(world)]
            if SHARDING[role] == 0:
                assert all(s == (0, fr, 0, fc) for s in shards)
            elif SHARDING[role] == 1:
                assert [s[0] for s in shards] == [r * fr // world for r in range(world)]
                assert sum(s[1] for s in shards) == fr and all(s[3] == fc for s in shards)
            else:
                assert [s[2] for s in shards] == [r * fc // world for r in range(world)]
                assert sum(s[3] for s in shards) == fc and all(s[1] == fr for s in shards)
            # Row-parallel shards hold whole quantization groups (group 128).
            if SHARDING[role] == 2:
                assert shards[0][3] % 128 == 0
