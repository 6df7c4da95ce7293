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


# ---- rank liveness between steps (starlight_b200/health.py) ---------------------

def _watch_main(rank, world, port, last_step, q):
    import datetime

    import torch.distributed as dist
    from starlight_b200.health import RankFailure, RankWatch
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    watch = RankWatch(store, rank, world, timeout_s=1.0)
    done, failure = [], None
    try:
        for i in range(last_step + 1):
            watch.step(i)
            done.append(i)
    except RankFailure as e:
        failure = (e.step, e.missing)
    q.put((rank, done, failure))
    if rank == 0:  # the store's server lives in rank 0: outlive the others' last use
        import time
        time.sleep(0.5)


def _run_watch(last_steps):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = len(last_steps)
    procs = [ctx.Process(target=_watch_main, args=(r, world, port, last_steps[r], q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (d, f)) for r, d, f in (q.get(timeout=60) for _ in range(world)))
    for p in procs:
        p.join(timeout=30)
    return res


def test_rank_watch_all_ranks_step_together():
    res = _run_watch([5, 5])
    for r in range(2):
        assert res[r] == (list(range(6)), None), res[r]


def test_rank_watch_detects_a_rank_that_left_between_steps():
    # Rank 1 leaves after step 2; rank 0 must learn it before step 3's work,
    # within the watch's bound, instead of entering a collective that waits.
    import time
    t0 = time.time()
    res = _run_watch([6, 2])
    assert res[1] == ([0, 1, 2], None), res[1]
    assert res[0] == ([0, 1, 2], (3, [1])), res[0]
    assert time.time() - t0 < 30
