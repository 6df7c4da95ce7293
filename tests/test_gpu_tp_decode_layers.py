"""The persistent decode-layer kernel under tensor parallelism (one process
per GPU): every rank runs its shard of the layers (q/k/v/gate/up rows, o/down
columns) in one cooperative launch per step, and the o and down partial sums
are all-reduced inside the kernel over peer memory (plain NVLink stores and
per-CTA flags, summed in rank order).

At batch 1 with command capture on, the logits of every decode step must
match the single-GPU run of the same model (itself checked against the CPU
oracle in test_gpu_decode_layers.py) within the reduction/matmul tolerance,
with the same token ids fed to both (teacher forcing). The fused path must
actually be taken: all ranks agree on it at comm_init, and replayed steps
launch a handful of kernels instead of one per command. Skipped with fewer
GPUs than ranks."""
import os

import numpy as np
import pytest

from tests.gpu_util import assert_reduction
from tests.test_gpu_tp import _free_port, _gpus

pytestmark = pytest.mark.gpu

# hidden 2048, 16 q heads / 8 kv heads of 128, FFN 4096: at 2, 4 and 8 ranks
# the shards have 4 / 2 / 1 kv heads, o rows of 512 / 256 / 128 code bytes
# and down rows of 1024 / 512 / 256 bytes (one chunk, scales by bulk copy).
CFG = dict(layers=2, hidden=2048, heads=16, kv_heads=8, head_dim=128, inter=4096, vocab=2048,
           batch=1, prefill_len=40, max_seq=64, eps=1e-5, theta=500000.0, group_size=128)
STEPS = 8


def _ids():
    rng = np.random.default_rng(23)
    seq = [rng.integers(0, CFG["vocab"], size=CFG["prefill_len"], dtype=np.uint32)]
    for _ in range(STEPS):
        seq.append(rng.integers(0, CFG["vocab"], size=1, dtype=np.uint32))
    return seq


def _run(rank, world, ids_seq):
    from starlight_b200.device import CudaDevice, QuantFormat, comm_unique_id
    from starlight_b200.engine import DECODE, PREFILL, Llama, LlamaConfig
    dev = CudaDevice(rank)
    status = None
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            t[:] = torch.frombuffer(bytearray(comm_unique_id()), dtype=torch.uint8)
        dist.broadcast(t, 0)
        dev.comm_init(bytes(t.numpy().tobytes()), rank, world)
        status = dev.peer_status()
    dev.set_capture(True)
    cfg = LlamaConfig(**CFG, quant=QuantFormat.Int4, tp_rank=rank, tp_world=world)
    model = Llama(dev, cfg)
    try:
        model.init_random(seed=41, std=0.02)
        T = cfg.prefill_len
        out = [model.step(PREFILL, ids_seq[0], np.arange(T, dtype=np.uint32), T, 0)]
        launches = []
        for s in range(1, STEPS + 1):
            past = T + s - 1
            before = dev.launch_count()
            out.append(model.step(DECODE, ids_seq[s], np.array([past], np.uint32), 1, past))
            launches.append(dev.launch_count() - before)
        stats = dev.decode_fusion_stats()
    finally:
        model.close()
        dev.close()
    return out, launches, stats, status


def _rank_main(rank, world, port, ids_seq, q):
    import datetime

    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        res = _run(rank, world, ids_seq)
        if rank == 0:
            q.put(res)
    except Exception as e:  # reported to the parent, which fails the test
        q.put(repr(e))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_fused_decode_layers_match_single_gpu(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ids_seq = _ids()
    single, single_launches, single_stats, _ = _run(0, 1, ids_seq)
    assert single_stats["launched"] > 0  # the reference run is the fused kernel too
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, ids_seq, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=540)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(res, str), res
    assert all(p.exitcode == 0 for p in procs)
    tp, launches, stats, status = res
    assert status == {"peer_allreduce": True, "decode_fusion": True}, status
    assert stats["launched"] > 0 and stats["refused"] == 0, stats
    # Replayed steps: gather, the fused layers, final norm, last token,
    # vocabulary projection, logits all-gather.
    assert max(launches[2:]) <= 8, launches
    assert len(tp) == len(single)
    for a, b in zip(tp, single):
        assert a.shape == b.shape
        assert_reduction(a.ravel(), b.ravel())
