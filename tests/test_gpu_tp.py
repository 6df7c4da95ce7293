"""Tensor parallelism on two GPUs (one process per GPU, NCCL over NVLink):
the llama-dense model split 2 ways (q/k/v/gate/up/lm_head by rows, o/down by
columns, all-reduce after o and down, all-gather of the logits) gives the
single-GPU logits within the matmul tolerance, prefill and decode, with and
without graph capture. The same token ids are fed to both runs (teacher
forcing), so a near-tie cannot make them diverge. Skipped with fewer than
two GPUs."""
import os
import socket

import numpy as np
import pytest

from tests.gpu_util import assert_reduction

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, hidden=512, heads=8, kv_heads=4, head_dim=128, inter=1024, vocab=2048,
           batch=2, prefill_len=16, max_seq=40, eps=1e-5, theta=500000.0, group_size=128)
STEPS = 6


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, capture, ids_seq):
    from starlight_b200.device import CudaDevice, QuantFormat, comm_unique_id
    from starlight_b200.engine import DECODE, PREFILL, Llama, LlamaConfig
    dev = CudaDevice(rank)
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            t[:] = torch.frombuffer(bytearray(comm_unique_id()), dtype=torch.uint8)
        dist.broadcast(t, 0)
        dev.comm_init(bytes(t.numpy().tobytes()), rank, world)
    if capture:
        dev.set_capture(True)
    cfg = LlamaConfig(**CFG, quant=QuantFormat.Int4, tp_rank=rank, tp_world=world)
    model = Llama(dev, cfg)
    model.init_random(seed=33, std=0.02)
    B, T = cfg.batch, cfg.prefill_len
    pos = np.tile(np.arange(T, dtype=np.uint32), B)
    out = [model.step(PREFILL, ids_seq[0], pos, T, 0)]
    for s in range(1, STEPS + 1):
        past = T + s - 1
        out.append(model.step(DECODE, ids_seq[s], np.full(B, past, np.uint32), 1, past))
    model.close()
    dev.close()
    return out


def _rank_main(rank, world, port, capture, ids_seq, q):
    import datetime

    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        out = _run(rank, world, capture, ids_seq)
        if rank == 0:
            q.put(out)
    except Exception as e:  # reported to the parent, which fails the test
        q.put(repr(e))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _reference_ids():
    rng = np.random.default_rng(17)
    B, T = CFG["batch"], CFG["prefill_len"]
    seq = [rng.integers(0, CFG["vocab"], size=B * T, dtype=np.uint32)]
    for _ in range(STEPS):
        seq.append(rng.integers(0, CFG["vocab"], size=B, dtype=np.uint32))
    return seq


@pytest.mark.timeout(600)
@pytest.mark.parametrize("capture", [False, True])
def test_tp2_logits_match_single_gpu(capture):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ids_seq = _reference_ids()
    single = _run(0, 1, capture, ids_seq)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, capture, ids_seq, q)) for r in range(2)]
    for p in procs:
        p.start()
    tp = q.get(timeout=540)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(tp, str), tp
    assert all(p.exitcode == 0 for p in procs)
    assert len(tp) == len(single)
    for a, b in zip(tp, single):
        assert a.shape == b.shape
        assert_reduction(a.ravel(), b.ravel())
