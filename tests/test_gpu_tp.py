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


# AllReduce(p) -> Add(x, p) -> RmsNorm: (rows, hidden, norm output reuses the
# residual's bytes). The last case has more rows than the peer exchange holds.
FUSED_CASES = [(1, 4096, True), (2, 512, False), (5, 1024, False), (3, 768, True),
               (40, 256, False)]


def _fused_expected_launches(rows, reuse):
    if reuse and rows > 1:
        return 2  # NCCL, then Add + RmsNorm fused (the output takes the input's bytes exactly)
    return 1 if rows <= 32 else 2  # peer-memory kernel, or NCCL + fused Add/RmsNorm


def _fused_rank(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    from oracle.pyoracle import Lcg
    from starlight_b200.device import BufferRef, CudaDevice, Op, OpCode, Value, comm_unique_id
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        dev = CudaDevice(rank)
        t = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            t[:] = torch.frombuffer(bytearray(comm_unique_id()), dtype=torch.uint8)
        dist.broadcast(t, 0)
        dev.comm_init(bytes(t.numpy().tobytes()), rank, world)
        F = Value.f32
        bufs = []
        for rows, hidden, reuse in FUSED_CASES:
            n = rows * hidden
            p0 = Lcg(100 * rows + hidden + rank).normal(n, 0.0, 1.0)
            x0 = Lcg(7 * rows + hidden).normal(n, 0.0, 1.0)
            w0 = Lcg(hidden).normal(hidden, 1.0, 0.1)
            init = np.zeros(4 * n + hidden, np.float32)
            init[:n], init[n:2 * n], init[4 * n:] = p0, x0, w0
            bufs.append((dev.allocate_f32(init.size), init))

        def run_case(ci):
            rows, hidden, reuse = FUSED_CASES[ci]
            n = rows * hidden
            ar, init = bufs[ci]
            dev.upload_f32(ar, init)
            dev.synchronize()
            p, x, s = BufferRef(ar, 0, n), BufferRef(ar, n, n), BufferRef(ar, 2 * n, n)
            o = BufferRef(ar, n, n) if reuse else BufferRef(ar, 3 * n, n)
            w = BufferRef(ar, 4 * n, hidden)
            shape = (rows, hidden)
            before = dev.launch_count()
            dev.dispatch(Op(OpCode.AllReduce), [p], [F(shape)], [], [])
            dev.dispatch(Op(OpCode.Add), [x, p], [F(shape), F(shape)], [s], [F(shape)])
            dev.dispatch(Op(OpCode.RmsNorm, eps=1e-5), [s, w], [F(shape), F((hidden,))], [o],
                         [F(shape)])
            dev.synchronize()
            launches = dev.launch_count() - before
            return dev.download_f32(ar)[:4 * n], launches

        eager = [run_case(ci) for ci in range(len(FUSED_CASES))]
        dev.set_capture(True)
        fused = [[run_case(ci) for ci in range(len(FUSED_CASES))] for _ in range(3)]
        dev.close()
        q.put((rank, eager, fused))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_add_rms_norm_matches_commands(world):
    # With capture on, the all-reduce and the Add + RmsNorm after it go out as
    # one peer-memory kernel, over repeated calls (the kernel's per-row epochs
    # and alternating slots). It sums the partials in rank order, so its bytes
    # are the same on every rank; at two ranks that sum is NCCL's, so every
    # byte (all-reduced partial, sum, normalised row) equals the
    # command-by-command run, while with more ranks NCCL adds in another order
    # and the two agree to a few ulps.
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (e, f)) for r, e, f in (q.get(timeout=240) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r][0], str), res[r][0]
    assert all(p.exitcode == 0 for p in procs)
    for r in range(world):
        eager, fused = res[r]
        for ci, (rows, hidden, reuse) in enumerate(FUSED_CASES):
            np.testing.assert_array_equal(eager[ci][0], res[0][0][ci][0])
            for rep in range(3):
                got, launches = fused[rep][ci]
                np.testing.assert_array_equal(got, res[0][1][rep][ci][0])
                if world == 2:
                    np.testing.assert_array_equal(got, eager[ci][0])
                else:
                    np.testing.assert_allclose(got, eager[ci][0], rtol=1e-5, atol=1e-5)
                if rep > 0:
                    assert launches == _fused_expected_launches(rows, reuse), (rows, reuse)


# ---- failure detection -----------------------------------------------------------

def _skip_rank(rank, world, port, q):
    # Both ranks run AllReduce -> Add -> RmsNorm (one row) three times under
    # capture (the peer-memory kernel); then rank 1 skips one call. Rank 0's
    # kernel waits for rank 1's flag at most 1 s, records the timeout in the
    # device error word and returns: slc_synchronize reports it, and nothing
    # is left waiting on the GPU (no NCCL call is involved).
    import datetime
    import time

    import torch
    import torch.distributed as dist
    from oracle.pyoracle import Lcg
    from starlight_b200.device import (BufferRef, CudaDevice, DeviceError, Op, OpCode, Value,
                                       comm_unique_id)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    err = None
    try:
        dev = CudaDevice(rank)
        t = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            t[:] = torch.frombuffer(bytearray(comm_unique_id()), dtype=torch.uint8)
        dist.broadcast(t, 0)
        dev.comm_init(bytes(t.numpy().tobytes()), rank, world)
        assert dev.peer_status()["peer_allreduce"]
        dev.set_capture(True)
        H, F = 4096, Value.f32
        buf = dev.allocate_f32(4 * H + H)
        init = np.concatenate([Lcg(5 + rank).normal(H, 0.0, 1.0), Lcg(6).normal(H, 0.0, 1.0),
                               np.zeros(2 * H, np.float32), Lcg(7).normal(H, 1.0, 0.1)])

        def call():
            dev.upload_f32(buf, init.astype(np.float32))
            p, x = BufferRef(buf, 0, H), BufferRef(buf, H, H)
            s, o, w = BufferRef(buf, 2 * H, H), BufferRef(buf, 3 * H, H), BufferRef(buf, 4 * H, H)
            dev.dispatch(Op(OpCode.AllReduce), [p], [F((1, H))], [], [])
            dev.dispatch(Op(OpCode.Add), [x, p], [F((1, H)), F((1, H))], [s], [F((1, H))])
            dev.dispatch(Op(OpCode.RmsNorm, eps=1e-5), [s, w], [F((1, H)), F((H,))], [o],
                         [F((1, H))])
            dev.synchronize()

        for _ in range(3):
            call()
        dist.barrier()
        if rank == 0:
            t0 = time.time()
            try:
                call()
            except DeviceError as e:
                err = (str(e), time.time() - t0)
        dev.close()
        q.put((rank, err))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "exception " + repr(e)))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_fused_allreduce_bounded_wait_reports_timeout():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skip_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), res
    assert res[1] is None, res
    assert res[0] is not None and "bounded wait timed out" in res[0][0], res
    assert res[0][1] < 10.0, res


def _leave_rank(rank, world, port, q):
    # Rank 1 leaves between steps (after one NCCL all-reduce both ranks ran).
    # Rank 0 learns it on the host before its next step (RankWatch), aborts
    # its communicator, and a collective it dispatches afterwards fails at
    # once instead of waiting for the missing rank.
    import datetime

    import torch
    import torch.distributed as dist
    from starlight_b200.device import BufferRef, CudaDevice, DeviceError, Op, OpCode, Value
    from starlight_b200.device import comm_unique_id
    from starlight_b200.health import RankFailure, RankWatch
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=60))
    watch = RankWatch(store, rank, world, timeout_s=1.0)
    out = None
    try:
        dev = CudaDevice(rank)
        if rank == 0:
            store.set("uid", bytes(comm_unique_id()))
        uid = store.get("uid")
        dev.comm_init(uid, rank, world)
        buf = dev.allocate_f32(1024)
        dev.upload_f32(buf, np.full(1024, rank + 1.0, np.float32))
        watch.step(0)
        dev.dispatch(Op(OpCode.AllReduce), [BufferRef(buf, 0, 1024)], [Value.f32((1, 1024))],
                     [], [])
        dev.synchronize()
        summed = dev.download_f32(buf)
        if rank == 1:
            dev.close()
            q.put((rank, float(summed[0]), None))
            return
        failure = None
        try:
            watch.step(1)
        except RankFailure as e:
            failure = (e.step, e.missing)
        dev.comm_abort()
        after = None
        try:
            dev.dispatch(Op(OpCode.AllReduce), [BufferRef(buf, 0, 1024)],
                         [Value.f32((1, 1024))], [], [])
            dev.synchronize()
        except DeviceError as e:
            after = str(e)
        checked = None
        try:
            dev.comm_check()
        except DeviceError as e:
            checked = str(e)
        dev.close()
        out = (failure, after is not None, checked is not None)
        q.put((rank, float(summed[0]), out))
    except Exception as e:
        q.put((rank, None, "exception " + repr(e)))
        raise
    finally:
        if rank == 0:
            import time
            time.sleep(0.5)


@pytest.mark.timeout(300)
def test_rank_leaving_between_steps_is_detected_and_comm_aborted():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leave_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (s, o)) for r, s, o in (q.get(timeout=240) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), res
    assert res[1] == (3.0, None), res  # 1 + 2 on both ranks
    assert res[0][0] == 3.0, res
    failure, dispatch_failed, check_failed = res[0][1]
    assert failure == (1, [1]), res
    assert dispatch_failed and check_failed, res
