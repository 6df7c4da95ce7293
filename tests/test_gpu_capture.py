"""Command capture and CUDA-graph replay (slc_set_capture): a captured and
replayed command sequence gives the results of eager execution (bit for bit
where the same kernels run; within the matmul tolerance where consecutive
MatMulNT commands on one input were grouped into one GEMV launch, which
changes the split-K summation order), with only past_len / seq_len changing
between replays; replays of one graph are bit-identical; validation errors
are still returned by slc_dispatch; cached graphs are dropped when a buffer
is released."""
import math

import numpy as np
import pytest

from oracle.pyoracle import Lcg
from starlight_b200.device import (CudaDevice, DeviceError, DType, Op, OpCode, QuantFormat, Status,
                                   Value, ValueRole)
from starlight_b200.engine import DECODE, PREFILL, Llama, LlamaConfig
from oracle import pyoracle as orc
from tests.gpu_util import assert_reduction, get, new_f32, put_f32, put_quant

pytestmark = pytest.mark.gpu

F = Value.f32


def small_8b_like(batch=1):
    # Shapes that take the TMA GEMV (K a multiple of 512) and the decode
    # attention kernel (head_dim 128, GQA 2:1).
    return LlamaConfig(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024,
                       vocab=2048, batch=batch, prefill_len=16, max_seq=48, eps=1e-5,
                       theta=500000.0, quant=QuantFormat.Int4, group_size=128)


def run_model(capture: bool, cfg, steps=8):
    dev = CudaDevice(0)
    if capture:
        dev.set_capture(True)
    model = Llama(dev, cfg)
    model.init_random(seed=21, std=0.02)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, cfg.vocab, size=cfg.batch * cfg.prefill_len, dtype=np.uint32)
    pos = np.tile(np.arange(cfg.prefill_len, dtype=np.uint32), cfg.batch)
    out = [model.step(PREFILL, prompt, pos, cfg.prefill_len, 0)]
    ids = out[-1].argmax(axis=1).astype(np.uint32)
    past = cfg.prefill_len
    for _ in range(steps):
        out.append(model.step(DECODE, ids, np.full(cfg.batch, past, np.uint32), 1, past))
        ids = out[-1].argmax(axis=1).astype(np.uint32)
        past += 1
    stats = dev.capture_stats() if capture else None
    model.close()
    dev.close()
    return out, stats


@pytest.mark.parametrize("batch", [1, 3])
def test_engine_steps_with_capture_equal_eager(batch):
    cfg = small_8b_like(batch)
    eager, _ = run_model(False, cfg)
    captured, stats = run_model(True, cfg)
    for a, b in zip(eager, captured):
        assert_reduction(b.ravel(), a.ravel())  # q/k/v grouped under capture
    # Prefill once (eager); decode: eager, captured, then replayed.
    assert stats["captures"] == 1
    assert stats["replays"] == 8 - 2


def test_fixture_with_capture_equal_eager():
    cfg = LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=4, head_dim=64, inter=688,
                      vocab=1024, batch=1, prefill_len=16, max_seq=32, eps=1e-5, theta=10000.0,
                      quant=QuantFormat.Int4, group_size=32)
    eager, _ = run_model(False, cfg, steps=10)
    captured, stats = run_model(True, cfg, steps=10)
    for a, b in zip(eager, captured):
        assert np.array_equal(a, b)
    assert stats["replays"] == 10 - 2


def _attention_segment(dev, bufs, past):
    q, k, v, cache, out = bufs
    s = dict(batch=1, layers=2, max_seq=40, kv_heads=2, head_dim=128)
    st = Value(DType.F32, (1, 2, 2, 40, 2, 128), ValueRole.State)
    op = Op(OpCode.CausalAttention, layer=1, heads=8, kv_heads=2, head_dim=128,
            scale=float(np.float32(1 / math.sqrt(128))))
    dev.dispatch(op, [q, k, v, cache], [F((1, 8, 1, 128)), F((1, 2, 1, 128)),
                                        F((1, 2, 1, 128)), st], [out], [F((1, 8, 1, 128))],
                 [past])
    return s


def test_replay_reads_new_past_len_each_time():
    lcg = Lcg(9)
    cache0 = lcg.fill(2 * 2 * 40 * 2 * 128, -1, 1)
    qs = [lcg.fill(8 * 128, -1, 1) for _ in range(6)]
    ks = [lcg.fill(2 * 128, -1, 1) for _ in range(6)]
    results = []
    for capture in (False, True):
        dev = CudaDevice(0)
        if capture:
            dev.set_capture(True)
        cache = put_f32(dev, cache0)
        q, k, v = new_f32(dev, 8 * 128), new_f32(dev, 2 * 128), new_f32(dev, 2 * 128)
        out = new_f32(dev, 8 * 128)
        outs = []
        for i, past in enumerate([3, 4, 5, 20, 21, 39]):
            dev.upload_f32(q.buffer, qs[i])
            dev.upload_f32(k.buffer, ks[i])
            dev.upload_f32(v.buffer, ks[(i + 1) % 6])
            _attention_segment(dev, (q, k, v, cache, out), past)
            outs.append((get(dev, out).copy(), get(dev, cache).copy()))
        if capture:
            st = dev.capture_stats()
            assert st["captures"] == 1 and st["replays"] == 4
        results.append(outs)
        dev.close()
    for (o1, c1), (o2, c2) in zip(*results):
        assert np.array_equal(o1, o2) and np.array_equal(c1, c2)


def test_errors_are_reported_by_dispatch_under_capture():
    dev = CudaDevice(0)
    dev.set_capture(True)
    cache = put_f32(dev, np.zeros(2 * 2 * 40 * 2 * 128, np.float32))
    bufs = (new_f32(dev, 8 * 128), new_f32(dev, 2 * 128), new_f32(dev, 2 * 128), cache,
            new_f32(dev, 8 * 128))
    with pytest.raises(DeviceError) as e:
        _attention_segment(dev, bufs, 40)  # past_len + seq > max_seq
    assert e.value.status == Status.Execution
    assert e.value.message == "past_len + seq exceeds max_seq"
    dev.synchronize()
    assert np.all(get(dev, cache) == 0)  # nothing ran
    dev.close()


def test_release_drops_graphs_and_results_stay_right():
    dev = CudaDevice(0)
    dev.set_capture(True)
    a, b = put_f32(dev, np.arange(1024, dtype=np.float32)), put_f32(dev, np.ones(1024, np.float32))
    out = new_f32(dev, 1024)
    spare = new_f32(dev, 16)
    for i in range(5):
        dev.dispatch(Op(OpCode.Add), [a, b], [F((1024,)), F((1024,))], [out], [F((1024,))])
        assert np.array_equal(get(dev, out), np.arange(1024, dtype=np.float32) + 1)
        if i == 2:
            dev.release(spare.buffer)
    st = dev.capture_stats()
    # run 1 eager, 2 captured, 3 replayed; the release drops the graph, so run
    # 4 (a key already seen) is captured again and run 5 replays it.
    assert st["captures"] == 2 and st["replays"] == 2
    dev.close()


def test_grouped_matmuls_under_capture():
    # q/k/v-like: three MatMulNT commands on one input become one grouped
    # GEMV launch; every run matches the oracle, replays are bit-identical.
    dev = CudaDevice(0)
    dev.set_capture(True)
    lcg = Lcg(44)
    k, m = 1024, 2
    x = lcg.fill(m * k, -1, 1)
    xr = put_f32(dev, x)
    mats, outs, wants = [], [], []
    for n in (512, 256, 256):
        w = lcg.normal(n * k, 0, 0.05)
        codes, scales = orc.quantize(orc.INT4, w, n, k, 128)
        cb, _, words = put_quant(dev, codes, scales, QuantFormat.Int4, 128)
        mats.append((cb, words, n))
        outs.append(new_f32(dev, m * n))
        wd = orc.dequantize(orc.INT4, codes, scales, n, k, 128).reshape(n, k)
        wants.append((x.reshape(m, k).astype(np.float64) @ wd.astype(np.float64).T).ravel())
    from starlight_b200.device import BufferRef
    runs = []
    for _ in range(4):
        for (cb, words, n), out in zip(mats, outs):
            dev.dispatch(Op(OpCode.MatMulNT), [xr, BufferRef(cb, 0, words)],
                         [F((m, k)), Value.quantized((n, k), QuantFormat.Int4, 128)], [out],
                         [F((m, n))])
        got = [get(dev, o).copy() for o in outs]
        for g_, w_ in zip(got, wants):
            assert_reduction(g_, w_)
        runs.append(got)
    for a, b in zip(runs[2], runs[3]):
        assert np.array_equal(a, b)
    st = dev.capture_stats()
    assert st["captures"] == 1 and st["replays"] == 2
    dev.close()



@pytest.mark.parametrize("heads,kv_heads,head_dim,batch", [(4, 4, 64, 1), (8, 2, 128, 1),
                                                           (4, 1, 128, 2)])
def test_fused_decode_attention_block_matches_commands(heads, kv_heads, head_dim, batch):
    # With capture on, the decode command run SplitHeads x3 -> Rope x2 ->
    # CausalAttention -> MergeHeads goes out as the fused two-launch block.
    # Every byte of the buffers it writes and the KV cache must equal the
    # command-by-command results, also where outputs reuse the bytes of dead
    # values as the engine's memory plan does: ks over q, vs over k, kr over
    # qs, am over qr (each command's own inputs and outputs stay disjoint).
    from starlight_b200.device import BufferRef
    B, H, Hkv, D, L, S, past = batch, heads, kv_heads, head_dim, 2, 40, 17
    lcg = Lcg(heads * 7 + head_dim)
    nq, nk = B * H * D, B * Hkv * D
    q0 = lcg.normal(nq, 0.0, 1.0)
    k0 = lcg.normal(nk, 0.0, 1.0)
    v0 = lcg.normal(nk, 0.0, 1.0)
    cache0 = lcg.normal(B * L * 2 * S * Hkv * D, 0.0, 1.0)
    pos = np.full(B, past, np.uint32)
    Q0 = nq + 2 * nk          # qs
    Q1 = Q0 + nq              # qr
    A = Q1 + nq               # a
    total = A + nq
    arena0 = np.zeros(total, np.float32)
    arena0[0:nq] = q0
    arena0[nq:nq + nk] = k0
    arena0[nq + nk:nq + 2 * nk] = v0

    def run(capture):
        dev = CudaDevice(0)
        if capture:
            dev.set_capture(True)
        ar = dev.allocate_f32(total)
        cache = dev.allocate_f32(cache0.size)
        pb = dev.allocate_u32(B)
        dev.upload_u32(pb, pos)
        R = lambda o, n: BufferRef(ar, o, n)
        q, k, v = R(0, nq), R(nq, nk), R(nq + nk, nk)
        qs, qr, a = R(Q0, nq), R(Q1, nq), R(A, nq)
        ks, vs, kr, am = R(0, nk), R(nq, nk), R(Q0, nk), R(Q1, nq)
        pref, cref = BufferRef(pb, 0, B), BufferRef(cache, 0, cache0.size)
        st = Value(DType.F32, (B, L, 2, S, Hkv, D), ValueRole.State)
        sq = Op(OpCode.SplitHeads, heads=H, head_dim=D)
        skv = Op(OpCode.SplitHeads, heads=Hkv, head_dim=D)
        rope = Op(OpCode.Rope, theta=10000.0)
        att = Op(OpCode.CausalAttention, layer=1, heads=H, kv_heads=Hkv, head_dim=D,
                 scale=1.0 / math.sqrt(D))
        mh = Op(OpCode.MergeHeads, heads=H, head_dim=D)
        results = []
        for _ in range(3 if capture else 1):  # eager run, capture, replay
            dev.upload_f32(ar, arena0)
            dev.upload_f32(cache, cache0)
            dev.dispatch(sq, [q], [F((B, 1, H * D))], [qs], [F((B, H, 1, D))])
            dev.dispatch(skv, [k], [F((B, 1, Hkv * D))], [ks], [F((B, Hkv, 1, D))])
            dev.dispatch(skv, [v], [F((B, 1, Hkv * D))], [vs], [F((B, Hkv, 1, D))])
            dev.dispatch(rope, [qs, pref], [F((B, H, 1, D)), Value.u32((B, 1))], [qr],
                         [F((B, H, 1, D))])
            dev.dispatch(rope, [ks, pref], [F((B, Hkv, 1, D)), Value.u32((B, 1))], [kr],
                         [F((B, Hkv, 1, D))])
            dev.dispatch(att, [qr, kr, vs, cref],
                         [F((B, H, 1, D)), F((B, Hkv, 1, D)), F((B, Hkv, 1, D)), st], [a],
                         [F((B, H, 1, D))], scalars=[past])
            dev.dispatch(mh, [a], [F((B, H, 1, D))], [am], [F((B, 1, H * D))])
            dev.synchronize()
            results.append((get(dev, R(0, total)), get(dev, cref)))
        stats = dev.capture_stats() if capture else None
        dev.close()
        return results, stats

    (eager,), _ = run(False)
    fused, stats = run(True)
    assert stats["replays"] >= 1
    for arena, cache in fused:
        np.testing.assert_array_equal(arena, eager[0])
        np.testing.assert_array_equal(cache, eager[1])


@pytest.mark.parametrize("rows,hidden,reuse", [(1, 4096, True), (1, 256, True), (3, 4096, False),
                                               (5, 1024, True), (8, 4096, True)])
def test_fused_add_rms_norm_matches_commands(rows, hidden, reuse):
    # Add(a, b) -> s then RmsNorm(s) -> o goes out as one launch with capture
    # on. With reuse the norm's output takes exactly the bytes of the dead
    # addend a (each CTA reads its row before writing the same row): every
    # byte must equal command-by-command execution.
    from starlight_b200.device import BufferRef
    lcg = Lcg(rows * 13 + hidden)
    n = rows * hidden
    a0, b0 = lcg.normal(n, 0.0, 1.0), lcg.normal(n, 0.0, 1.0)
    w0 = lcg.normal(hidden, 1.0, 0.1)
    total = 4 * n

    def run(capture):
        dev = CudaDevice(0)
        if capture:
            dev.set_capture(True)
        ar = dev.allocate_f32(total)
        wb = dev.allocate_f32(hidden)
        dev.upload_f32(wb, w0)
        a, b, s = BufferRef(ar, 0, n), BufferRef(ar, n, n), BufferRef(ar, 2 * n, n)
        o = BufferRef(ar, 0, n) if reuse else BufferRef(ar, 3 * n, n)
        init = np.zeros(total, np.float32)
        init[:n], init[n:2 * n] = a0, b0
        shape = (rows, hidden)
        outs = []
        for _ in range(3 if capture else 1):
            dev.upload_f32(ar, init)
            dev.dispatch(Op(OpCode.Add), [a, b], [F(shape), F(shape)], [s], [F(shape)])
            dev.dispatch(Op(OpCode.RmsNorm, eps=1e-5), [s, BufferRef(wb, 0, hidden)],
                         [F(shape), F((hidden,))], [o], [F(shape)])
            dev.synchronize()
            outs.append(get(dev, BufferRef(ar, 0, total)))
        dev.close()
        return outs

    (eager,) = run(False)
    for got in run(True):
        np.testing.assert_array_equal(got, eager)
