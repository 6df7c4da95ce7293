"""GPU parity of every backend-cuda operator against the CPU oracle, through the
C ABI (`slc_dispatch`), following the CpuDevice device tests
(crates/backends/backend-cpu/src/device.rs:1490-2286): the same operator
signatures and shapes, compared with the restated reference kernels.
Tolerances are defined in tests/gpu_util.py."""
import math

import numpy as np
import pytest

from oracle import pyoracle as orc
from oracle.pyoracle import Lcg
from starlight_b200.device import (BufferRef, CudaDevice, DeviceError, Op, OpCode, QuantFormat,
                                   RopeVariant, Status, Value, ValueRole)
from tests.gpu_util import (assert_elementwise, assert_reduction, get, new_f32, put_f32,
                            put_quant, put_u32)

pytestmark = pytest.mark.gpu

F = Value.f32
T = ValueRole.Temp


@pytest.fixture(scope="module")
def dev():
    d = CudaDevice(0)
    yield d
    d.close()


def run1(dev, op, ins, in_vals, out_shape, scalars=()):
    n = int(np.prod(out_shape)) if len(out_shape) else 1
    out = new_f32(dev, n)
    dev.dispatch(op, ins, in_vals, [out], [F(out_shape)], scalars)
    return get(dev, out)


# ------------------------------------------------------------ elementwise --

@pytest.mark.parametrize("n", [1, 5, 33, 4096 * 3 + 1, 1 << 20])
def test_add_mul_scale_bit_exact(dev, n):
    lcg = Lcg(n)
    a, b = lcg.fill(n, -2, 2), lcg.fill(n, -2, 2)
    ra, rb = put_f32(dev, a), put_f32(dev, b)
    got = run1(dev, Op(OpCode.Add), [ra, rb], [F((n,)), F((n,))], (n,))
    assert np.array_equal(got, orc.add(a, b, n))
    got = run1(dev, Op(OpCode.Mul), [ra, rb], [F((n,)), F((n,))], (n,))
    assert np.array_equal(got, orc.mul(a, b, n))
    got = run1(dev, Op(OpCode.Scale, factor=-1.5), [ra], [F((n,))], (n,))
    assert np.array_equal(got, orc.scale(a, -1.5))


@pytest.mark.parametrize("rows,cols,offset", [(1, 1, 0), (3, 5, 0), (16, 4096, 0), (7, 4096, 1),
                                              (256, 4096, 0)])
def test_add_bias_bit_exact(dev, rows, cols, offset):
    # Extension op (BASELINE configs[1] residual add plus broadcast bias):
    # (a + b) + bias[col], each sum rounded as f32; an element offset of 1
    # takes the scalar path.
    lcg = Lcg(rows * 7 + cols)
    a, b = lcg.fill(rows * cols, -2, 2), lcg.fill(rows * cols, -2, 2)
    bias = lcg.fill(cols, -1, 1)
    abuf = put_f32(dev, np.concatenate([np.zeros(offset, np.float32), a]))
    ra = BufferRef(abuf.buffer, offset, rows * cols)
    got = run1(dev, Op(OpCode.AddBias), [ra, put_f32(dev, b), put_f32(dev, bias)],
               [F((rows, cols)), F((rows, cols)), F((cols,), ValueRole.Param)], (rows, cols))
    want = ((a.reshape(rows, cols) + b.reshape(rows, cols)).astype(np.float32) + bias).ravel()
    assert np.array_equal(got, want.astype(np.float32))


def test_add_bias_rejects_a_bias_of_the_wrong_length(dev):
    a, b = put_f32(dev, np.zeros(8, np.float32)), put_f32(dev, np.zeros(8, np.float32))
    with pytest.raises(DeviceError, match="bias must have shape"):
        run1(dev, Op(OpCode.AddBias), [a, b, put_f32(dev, np.zeros(3, np.float32))],
             [F((2, 4)), F((2, 4)), F((3,))], (2, 4))


@pytest.mark.parametrize("n", [1, 7, 33, 1 << 18])
def test_silu(dev, n):
    x = Lcg(n + 1).fill(n, -8, 8)
    got = run1(dev, Op(OpCode.Silu), [put_f32(dev, x)], [F((n,))], (n,))
    assert_elementwise(got, orc.silu(x))
    ext = np.array([-100, -10, 0, 10, 100], np.float32)
    got = run1(dev, Op(OpCode.Silu), [put_f32(dev, ext)], [F((5,))], (5,))
    assert_elementwise(got, orc.silu(ext))


def test_unaligned_offsets_take_the_scalar_path(dev):
    # An element offset of 1 breaks 16-byte alignment of the vector path.
    a = Lcg(3).fill(1025, -1, 1)
    buf = put_f32(dev, a)
    ref = BufferRef(buf.buffer, 1, 1024)
    got = run1(dev, Op(OpCode.Add), [ref, put_f32(dev, a[1:])], [F((1024,)), F((1024,))], (1024,))
    assert np.array_equal(got, orc.add(a[1:], a[1:], 1024))


# ------------------------------------------------------------------ norm ----

@pytest.mark.parametrize("rows,hidden,eps,seed", [(1, 1, 1e-5, 1), (3, 7, 1e-6, 2), (4, 16, 1e-5, 3),
                                                  (2, 33, 1e-6, 4), (1, 4096, 1e-5, 5),
                                                  (256, 4096, 1e-5, 6), (300, 256, 1e-5, 7),
                                                  (3, 8192, 1e-5, 8), (2, 10000, 1e-5, 9)])
def test_rms_norm(dev, rows, hidden, eps, seed):
    lcg = Lcg(seed)
    x, w = lcg.fill(rows * hidden, -2, 2), lcg.fill(hidden, 0.5, 1.5)
    got = run1(dev, Op(OpCode.RmsNorm, eps=eps), [put_f32(dev, x), put_f32(dev, w)],
               [F((rows, hidden)), F((hidden,), ValueRole.Param)], (rows, hidden))
    assert_reduction(got, orc.rms_norm(x, w, rows, hidden, eps))


# --------------------------------------------------------------- softmax ----

@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (6, 17), (64, 2048), (5, 4100), (8, 128)])
def test_softmax(dev, rows, cols):
    x = Lcg(rows * 7 + cols).fill(rows * cols, -4, 4)
    got = run1(dev, Op(OpCode.Softmax), [put_f32(dev, x)], [F((rows, cols))], (rows, cols))
    assert_reduction(got, orc.softmax(x, rows, cols))


def test_softmax_extreme_values(dev):
    x = np.array([1000.0, 999.0, -1000.0, 0.0], np.float32)
    got = run1(dev, Op(OpCode.Softmax), [put_f32(dev, x)], [F((2, 2))], (2, 2))
    assert np.all(np.isfinite(got))
    assert_reduction(got, orc.softmax(x, 2, 2))


@pytest.mark.parametrize("rows,seq,past", [(2, 2, 0), (12, 4, 1), (4, 1, 7), (6, 3, 2), (64, 16, 48)])
def test_softmax_causal(dev, rows, seq, past):
    cols = past + seq
    x = Lcg(rows + seq + past).fill(rows * cols, -3, 3)
    got = run1(dev, Op(OpCode.SoftmaxCausal), [put_f32(dev, x)], [F((rows, cols))], (rows, cols),
               scalars=[seq, past])
    assert_reduction(got, orc.softmax_causal(x, rows, cols, seq, past))


# ------------------------------------------------------------------ rope ----

@pytest.mark.parametrize("variant", ["neox", "gptj"])
@pytest.mark.parametrize("shape", [(1, 1, 1, 2, 10000.0), (2, 3, 5, 4, 10000.0), (2, 2, 4, 8, 500000.0),
                                   (1, 2, 3, 10, 1000000.0), (1, 32, 64, 128, 500000.0),
                                   (2, 8, 3, 128, 500000.0)])
def test_rope(dev, variant, shape):
    b, h, s, hd, theta = shape
    lcg = Lcg(b * 100 + h * 10 + s)
    x = lcg.fill(b * h * s * hd, -2, 2)
    pos = np.array([3 + i * 2 + lcg.below(5) for i in range(b * s)], np.uint32)
    v = RopeVariant.Neox if variant == "neox" else RopeVariant.GptJ
    got = run1(dev, Op(OpCode.Rope, theta=theta, variant=v), [put_f32(dev, x), put_u32(dev, pos)],
               [F((b, h, s, hd)), Value.u32((b, s))], (b, h, s, hd))
    assert_elementwise(got, orc.rope(x, pos, b, h, s, hd, theta, variant))


def test_rope_large_positions(dev):
    # T up to 16384 with theta 5e5: the f64 angle keeps the 1e-5 bound.
    t, h, hd = 16384, 2, 128
    x = Lcg(11).fill(t * h * hd, -1, 1)
    pos = np.arange(t, dtype=np.uint32)
    got = run1(dev, Op(OpCode.Rope, theta=500000.0), [put_f32(dev, x), put_u32(dev, pos)],
               [F((1, h, t, hd)), Value.u32((1, t))], (1, h, t, hd))
    assert_elementwise(got, orc.rope(x, pos, 1, h, t, hd, 500000.0))


def test_rope_rank3_input(dev):
    b, s, hd = 2, 3, 8
    x = Lcg(5).fill(b * s * hd, -1, 1)
    pos = np.arange(b * s, dtype=np.uint32)
    got = run1(dev, Op(OpCode.Rope, theta=10000.0), [put_f32(dev, x), put_u32(dev, pos)],
               [F((b, s, hd)), Value.u32((b, s))], (b, s, hd))
    assert_elementwise(got, orc.rope(x, pos, b, 1, s, hd, 10000.0))


# ---------------------------------------------------------------- layout ----

@pytest.mark.parametrize("vocab,hidden,rows", [(10, 5, 3), (1, 1, 1), (4, 7, 0), (13, 9, 6),
                                               (1024, 256, 16), (128256, 64, 32)])
def test_gather_bit_exact(dev, vocab, hidden, rows):
    lcg = Lcg(vocab + rows)
    table = lcg.fill(vocab * hidden, -1, 1)
    ids = np.array([lcg.below(vocab) for _ in range(rows)], np.uint32)
    got = run1(dev, Op(OpCode.Gather), [put_f32(dev, table), put_u32(dev, ids)],
               [F((vocab, hidden), ValueRole.Param), Value.u32((1, rows))], (1, rows, hidden))
    assert np.array_equal(got, orc.gather(table, ids, vocab, hidden, rows))


def test_gather_rejects_bad_ids_before_writing(dev):
    table = put_f32(dev, [1, 2, 3, 4])
    out = new_f32(dev, 2, fill=0.0)
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Gather), [table, put_u32(dev, [4])],
                     [F((2, 2), ValueRole.Param), Value.u32((1,))], [out], [F((1, 2))])
    assert e.value.status == Status.Execution and e.value.message == "id out of range"
    assert np.array_equal(get(dev, out), np.zeros(2, np.float32))


@pytest.mark.parametrize("batch,seq,hidden,seq_len", [(1, 1, 3, 1), (3, 5, 4, 5), (2, 4, 7, 2),
                                                      (8, 16, 4096, 9)])
def test_last_token_bit_exact(dev, batch, seq, hidden, seq_len):
    x = Lcg(batch + seq).fill(batch * seq * hidden, -1, 1)
    got = run1(dev, Op(OpCode.LastToken), [put_f32(dev, x)], [F((batch, seq, hidden))],
               (batch, hidden), scalars=[seq_len])
    assert np.array_equal(got, orc.last_token(x, batch, seq, hidden, seq_len))


@pytest.mark.parametrize("shape", [(1, 1, 1, 2), (2, 3, 4, 4), (2, 5, 3, 6), (1, 4, 2, 8),
                                   (4, 17, 32, 128)])
def test_split_merge_heads_bit_exact(dev, shape):
    b, s, h, hd = shape
    x = Lcg(b * s + h).fill(b * s * h * hd, -1, 1)
    split = run1(dev, Op(OpCode.SplitHeads, heads=h, head_dim=hd), [put_f32(dev, x)],
                 [F((b, s, h * hd))], (b, h, s, hd))
    assert np.array_equal(split, orc.split_heads(x, b, s, h, hd))
    merged = run1(dev, Op(OpCode.MergeHeads, heads=h, head_dim=hd), [put_f32(dev, split)],
                  [F((b, h, s, hd))], (b, s, h * hd))
    assert np.array_equal(merged, x)


# ------------------------------------------------------------- attention ----

def state_value(s):
    from starlight_b200.device import DType
    return Value(DType.F32, (s["batch"], s["layers"], 2, s["max_seq"], s["kv_heads"], s["head_dim"]),
                 ValueRole.State)


KV_CASES = [
    (1, dict(batch=1, layers=1, layer=0, heads=1, kv_heads=1, seq=2, past_len=0, head_dim=2, max_seq=4)),
    (2, dict(batch=2, layers=2, layer=1, heads=2, kv_heads=2, seq=3, past_len=2, head_dim=3, max_seq=5)),
    (3, dict(batch=1, layers=1, layer=0, heads=2, kv_heads=2, seq=1, past_len=0, head_dim=8, max_seq=1)),
    (4, dict(batch=1, layers=1, layer=0, heads=1, kv_heads=1, seq=0, past_len=2, head_dim=4, max_seq=4)),
    (5, dict(batch=4, layers=3, layer=2, heads=8, kv_heads=8, seq=7, past_len=100, head_dim=128, max_seq=128)),
]

ATTN_CASES = [
    (11, dict(batch=1, layers=1, layer=0, heads=2, kv_heads=2, seq=3, past_len=0, head_dim=4, max_seq=4)),
    (12, dict(batch=2, layers=1, layer=0, heads=2, kv_heads=2, seq=1, past_len=3, head_dim=8, max_seq=6)),
    (13, dict(batch=2, layers=2, layer=1, heads=4, kv_heads=2, seq=2, past_len=2, head_dim=8, max_seq=5)),
    (14, dict(batch=2, layers=1, layer=0, heads=2, kv_heads=1, seq=1, past_len=5, head_dim=2, max_seq=7)),
    (15, dict(batch=1, layers=1, layer=0, heads=6, kv_heads=3, seq=2, past_len=1, head_dim=4, max_seq=4)),
    (16, dict(batch=1, layers=1, layer=0, heads=3, kv_heads=1, seq=1, past_len=2, head_dim=4, max_seq=3)),
    # 8B decode shape, GQA 4:1, long past (split-K with combine)
    (17, dict(batch=1, layers=2, layer=1, heads=32, kv_heads=8, seq=1, past_len=1279, head_dim=128, max_seq=1280)),
    (18, dict(batch=4, layers=1, layer=0, heads=32, kv_heads=8, seq=1, past_len=300, head_dim=128, max_seq=512)),
    # decode kernel (seq 1, head_dim 64/128, up to 8 query heads per KV head):
    # one key, one chunk, GQA 2/8, long pasts split over many chunks
    (21, dict(batch=1, layers=1, layer=0, heads=8, kv_heads=8, seq=1, past_len=0, head_dim=64, max_seq=4)),
    (22, dict(batch=3, layers=2, layer=0, heads=64, kv_heads=8, seq=1, past_len=777, head_dim=128, max_seq=800)),
    (23, dict(batch=1, layers=1, layer=0, heads=4, kv_heads=2, seq=1, past_len=17, head_dim=64, max_seq=20)),
    (24, dict(batch=2, layers=3, layer=2, heads=16, kv_heads=2, seq=1, past_len=2047, head_dim=128, max_seq=2048)),
    (25, dict(batch=1, layers=1, layer=0, heads=4, kv_heads=4, seq=1, past_len=63, head_dim=64, max_seq=64)),
    # prefill chunk with a past
    (19,dict(batch=1, layers=1, layer=0, heads=8, kv_heads=2, seq=40, past_len=9, head_dim=64, max_seq=64)),
    (20, dict(batch=2, layers=1, layer=0, heads=4, kv_heads=4, seq=33, past_len=0, head_dim=64, max_seq=40)),
]


def sizes(s):
    q = s["batch"] * s["heads"] * s["seq"] * s["head_dim"]
    kv = s["batch"] * s["kv_heads"] * s["seq"] * s["head_dim"]
    cache = s["batch"] * s["layers"] * 2 * s["max_seq"] * s["kv_heads"] * s["head_dim"]
    return q, kv, cache


@pytest.mark.parametrize("seed,s", KV_CASES)
def test_kv_append_bit_exact(dev, seed, s):
    _, kvl, cl = sizes(s)
    lcg = Lcg(seed)
    k, v, cache = lcg.fill(kvl, -1, 1), lcg.fill(kvl, -1, 1), lcg.fill(cl, -1, 1)
    cref = put_f32(dev, cache)
    kv_shape = (s["batch"], s["kv_heads"], s["seq"], s["head_dim"])
    dev.dispatch(Op(OpCode.KvAppend, layer=s["layer"]), [put_f32(dev, k), put_f32(dev, v), cref],
                 [F(kv_shape), F(kv_shape), state_value(s)], [], [], [s["past_len"]])
    want = orc.kv_append(k, v, cache, s["batch"], s["layers"], s["layer"], s["kv_heads"],
                         s["head_dim"], s["max_seq"], s["past_len"], s["seq"])
    assert np.array_equal(get(dev, cref), want)


def test_kv_append_documented_layout(dev):  # attention.rs:509-527
    cref = put_f32(dev, np.zeros(24))
    s = dict(batch=1, layers=2, max_seq=3, kv_heads=1, head_dim=2)
    dev.dispatch(Op(OpCode.KvAppend, layer=1), [put_f32(dev, [1, 2]), put_f32(dev, [3, 4]), cref],
                 [F((1, 1, 1, 2)), F((1, 1, 1, 2)), state_value(s)], [], [], [1])
    c = get(dev, cref)
    assert list(c[14:16]) == [1, 2] and list(c[20:22]) == [3, 4]
    assert np.count_nonzero(c) == 4


@pytest.mark.parametrize("seed,s", ATTN_CASES)
def test_causal_attention(dev, seed, s):
    ql, kvl, cl = sizes(s)
    lcg = Lcg(seed)
    q, k, v, cache = (lcg.fill(ql, -1, 1), lcg.fill(kvl, -1, 1), lcg.fill(kvl, -1, 1),
                      lcg.fill(cl, -1, 1))
    scale = float(np.float32(1.0 / math.sqrt(s["head_dim"])))
    cref = put_f32(dev, cache)
    q_shape = (s["batch"], s["heads"], s["seq"], s["head_dim"])
    kv_shape = (s["batch"], s["kv_heads"], s["seq"], s["head_dim"])
    op = Op(OpCode.CausalAttention, layer=s["layer"], heads=s["heads"], kv_heads=s["kv_heads"],
            head_dim=s["head_dim"], scale=scale)
    out = new_f32(dev, ql)
    dev.dispatch(op, [put_f32(dev, q), put_f32(dev, k), put_f32(dev, v), cref],
                 [F(q_shape), F(kv_shape), F(kv_shape), state_value(s)], [out], [F(q_shape)],
                 [s["past_len"]])
    want_out, want_cache = orc.causal_attention(q, k, v, cache, s["batch"], s["layers"], s["layer"],
                                                s["heads"], s["kv_heads"], s["seq"], s["past_len"],
                                                s["head_dim"], s["max_seq"], scale)
    assert np.array_equal(get(dev, cref), want_cache)
    assert_reduction(get(dev, out), want_out)


def test_causal_attention_hand_computed_decode(dev):  # attention.rs:529-542
    s = dict(batch=1, layers=1, max_seq=1, kv_heads=1, head_dim=2)
    out = new_f32(dev, 2)
    dev.dispatch(Op(OpCode.CausalAttention, layer=0, heads=1, kv_heads=1, head_dim=2, scale=1.0),
                 [put_f32(dev, [1, 0]), put_f32(dev, [1, 0]), put_f32(dev, [3, 4]),
                  put_f32(dev, np.zeros(4))],
                 [F((1, 1, 1, 2)), F((1, 1, 1, 2)), F((1, 1, 1, 2)), state_value(s)], [out],
                 [F((1, 1, 1, 2))], [0])
    assert_reduction(get(dev, out), [3.0, 4.0])


def test_attention_rejects_state_overflow(dev):
    s = dict(batch=1, layers=1, max_seq=3, kv_heads=2, head_dim=4)
    cref = put_f32(dev, np.full(48, 7.0))
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.CausalAttention, layer=0, heads=2, kv_heads=2, head_dim=4, scale=0.5),
                     [put_f32(dev, np.zeros(16)), put_f32(dev, np.zeros(16)), put_f32(dev, np.zeros(16)),
                      cref],
                     [F((1, 2, 2, 4)), F((1, 2, 2, 4)), F((1, 2, 2, 4)), state_value(s)],
                     [new_f32(dev, 16)], [F((1, 2, 2, 4))], [2])
    assert e.value.message == "past_len + seq exceeds max_seq"
    assert np.all(get(dev, cref) == 7.0)


# ---------------------------------------------------------------- matmul ----

@pytest.mark.parametrize("nt", [True, False])
@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (2, 3, 5, 7), (2, 4, 9, 6), (1, 16, 256, 1024),
                                   (1, 70, 300, 129)])
def test_matmul_f32(dev, nt, shape):
    batch, m, k, n = shape
    lcg = Lcg(sum(shape))
    a, b = lcg.fill(batch * m * k, -1, 1), lcg.fill(batch * n * k, -1, 1)
    bshape = (batch, n, k) if nt else (batch, k, n)
    got = run1(dev, Op(OpCode.MatMulNT if nt else OpCode.MatMulNN), [put_f32(dev, a), put_f32(dev, b)],
               [F((batch, m, k)), F(bshape)], (batch, m, n))
    want = (orc.matmul_nt if nt else orc.matmul_nn)(a, b, batch, m, k, n)
    assert_reduction(got, want)


def test_matmul_broadcast_weight(dev):
    # [B, M, K] x [N, K] (2-D weight shared by every batch index, device.rs:1355-1407)
    batch, m, k, n = 3, 4, 32, 10
    lcg = Lcg(9)
    a, w = lcg.fill(batch * m * k, -1, 1), lcg.fill(n * k, -1, 1)
    got = run1(dev, Op(OpCode.MatMulNT), [put_f32(dev, a), put_f32(dev, w)],
               [F((batch, m, k)), F((n, k), ValueRole.Param)], (batch, m, n))
    want = np.concatenate([orc.matmul_nt(a[i * m * k:(i + 1) * m * k], w, 1, m, k, n)
                           for i in range(batch)])
    assert_reduction(got, want)


def test_matmul_zero_k_writes_zeros(dev):
    out = new_f32(dev, 6, fill=1.0)
    dev.dispatch(Op(OpCode.MatMulNT), [put_f32(dev, []), put_f32(dev, [])],
                 [F((1, 2, 0)), F((1, 3, 0))], [out], [F((1, 2, 3))])
    assert np.array_equal(get(dev, out), np.zeros(6, np.float32))


# ---------------------------------------------------------- quantization ----

@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("n,k,group", [(16, 256, 32), (5, 688, 32), (64, 4096, 128), (3, 33, 7),
                                       (7, 130, 128)])
def test_quantize_and_dequantize_bit_exact(dev, fmt, n, k, group):
    w = Lcg(n * k + group).normal(n * k, 0.0, 0.02)
    codes, scales = orc.quantize(fmt, w, n, k, group)
    wref = put_f32(dev, w)
    words = (codes.size + 3) // 4
    cb = dev.allocate_u32(words)
    sb = dev.allocate_f32(scales.size)
    qf = QuantFormat.Int4 if fmt == orc.INT4 else QuantFormat.Int8
    dev.quantize(wref, n, k, qf, group, cb, sb)
    dev.synchronize()
    got_codes = dev.download_u32(cb).view(np.uint8)[:codes.size]
    assert np.array_equal(got_codes, codes)
    assert np.array_equal(dev.download_f32(sb), scales)
    out = new_f32(dev, n * k)
    dev.dequantize(cb, sb, n, k, qf, group, out)
    assert np.array_equal(get(dev, out), orc.dequantize(fmt, codes, scales, n, k, group))


def _qmatmul_case(dev, fmt, m, k, n, group, seed, spot_rows=None):
    lcg = Lcg(seed)
    w = lcg.normal(n * k, 0.0, 0.02)
    x = lcg.normal(m * k, 0.0, 1.0)
    codes, scales = orc.quantize(fmt, w, n, k, group)
    qf = QuantFormat.Int4 if fmt == orc.INT4 else QuantFormat.Int8
    cb, sb, words = put_quant(dev, codes, scales, qf, group)
    out = new_f32(dev, m * n)
    dev.dispatch(Op(OpCode.MatMulNT), [put_f32(dev, x), BufferRef(cb, 0, words)],
                 [F((1, m, k)), Value.quantized((n, k), qf, group)], [out], [F((1, m, n))])
    got = get(dev, out).reshape(m, n)
    wd = orc.dequantize(fmt, codes, scales, n, k, group).reshape(n, k)
    rows = np.arange(n) if spot_rows is None else spot_rows
    want = x.reshape(m, k).astype(np.float64) @ wd[rows].astype(np.float64).T
    return assert_reduction(got[:, rows].ravel(), want.ravel())


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("m", [1, 4, 8, 16, 32, 33])
@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 1024), (1024, 4096)])
def test_quantized_matmul_g128(dev, fmt, m, k, n):
    err = _qmatmul_case(dev, fmt, m, k, n, 128, seed=m * 31 + k + n)
    # Regression bound well inside the tolerance: outputs here are ~N(0, 1.3),
    # an f32-class dot product of 4096 terms stays below 1e-4 absolute.
    assert err < 1e-4, err


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("m,k,n,group", [(1, 256, 256, 32), (16, 256, 688, 32), (1, 688, 256, 32),
                                         (3, 100, 48, 7), (2, 256, 40, 64)])
def test_quantized_matmul_irregular(dev, fmt, m, k, n, group):
    _qmatmul_case(dev, fmt, m, k, n, group, seed=m + k + n + group)


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("m,k,n,group", [
    (1, 640, 1040, 128),     # 5 warp-steps per row, a ragged last row block
    (3, 640, 1040, 128),
    (1, 256, 16, 128),       # one row block shared by many CTAs
    (2, 1024, 48, 256),      # group spanning two warp-steps (INT4)
    (32, 4096, 1024, 128),   # activation windows shorter than the row
    (17, 14336, 512, 128),   # three n-tiles, windows
    (5, 8192, 2064, 128),
    (1, 4096, 16032, 128),   # 8-way TP vocabulary slice: many tiles, ragged last block
    (1, 1792, 4096, 128),    # 8-way TP down projection K
    # K slices (at most 8 rows): digits of whole rows do not fit beside the
    # ring, so each CTA stages one slice and every slice's CTAs add partial sums
    (8, 14336, 512, 128),
    (8, 8192, 2064, 128),
    (3, 14336, 1040, 128),
    # more rows with long K: the other GEMV kernels
    (16, 8192, 1024, 128),
    (12, 8192, 2064, 128),
    (16, 28672, 256, 128),   # 70B down projection at batch 16
    (24, 4096, 1024, 128),
])
def test_quantized_matmul_tma_shapes(dev, fmt, m, k, n, group):
    # The TMA-fed decode GEMV: ranges that split row blocks across CTAs
    # (partial slots + ticket), windows, ragged row blocks, both formats.
    err = _qmatmul_case(dev, fmt, m, k, n, group, seed=m * 13 + k + n + group)
    assert err < 1e-4 * max(1.0, (k / 4096) ** 0.5), err


@pytest.mark.parametrize("fmt,m,k,n,group", [
    (orc.INT4, 65, 256, 256, 64),       # one partial M tile, groups of one stage
    (orc.INT4, 128, 4096, 512, 128),    # 32 groups through both TMEM buffers
    (orc.INT4, 200, 1024, 700, 128),    # ragged M and N (scalar tail columns)
    (orc.INT8, 130, 512, 384, 128),
    (orc.INT4, 96, 192, 260, 192),      # one group of three stages, N % 256 = 4
    (orc.INT8, 257, 4160, 256, 64),     # K beyond a multiple of 128
    (orc.INT4, 600, 14336, 256, 128),   # two passes of the activation split
    (orc.INT8, 512, 4096, 1024, 128),
])
def test_quantized_matmul_prefill_tensor_cores(dev, fmt, m, k, n, group):
    # Prefill-sized M: the tcgen05 GEMM (bf16 hi/lo activations, codes
    # expanded in shared memory, per-group TMEM partials scaled in f32).
    err = _qmatmul_case(dev, fmt, m, k, n, group, seed=m * 7 + k + n + group)
    assert err < 1e-4 * max(1.0, (k / 4096) ** 0.5), err


@pytest.mark.parametrize("fmt,k,n", [(orc.INT4, 14336, 4096), (orc.INT4, 4096, 14336),
                                     (orc.INT8, 8192, 1024), (orc.INT4, 4096, 128256),
                                     (orc.INT8, 8192, 32000)])
def test_quantized_matmul_full_size_spot_rows(dev, fmt, k, n):
    # The last two are the 8B vocabulary projection (INT4) and the 70B one
    # (INT8) at their full N.
    rows = np.array(sorted(set([0, 1, 15, 16, 127, 128, n // 2, n - 17, n - 1] +
                               list(Lcg(5).fill(32, 0, n - 1).astype(int)))))
    _qmatmul_case(dev, fmt, 1, k, n, 128, seed=k + n, spot_rows=rows)


# -------------------------------------------------------------- composites --

@pytest.mark.parametrize("quant", [None, orc.INT4, orc.INT8])
@pytest.mark.parametrize("rows,hidden,inter", [(1, 1, 1), (3, 5, 7), (4, 6, 13), (16, 256, 688),
                                               (1, 256, 512)])
def test_swiglu(dev, quant, rows, hidden, inter):
    lcg = Lcg(rows + hidden + inter)
    x = lcg.fill(rows * hidden, -1, 1)
    ws = [lcg.normal(inter * hidden, 0, 0.1), lcg.normal(inter * hidden, 0, 0.1),
          lcg.normal(hidden * inter, 0, 0.1)]
    shapes = [(inter, hidden), (inter, hidden), (hidden, inter)]
    refs, vals, dense = [], [], []
    for w, shp in zip(ws, shapes):
        if quant is None:
            refs.append(put_f32(dev, w))
            vals.append(F(shp, ValueRole.Param))
            dense.append(w)
        else:
            group = 32 if shp[1] % 32 == 0 else 7
            codes, scales = orc.quantize(quant, w, shp[0], shp[1], group)
            qf = QuantFormat.Int4 if quant == orc.INT4 else QuantFormat.Int8
            cb, _, words = put_quant(dev, codes, scales, qf, group)
            refs.append(BufferRef(cb, 0, words))
            vals.append(Value.quantized(shp, qf, group))
            dense.append(orc.dequantize(quant, codes, scales, shp[0], shp[1], group))
    got = run1(dev, Op(OpCode.SwiGlu), [put_f32(dev, x)] + refs, [F((rows, hidden))] + vals,
               (rows, hidden))
    assert_reduction(got, orc.swiglu(x, dense[0], dense[1], dense[2], rows, hidden, inter))


@pytest.mark.parametrize("quant", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("rows,hidden,inter", [(1, 512, 1024), (3, 512, 1536), (8, 1024, 512),
                                               (32, 512, 512)])
def test_swiglu_decode_grouped_path(dev, quant, rows, hidden, inter):
    # Group 128 and K a multiple of 512: gate and up in one TMA GEMV launch,
    # down with silu(gate) * up computed while its input is staged.
    lcg = Lcg(rows * 3 + hidden + inter)
    x = lcg.fill(rows * hidden, -1, 1)
    shapes = [(inter, hidden), (inter, hidden), (hidden, inter)]
    qf = QuantFormat.Int4 if quant == orc.INT4 else QuantFormat.Int8
    refs, vals, dense = [], [], []
    for shp in shapes:
        w = lcg.normal(shp[0] * shp[1], 0, 0.05)
        codes, scales = orc.quantize(quant, w, shp[0], shp[1], 128)
        cb, _, words = put_quant(dev, codes, scales, qf, 128)
        refs.append(BufferRef(cb, 0, words))
        vals.append(Value.quantized(shp, qf, 128))
        dense.append(orc.dequantize(quant, codes, scales, shp[0], shp[1], 128))
    got = run1(dev, Op(OpCode.SwiGlu), [put_f32(dev, x)] + refs, [F((rows, hidden))] + vals,
               (rows, hidden))
    assert_reduction(got, orc.swiglu(x, dense[0], dense[1], dense[2], rows, hidden, inter))


@pytest.mark.parametrize("rows,hidden,nout", [(1, 1, 1), (3, 7, 5), (2, 33, 17), (4, 16, 9),
                                              (8, 4096, 256)])
def test_rms_norm_matmul(dev, rows, hidden, nout):
    lcg = Lcg(rows * hidden + nout)
    x, g, w = lcg.fill(rows * hidden, -2, 2), lcg.fill(hidden, 0.5, 1.5), lcg.fill(nout * hidden, -1, 1)
    got = run1(dev, Op(OpCode.RmsNormMatMul, eps=1e-5), [put_f32(dev, x), put_f32(dev, g), put_f32(dev, w)],
               [F((rows, hidden)), F((hidden,), ValueRole.Param), F((nout, hidden), ValueRole.Param)],
               (rows, nout))
    assert_reduction(got, orc.rms_norm_matmul(x, g, w, rows, hidden, nout, 1e-5))


# ------------------------------------------------------------ validation ----

def test_alias_and_port_rejections(dev):  # device.rs:2250-2285 and validate_* rules
    buf = put_f32(dev, np.zeros(16))
    a = BufferRef(buf.buffer, 0, 8)
    overlapping = BufferRef(buf.buffer, 4, 8)
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add), [a, BufferRef(buf.buffer, 8, 8)], [F((8,)), F((8,))],
                     [overlapping], [F((8,))])
    assert e.value.message == "a command output aliases an overlapping input range"
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add), [a, a], [F((8,)), F((8,))], [BufferRef(buf.buffer, 8, 8)], [F((8,))])
    assert e.value.message == "one command aliases overlapping input ranges"
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add), [a, BufferRef(buf.buffer, 8, 7)], [F((8,)), F((8,))],
                     [new_f32(dev, 8)], [F((8,))])
    assert e.value.message == "BufferRef length does not match the value element count"
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add), [a, BufferRef(buf.buffer, 12, 8)], [F((8,)), F((8,))],
                     [new_f32(dev, 8)], [F((8,))])
    assert e.value.status == Status.InvalidRange
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add), [a], [F((8,))], [new_f32(dev, 8)], [F((8,))])
    assert e.value.message == "input buffer count does not match the operator signature"
    u = put_u32(dev, np.zeros(8))
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Silu), [a], [F((8,))], [u], [Value.u32((8,), ValueRole.Temp)])
    assert e.value.message == "integer command outputs are not supported"
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Silu), [u], [F((8,))], [new_f32(dev, 8)], [F((8,))])
    assert e.value.status == Status.InvalidBuffer
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.LastToken), [a], [F((2, 4, 1))], [new_f32(dev, 2)], [F((2, 1))], [0])
    assert e.value.message == "last_token requires 1 <= seq_len <= seq"


def test_unknown_opcode_is_unsupported(dev):
    with pytest.raises(DeviceError) as e:
        dev.dispatch(Op(OpCode.Add).__class__(code=99), [], [], [], [])
    assert e.value.status == Status.UnsupportedOp


def test_upload_download_length_rules(dev):  # device.rs:123-173
    b = dev.allocate_f32(4)
    with pytest.raises(DeviceError) as e:
        dev.upload_f32(b, [1, 2, 3])
    assert e.value.status == Status.InvalidRange
    with pytest.raises(DeviceError) as e:
        dev.download_u32(b)
    assert e.value.status == Status.InvalidBuffer
    with pytest.raises(DeviceError) as e:
        dev.allocate_f32(4, 3)
    assert e.value.message == "alignment must be a nonzero power of two"
    b2 = dev.allocate_f32(5, 4096)
    assert dev.device_ptr(b2) % 4096 == 0
