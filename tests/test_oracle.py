"""Pins the CPU oracle to the reference's own tests.

Every case below restates a unit test of crates/backends/backend-cpu/src/
reference/*.rs (same shapes, same LCG seeds, same fill ranges, the same
independent f64 oracle and the same `assert_close(abs 1e-4 OR rel 1e-5)`,
reference/mod.rs:154-165), plus the known-answer tests and the
starlight-runtime end-to-end fixture (tests/end_to_end.rs:38-68). The Rust
reference cannot be compiled here (no cargo; its sl-* dependencies are empty
submodules), so these restated tests are the pin.
"""
import math

import numpy as np
import pytest

from oracle import pyoracle as orc
from oracle.pyoracle import Lcg, OracleError


def assert_close(actual, expected, abs_tol=1e-4, rel_tol=1e-5):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape
    diff = np.abs(actual - expected)
    tol = np.maximum(abs_tol, rel_tol * np.abs(expected))
    bad = np.nonzero(diff > tol)[0]
    assert bad.size == 0, f"mismatch at {bad[:5]}: {actual[bad[:5]]} vs {expected[bad[:5]]}"


def raises(code, fn, *a, **k):
    with pytest.raises(OracleError) as e:
        fn(*a, **k)
    assert e.value.code == code, e.value
    return e.value


# ---------------------------------------------------------------- LCG ------

def test_lcg_matches_pcg_constants():
    # mod.rs:125-131: state = state * 6364136223846793005 + 1442695040888963407
    lcg = Lcg(1)
    state = 1
    for _ in range(5):
        state = (state * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        assert lcg.next_u32() == state >> 33
    # uniform(lo, hi) = lo + (hi - lo) * (u32 / u32::MAX as f64) as f32
    lcg = Lcg(7)
    ref = Lcg(7)
    u = ref.next_u32()
    unit = np.float32(u / 4294967295.0)
    want = np.float32(np.float32(-2.0) + np.float32(np.float32(4.0) * unit))
    assert lcg.uniform(-2.0, 2.0) == want


# ------------------------------------------------------------- matmul ------

def f64_matmul_nt(a, b, batch, m, k, n):
    a = a.astype(np.float64).reshape(batch, m, k)
    b = b.astype(np.float64).reshape(batch, n, k)
    return np.einsum("bmk,bnk->bmn", a, b).ravel()


def f64_matmul_nn(a, b, batch, m, k, n):
    a = a.astype(np.float64).reshape(batch, m, k)
    b = b.astype(np.float64).reshape(batch, k, n)
    return np.einsum("bmk,bkn->bmn", a, b).ravel()


@pytest.mark.parametrize("seed,shape", [(1, (1, 1, 1, 1)), (2, (2, 3, 5, 7)), (3, (2, 4, 9, 6))])
def test_matmul_nt_matches_f64_oracle(seed, shape):  # matmul.rs:357-362
    batch, m, k, n = shape
    lcg = Lcg(seed)
    a = lcg.fill(batch * m * k, -1.0, 1.0)
    b = lcg.fill(batch * n * k, -1.0, 1.0)
    assert_close(orc.matmul_nt(a, b, batch, m, k, n), f64_matmul_nt(a, b, batch, m, k, n))


@pytest.mark.parametrize("seed,shape", [(11, (1, 1, 1, 1)), (12, (3, 4, 7, 5)), (13, (2, 5, 3, 9))])
def test_matmul_nn_matches_f64_oracle(seed, shape):  # matmul.rs:364-370
    batch, m, k, n = shape
    lcg = Lcg(seed)
    a = lcg.fill(batch * m * k, -1.0, 1.0)
    b = lcg.fill(batch * k * n, -1.0, 1.0)
    assert_close(orc.matmul_nn(a, b, batch, m, k, n), f64_matmul_nn(a, b, batch, m, k, n))


def test_matmul_accepts_empty_dimensions():  # matmul.rs:372-394
    e = np.zeros(0, np.float32)
    orc.matmul_nt(e, e, 0, 2, 3, 4)
    orc.matmul_nn(e, e, 0, 2, 3, 4)
    empty_b = np.zeros(2 * 4 * 3, np.float32)
    orc.matmul_nt(e, empty_b, 2, 0, 3, 4, out_len=0)
    orc.matmul_nn(e, empty_b, 2, 0, 3, 4, out_len=0)
    out = orc.matmul_nt(e, e, 1, 2, 0, 3)
    assert np.array_equal(out, np.zeros(6, np.float32))
    out = orc.matmul_nn(e, e, 1, 2, 0, 3)
    assert np.array_equal(out, np.zeros(6, np.float32))


def test_matmul_rejects_wrong_lengths():  # matmul.rs:396-423
    a = np.zeros(2 * 3 * 4, np.float32)
    b_nt = np.zeros(2 * 5 * 4, np.float32)
    b_nn = np.zeros(2 * 4 * 5, np.float32)
    raises(orc.LENGTH_MISMATCH, orc.matmul_nt, a[:-1], b_nt, 2, 3, 4, 5)
    raises(orc.LENGTH_MISMATCH, orc.matmul_nt, a, b_nt[:-1], 2, 3, 4, 5)
    raises(orc.LENGTH_MISMATCH, orc.matmul_nn, a, b_nn, 2, 3, 4, 5, out_len=29)
    raises(orc.LENGTH_MISMATCH, orc.matmul_nn, a, b_nn[:-1], 2, 3, 4, 5)


def test_matmul_reports_shape_overflow():  # matmul.rs:425-432
    e = np.zeros(0, np.float32)
    raises(orc.SHAPE_OVERFLOW, orc.matmul_nt, e, e, 2**64 - 1, 2, 1, 1, out_len=0)


# --------------------------------------------------------------- norm ------

def f64_rms_norm(x, w, rows, hidden, eps):
    x = x.astype(np.float64).reshape(rows, hidden)
    ms = (x * x).sum(axis=1, keepdims=True) / hidden
    return (x * (1.0 / np.sqrt(ms + np.float64(np.float32(eps)))) * w.astype(np.float64)).ravel()


@pytest.mark.parametrize("rows,hidden,eps,seed", [(1, 1, 1e-5, 1), (3, 7, 1e-6, 2),
                                                  (4, 16, 1e-5, 3), (2, 33, 1e-6, 4)])
def test_rms_norm_matches_f64_oracle(rows, hidden, eps, seed):  # norm.rs:105-111
    lcg = Lcg(seed)
    x = lcg.fill(rows * hidden, -2.0, 2.0)
    w = lcg.fill(hidden, 0.5, 1.5)
    assert_close(orc.rms_norm(x, w, rows, hidden, eps), f64_rms_norm(x, w, rows, hidden, eps))


def test_rms_norm_zero_rows_and_invalid():  # norm.rs:113-143
    orc.rms_norm(np.zeros(0), np.ones(4), 0, 4, 1e-5)
    raises(orc.INVALID_SHAPE, orc.rms_norm, np.zeros(0), np.zeros(0), 2, 0, 1e-5, out_len=0)
    x, w = np.ones(8), np.ones(4)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm, x, w[:3], 2, 4, 1e-5)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm, x[:7], w, 2, 4, 1e-5)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm, x, w, 2, 4, 1e-5, out_len=7)


# --------------------------------------------------------------- rope ------

def make_positions(lcg, batch, seq, past_offset):  # rope.rs:292-298
    return np.array([past_offset + i * 2 + lcg.below(5) for i in range(batch * seq)], np.uint32)


def f64_rope(x, pos, batch, heads, seq, hd, theta, gptj):
    out = x.astype(np.float64).copy()
    half = hd // 2
    for b in range(batch):
        for t in range(seq):
            p = float(pos[b * seq + t])
            for pair in range(half):
                ang = p / (float(np.float32(theta)) ** (2.0 * pair / hd))
                s, c = math.sin(ang), math.cos(ang)
                for h in range(heads):
                    base = ((b * heads + h) * seq + t) * hd
                    i0, i1 = (base + 2 * pair, base + 2 * pair + 1) if gptj else (base + pair, base + pair + half)
                    f, g = float(x[i0]), float(x[i1])
                    out[i0] = f * c - g * s
                    out[i1] = f * s + g * c
    return out


@pytest.mark.parametrize("seed,shape", [(1, (1, 1, 1, 2, 10000.0)), (2, (2, 3, 5, 4, 10000.0)),
                                        (3, (2, 2, 4, 8, 500000.0)), (4, (1, 3, 3, 6, 10000.0))])
def test_rope_neox_matches_f64_oracle(seed, shape):  # rope.rs:382-392
    batch, heads, seq, hd, theta = shape
    lcg = Lcg(seed)
    x = lcg.fill(batch * heads * seq * hd, -2.0, 2.0)
    pos = make_positions(lcg, batch, seq, 3)
    assert_close(orc.rope(x, pos, batch, heads, seq, hd, theta, "neox"),
                 f64_rope(x, pos, batch, heads, seq, hd, theta, False))


@pytest.mark.parametrize("seed,shape", [(11, (1, 1, 1, 2, 10000.0)), (12, (2, 3, 5, 4, 10000.0)),
                                        (13, (2, 2, 4, 8, 500000.0)), (14, (1, 2, 3, 10, 1000000.0))])
def test_rope_gptj_matches_f64_oracle(seed, shape):  # rope.rs:394-404
    batch, heads, seq, hd, theta = shape
    lcg = Lcg(seed)
    x = lcg.fill(batch * heads * seq * hd, -2.0, 2.0)
    pos = make_positions(lcg, batch, seq, 1)
    assert_close(orc.rope(x, pos, batch, heads, seq, hd, theta, "gptj"),
                 f64_rope(x, pos, batch, heads, seq, hd, theta, True))


def test_rope_rejects_invalid_shapes():  # rope.rs:406-426
    x = np.zeros(8, np.float32)
    p = np.zeros(2, np.uint32)
    raises(orc.INVALID_SHAPE, orc.rope, x, p, 1, 1, 2, 3, 10000.0, "neox")
    raises(orc.INVALID_SHAPE, orc.rope, x, p, 1, 1, 2, 0, 10000.0, "gptj")
    raises(orc.LENGTH_MISMATCH, orc.rope, x, p[:1], 1, 1, 2, 4, 10000.0, "neox")
    raises(orc.LENGTH_MISMATCH, orc.rope, x[:7], p, 1, 1, 2, 4, 10000.0, "gptj")


# -------------------------------------------------------- elementwise ------

def f64_silu(x):
    x = x.astype(np.float64)
    return x / (1.0 + np.exp(-x))


@pytest.mark.parametrize("seed,n", [(1, 1), (2, 7), (3, 33)])
def test_silu_matches_f64_oracle(seed, n):  # elementwise.rs:517-532
    x = Lcg(seed).fill(n, -8.0, 8.0)
    assert_close(orc.silu(x), f64_silu(x))


def test_silu_extreme_values():  # elementwise.rs:528-531
    x = np.array([-100.0, -10.0, 0.0, 10.0, 100.0], np.float32)
    assert_close(orc.silu(x), f64_silu(x))


@pytest.mark.parametrize("seed,n", [(11, 0), (12, 1), (13, 5), (14, 33)])
def test_mul_add_scale_match_f64_oracle(seed, n):  # elementwise.rs:534-570
    lcg = Lcg(seed)
    a = lcg.fill(n, -2.0, 2.0)
    b = lcg.fill(n, -2.0, 2.0)
    assert_close(orc.mul(a, b, n), a.astype(np.float64) * b)
    assert_close(orc.add(a, b, n), a.astype(np.float64) + b)
    assert_close(orc.scale(a, -1.5), a.astype(np.float64) * -1.5)


def test_elementwise_rejects_wrong_lengths():  # elementwise.rs:572-596
    a = np.array([1, 2, 3], np.float32)
    b = np.array([4, 5, 6], np.float32)
    raises(orc.LENGTH_MISMATCH, orc.mul, a, b[:2], 3)
    raises(orc.LENGTH_MISMATCH, orc.mul, a[:2], b, 3)
    raises(orc.LENGTH_MISMATCH, orc.add, a, b, 3, out_len=2)
    raises(orc.LENGTH_MISMATCH, orc.add, a, b[:2], 3)
    e = np.zeros(0, np.float32)
    orc.silu(e); orc.scale(e, 2.0); orc.mul(e, e, 0); orc.add(e, e, 0)


# ------------------------------------------------------------ softmax ------

def f64_softmax(x, rows, cols):
    x = x.astype(np.float64).reshape(rows, cols)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)).ravel()


def f64_softmax_causal(x, rows, cols, seq, past):
    x = x.astype(np.float64).reshape(rows, cols)
    out = np.zeros_like(x)
    for r in range(rows):
        last = past + r % seq
        row = x[r, :last + 1]
        e = np.exp(row - row.max())
        out[r, :last + 1] = e / e.sum()
    return out.ravel()


@pytest.mark.parametrize("seed,shape", [(1, (1, 1)), (2, (3, 5)), (3, (6, 17))])
def test_softmax_matches_f64_oracle(seed, shape):  # softmax.rs:194-199
    rows, cols = shape
    x = Lcg(seed).fill(rows * cols, -4.0, 4.0)
    assert_close(orc.softmax(x, rows, cols), f64_softmax(x, rows, cols))


def test_softmax_is_stable_for_extreme_values():  # softmax.rs:201-208
    x = np.array([1000.0, 999.0, -1000.0, 0.0], np.float32)
    out = orc.softmax(x, 2, 2)
    assert_close(out, f64_softmax(x, 2, 2))
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("seed,shape", [(11, (2, 2, 0)), (12, (12, 4, 1)), (13, (4, 1, 7)),
                                        (14, (6, 3, 2))])
def test_softmax_causal_matches_f64_oracle(seed, shape):  # softmax.rs:210-220
    rows, seq, past = shape
    cols = past + seq
    x = Lcg(seed).fill(rows * cols, -3.0, 3.0)
    assert_close(orc.softmax_causal(x, rows, cols, seq, past),
                 f64_softmax_causal(x, rows, cols, seq, past))


def test_softmax_rejects_invalid_shapes():  # softmax.rs:222-254
    e = np.zeros(0, np.float32)
    raises(orc.INVALID_SHAPE, orc.softmax, e, 0, 4)
    raises(orc.INVALID_SHAPE, orc.softmax, e, 4, 0)
    raises(orc.LENGTH_MISMATCH, orc.softmax, np.zeros(5), 2, 3)
    raises(orc.INVALID_SHAPE, orc.softmax_causal, np.zeros(6), 2, 3, 2, 0)
    raises(orc.INVALID_SHAPE, orc.softmax_causal, np.zeros(4), 2, 2, 0, 2)
    raises(orc.INVALID_SHAPE, orc.softmax_causal, np.zeros(6), 3, 2, 2, 0)
    raises(orc.LENGTH_MISMATCH, orc.softmax_causal, np.zeros(5), 2, 3, 2, 1)


# ------------------------------------------------------------- layout ------

@pytest.mark.parametrize("seed,shape", [(1, (10, 5, 3)), (2, (1, 1, 1)), (3, (4, 7, 0)),
                                        (4, (13, 9, 6))])
def test_gather_matches_f64_oracle(seed, shape):  # layout.rs:1075-1085
    vocab, hidden, rows = shape
    lcg = Lcg(seed)
    table = lcg.fill(vocab * hidden, -1.0, 1.0)
    ids = np.array([lcg.below(vocab) for _ in range(rows)], np.uint32)
    want = table.reshape(vocab, hidden)[ids].ravel() if rows else np.zeros(0)
    assert_close(orc.gather(table, ids, vocab, hidden, rows), want)


def test_gather_rejects_bad_ids_and_lengths():  # layout.rs:1087-1107
    table = np.array([1, 2, 3, 4], np.float32)
    out = np.zeros(2, np.float32)
    e = raises(orc.INVALID_SHAPE, orc.gather, table, [4], 2, 2, 1, out=out)
    assert e.reason == "id out of range"
    assert np.array_equal(out, np.zeros(2, np.float32))
    raises(orc.LENGTH_MISMATCH, orc.gather, table[:3], [0], 2, 2, 1)
    raises(orc.LENGTH_MISMATCH, orc.gather, table, [0, 1], 2, 2, 1)
    raises(orc.LENGTH_MISMATCH, orc.gather, table, [0], 2, 2, 1, out=np.zeros(1, np.float32))


@pytest.mark.parametrize("seed,shape", [(11, (1, 1, 3, 1)), (12, (3, 5, 4, 5)), (13, (2, 4, 7, 2))])
def test_last_token_matches_f64_oracle(seed, shape):  # layout.rs:1109-1116
    batch, seq, hidden, seq_len = shape
    x = Lcg(seed).fill(batch * seq * hidden, -1.0, 1.0)
    want = x.reshape(batch, seq, hidden)[:, seq_len - 1].ravel()
    assert_close(orc.last_token(x, batch, seq, hidden, seq_len), want)


def test_last_token_rejects_bad_seq_len_and_lengths():  # layout.rs:1118-1138
    x = np.zeros(16, np.float32)
    raises(orc.INVALID_SHAPE, orc.last_token, x, 2, 4, 2, 0)
    raises(orc.INVALID_SHAPE, orc.last_token, x, 2, 4, 2, 5)
    raises(orc.LENGTH_MISMATCH, orc.last_token, x[:15], 2, 4, 2, 4)
    raises(orc.LENGTH_MISMATCH, orc.last_token, x, 2, 4, 2, 4, out_len=3)


@pytest.mark.parametrize("seed,shape", [(21, (1, 1, 1, 2)), (22, (2, 3, 4, 4)), (23, (2, 5, 3, 6)),
                                        (24, (1, 4, 2, 8))])
def test_split_and_merge_heads_match_f64_oracle(seed, shape):  # layout.rs:1140-1150
    batch, seq, heads, hd = shape
    x = Lcg(seed).fill(batch * seq * heads * hd, -1.0, 1.0)
    split = orc.split_heads(x, batch, seq, heads, hd)
    assert_close(split, x.reshape(batch, seq, heads, hd).transpose(0, 2, 1, 3).ravel())
    merged = orc.merge_heads(split, batch, seq, heads, hd)
    assert_close(merged, x)


def test_split_and_merge_reject_wrong_lengths():  # layout.rs:1152-1172
    x = np.zeros(16, np.float32)
    raises(orc.LENGTH_MISMATCH, orc.split_heads, x[:15], 2, 2, 2, 2)
    raises(orc.LENGTH_MISMATCH, orc.split_heads, x, 2, 2, 2, 2, out_len=15)
    raises(orc.LENGTH_MISMATCH, orc.merge_heads, x[:15], 2, 2, 2, 2)
    raises(orc.LENGTH_MISMATCH, orc.merge_heads, x, 2, 2, 2, 2, out_len=15)


# ---------------------------------------------------------- attention ------

SHAPE_FIELDS = ("batch", "layers", "layer", "heads", "kv_heads", "seq", "past_len", "head_dim",
                "max_seq")


def f64_kv_append(k, v, cache, s):
    cache = cache.astype(np.float64).copy()
    ts = s["kv_heads"] * s["head_dim"]
    ps = s["max_seq"] * ts
    ls = 2 * ps
    bs = s["layers"] * ls
    for b in range(s["batch"]):
        for h in range(s["kv_heads"]):
            for t in range(s["seq"]):
                src = ((b * s["kv_heads"] + h) * s["seq"] + t) * s["head_dim"]
                dst = b * bs + s["layer"] * ls + (s["past_len"] + t) * ts + h * s["head_dim"]
                cache[dst:dst + s["head_dim"]] = k[src:src + s["head_dim"]]
                cache[dst + ps:dst + ps + s["head_dim"]] = v[src:src + s["head_dim"]]
    return cache


def f64_attention(q, k, v, cache_seed, s, scale):
    cache = f64_kv_append(k, v, cache_seed, s)
    ts = s["kv_heads"] * s["head_dim"]
    ps = s["max_seq"] * ts
    ls = 2 * ps
    bs = s["layers"] * ls
    group = s["heads"] // s["kv_heads"]
    hd = s["head_dim"]
    out = np.zeros(s["batch"] * s["heads"] * s["seq"] * hd)
    for b in range(s["batch"]):
        for h in range(s["heads"]):
            kvh = h // group
            for t in range(s["seq"]):
                n = s["past_len"] + t + 1
                qb = ((b * s["heads"] + h) * s["seq"] + t) * hd
                kb = b * bs + s["layer"] * ls + kvh * hd
                vb = kb + ps
                keys = np.stack([cache[kb + j * ts:kb + j * ts + hd] for j in range(n)])
                vals = np.stack([cache[vb + j * ts:vb + j * ts + hd] for j in range(n)])
                sc = keys @ q[qb:qb + hd].astype(np.float64) * float(scale)
                p = np.exp(sc - sc.max())
                p /= p.sum()
                out[qb:qb + hd] = p @ vals
    return out, cache


KV_CASES = [
    (1, dict(batch=1, layers=1, layer=0, heads=1, kv_heads=1, seq=2, past_len=0, head_dim=2, max_seq=4)),
    (2, dict(batch=2, layers=2, layer=1, heads=2, kv_heads=2, seq=3, past_len=2, head_dim=3, max_seq=5)),
    (3, dict(batch=1, layers=1, layer=0, heads=2, kv_heads=2, seq=1, past_len=0, head_dim=8, max_seq=1)),
    (4, dict(batch=1, layers=1, layer=0, heads=1, kv_heads=1, seq=0, past_len=2, head_dim=4, max_seq=4)),
]

ATTENTION_CASES = [
    (11, dict(batch=1, layers=1, layer=0, heads=2, kv_heads=2, seq=3, past_len=0, head_dim=4, max_seq=4)),
    (12, dict(batch=2, layers=1, layer=0, heads=2, kv_heads=2, seq=1, past_len=3, head_dim=8, max_seq=6)),
    (13, dict(batch=2, layers=2, layer=1, heads=4, kv_heads=2, seq=2, past_len=2, head_dim=8, max_seq=5)),
    (14, dict(batch=2, layers=1, layer=0, heads=2, kv_heads=1, seq=1, past_len=5, head_dim=2, max_seq=7)),
    (15, dict(batch=1, layers=1, layer=0, heads=6, kv_heads=3, seq=2, past_len=1, head_dim=4, max_seq=4)),
    (16, dict(batch=1, layers=1, layer=0, heads=3, kv_heads=1, seq=1, past_len=2, head_dim=4, max_seq=3)),
]


def sizes(s):
    q = s["batch"] * s["heads"] * s["seq"] * s["head_dim"]
    kv = s["batch"] * s["kv_heads"] * s["seq"] * s["head_dim"]
    cache = s["batch"] * s["layers"] * 2 * s["max_seq"] * s["kv_heads"] * s["head_dim"]
    return q, kv, cache


@pytest.mark.parametrize("seed,s", KV_CASES)
def test_kv_append_matches_f64_oracle(seed, s):  # attention.rs:405-467
    _, kvl, cl = sizes(s)
    lcg = Lcg(seed)
    k = lcg.fill(kvl, -1.0, 1.0)
    v = lcg.fill(kvl, -1.0, 1.0)
    cache = lcg.fill(cl, -1.0, 1.0)
    got = orc.kv_append(k, v, cache, s["batch"], s["layers"], s["layer"], s["kv_heads"],
                        s["head_dim"], s["max_seq"], s["past_len"], s["seq"])
    assert_close(got, f64_kv_append(k, v, cache, s))


def test_kv_append_rejects_invalid_shapes():  # attention.rs:469-507
    k = np.zeros(8, np.float32)
    v = np.zeros(8, np.float32)
    cache = np.zeros(24, np.float32)
    raises(orc.LENGTH_MISMATCH, orc.kv_append, k[:-1], v, cache, 1, 1, 0, 1, 4, 3, 1, 2)
    raises(orc.LENGTH_MISMATCH, orc.kv_append, k, v[:-1], cache, 1, 1, 0, 1, 4, 3, 1, 2)
    raises(orc.LENGTH_MISMATCH, orc.kv_append, k, v, cache[:-1], 1, 1, 0, 1, 4, 3, 1, 2)
    raises(orc.INVALID_SHAPE, orc.kv_append, k, v, cache, 1, 1, 1, 1, 4, 3, 1, 2)
    raises(orc.INVALID_SHAPE, orc.kv_append, k, v, cache, 1, 1, 0, 1, 4, 3, 2, 2)


def test_kv_append_writes_documented_layout():  # attention.rs:509-527 (known answer)
    cache = orc.kv_append([1.0, 2.0], [3.0, 4.0], np.zeros(24), 1, 2, 1, 1, 2, 3, 1, 1)
    assert list(cache[14:16]) == [1.0, 2.0]
    assert list(cache[20:22]) == [3.0, 4.0]
    for i, val in enumerate(cache):
        if i not in (14, 15, 20, 21):
            assert val == 0.0


def test_causal_attention_matches_hand_computed_decode():  # attention.rs:529-542
    out, _ = orc.causal_attention([1.0, 0.0], [1.0, 0.0], [3.0, 4.0], np.zeros(4), 1, 1, 0, 1, 1,
                                  1, 0, 2, 1, 1.0)
    assert_close(out, [3.0, 4.0])


@pytest.mark.parametrize("seed,s", ATTENTION_CASES)
def test_causal_attention_matches_f64_oracle(seed, s):  # attention.rs:544-634
    ql, kvl, cl = sizes(s)
    lcg = Lcg(seed)
    q = lcg.fill(ql, -1.0, 1.0)
    k = lcg.fill(kvl, -1.0, 1.0)
    v = lcg.fill(kvl, -1.0, 1.0)
    cache = lcg.fill(cl, -1.0, 1.0)
    scale = np.float32(1.0 / math.sqrt(s["head_dim"]))
    out, new_cache = orc.causal_attention(q, k, v, cache, *(s[f] for f in SHAPE_FIELDS[:3]),
                                          s["heads"], s["kv_heads"], s["seq"], s["past_len"],
                                          s["head_dim"], s["max_seq"], float(scale))
    want_out, want_cache = f64_attention(q, k, v, cache, s, scale)
    assert_close(out, want_out)
    assert_close(new_cache, want_cache)


def test_causal_attention_accepts_empty_sequence():  # attention.rs:636-675
    cache = Lcg(21).fill(1 * 1 * 2 * 4 * 1 * 4, -1.0, 1.0)
    out, new_cache = orc.causal_attention(np.zeros(0), np.zeros(0), np.zeros(0), cache, 1, 1, 0, 1,
                                          1, 0, 2, 4, 4, 0.5)
    assert_close(new_cache, cache)
    assert out.size == 0


def test_causal_attention_rejects_invalid_shapes():  # attention.rs:677-787
    # shape: batch 1, layers 1, heads 2, kv_heads 2, seq 2, past 1, head_dim 4, max_seq 3
    q = np.zeros(16, np.float32)
    k = np.zeros(16, np.float32)
    v = np.zeros(16, np.float32)
    cache = np.zeros(48, np.float32)
    ca = orc.causal_attention
    raises(orc.INVALID_SHAPE, ca, q, k, v, cache, 1, 1, 0, 3, 2, 2, 1, 4, 3, 0.5, out_len=16)
    raises(orc.INVALID_SHAPE, ca, q, k, v, cache, 1, 1, 0, 0, 0, 2, 1, 4, 3, 0.5, out_len=16)
    raises(orc.INVALID_SHAPE, ca, q, k, v, cache, 1, 1, 0, 0, 1, 2, 1, 4, 3, 0.5, out_len=16)
    raises(orc.INVALID_SHAPE, ca, q, k, v, cache, 1, 1, 1, 2, 2, 2, 1, 4, 3, 0.5)
    raises(orc.INVALID_SHAPE, ca, q, k, v, cache, 1, 1, 0, 2, 2, 2, 2, 4, 3, 0.5)
    raises(orc.LENGTH_MISMATCH, ca, q[:-1], k, v, cache, 1, 1, 0, 2, 2, 2, 1, 4, 3, 0.5, out_len=16)
    raises(orc.LENGTH_MISMATCH, ca, q, k, v, cache, 1, 1, 0, 2, 2, 2, 1, 4, 3, 0.5, out_len=15)
    raises(orc.LENGTH_MISMATCH, ca, q, k, v, cache[:-1], 1, 1, 0, 2, 2, 2, 1, 4, 3, 0.5)


# -------------------------------------------------------------- fused ------

def f64_swiglu(x, g, u, d, rows, hidden, inter):
    x = x.astype(np.float64).reshape(rows, hidden)
    gate = x @ g.astype(np.float64).reshape(inter, hidden).T
    up = x @ u.astype(np.float64).reshape(inter, hidden).T
    h = gate / (1.0 + np.exp(-gate)) * up
    return (h @ d.astype(np.float64).reshape(hidden, inter).T).ravel()


@pytest.mark.parametrize("rows,hidden,inter,seed", [(1, 1, 1, 1), (3, 5, 7, 2), (2, 8, 4, 3),
                                                    (4, 6, 13, 4)])
def test_swiglu_matches_f64_oracle(rows, hidden, inter, seed):  # swiglu.rs:399-405
    lcg = Lcg(seed)
    x = lcg.fill(rows * hidden, -1.0, 1.0)
    g = lcg.fill(inter * hidden, -1.0, 1.0)
    u = lcg.fill(inter * hidden, -1.0, 1.0)
    d = lcg.fill(hidden * inter, -1.0, 1.0)
    assert_close(orc.swiglu(x, g, u, d, rows, hidden, inter), f64_swiglu(x, g, u, d, rows, hidden, inter))


def test_swiglu_zero_rows_and_invalid():  # swiglu.rs:407-455
    orc.swiglu(np.zeros(0), np.full(6, 0.5), np.full(6, 0.25), np.full(6, 0.75), 0, 3, 2)
    e = np.zeros(0, np.float32)
    raises(orc.INVALID_SHAPE, orc.swiglu, e, e, e, e, 0, 0, 2)
    raises(orc.INVALID_SHAPE, orc.swiglu, e, e, e, e, 0, 2, 0)
    x, w = np.ones(4), np.ones(8)
    raises(orc.LENGTH_MISMATCH, orc.swiglu, x[:3], w, w, w, 2, 2, 4)
    raises(orc.LENGTH_MISMATCH, orc.swiglu, x, w[:7], w, w, 2, 2, 4)
    raises(orc.LENGTH_MISMATCH, orc.swiglu, x, w, w[:7], w, 2, 2, 4)
    raises(orc.LENGTH_MISMATCH, orc.swiglu, x, w, w, w[:7], 2, 2, 4)
    raises(orc.LENGTH_MISMATCH, orc.swiglu, x, w, w, w, 2, 2, 4, out_len=3)


def f64_rms_norm_matmul(x, g, w, rows, hidden, nout, eps):
    n = f64_rms_norm(x, g, rows, hidden, eps).reshape(rows, hidden)
    return (n @ w.astype(np.float64).reshape(nout, hidden).T).ravel()


@pytest.mark.parametrize("rows,hidden,nout,eps,seed", [(1, 1, 1, 1e-5, 1), (3, 7, 5, 1e-6, 2),
                                                       (2, 33, 17, 1e-5, 3), (4, 16, 9, 1e-6, 4)])
def test_rms_norm_matmul_matches_f64_oracle(rows, hidden, nout, eps, seed):  # fused.rs:601-608
    lcg = Lcg(seed)
    x = lcg.fill(rows * hidden, -2.0, 2.0)
    g = lcg.fill(hidden, 0.5, 1.5)
    w = lcg.fill(nout * hidden, -1.0, 1.0)
    assert_close(orc.rms_norm_matmul(x, g, w, rows, hidden, nout, eps),
                 f64_rms_norm_matmul(x, g, w, rows, hidden, nout, eps))


def test_rms_norm_matmul_zero_rows_and_invalid():  # fused.rs:610-656
    orc.rms_norm_matmul(np.zeros(0), [1.0, 0.5, 2.0], np.ones(6), 0, 3, 2, 1e-5)
    e = np.zeros(0, np.float32)
    x, g, w = np.ones(8), np.ones(4), np.ones(12)
    raises(orc.INVALID_SHAPE, orc.rms_norm_matmul, e, e, e, 2, 0, 3, 1e-5, out_len=0)
    raises(orc.INVALID_SHAPE, orc.rms_norm_matmul, e, e, e, 2, 4, 0, 1e-5, out_len=0)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm_matmul, x[:7], g, w, 2, 4, 3, 1e-5)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm_matmul, x, g[:3], w, 2, 4, 3, 1e-5)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm_matmul, x, g, w[:11], 2, 4, 3, 1e-5)
    raises(orc.LENGTH_MISMATCH, orc.rms_norm_matmul, x, g, w, 2, 4, 3, 1e-5, out_len=5)
    raises(orc.SHAPE_OVERFLOW, orc.rms_norm_matmul, e, g, w, 2**64 - 1, 4, 3, 1e-5, out_len=0)


# ---------------------------------------------- end-to-end 4-op fixture -----

def fixture_weights():  # distros/starlight-runtime/src/fixture.rs:200-217
    embed = np.array([(i - 3.0) * 0.1 for i in range(32)], np.float32)
    norm = np.array([1.0, 0.5, 1.5, 0.75], np.float32)
    lm_head = np.array([((i % 5) - 2.0) * 0.1 for i in range(32)], np.float32)
    return embed, norm, lm_head


def test_fixture_constants():  # fixture.rs:259-271
    embed, norm, lm_head = fixture_weights()
    assert embed[0] == np.float32(-0.3) and embed[3] == 0.0 and embed[31] == np.float32(2.8)
    assert lm_head[0] == np.float32(-0.2) and lm_head[4] == np.float32(0.2)
    assert lm_head[5] == np.float32(-0.2)


def expected_fixture_logits(ids):  # tests/end_to_end.rs:38-68 (independent f64)
    embedding = [(i - 3.0) * 0.1 for i in range(32)]
    norm = [1.0, 0.5, 1.5, 0.75]
    lm = [((i % 5) - 2.0) * 0.1 for i in range(32)]
    last = None
    for tok in ids:
        row = embedding[tok * 4:tok * 4 + 4]
        ms = sum(v * v for v in row) / 4
        sc = 1.0 / math.sqrt(ms + 1e-5)
        last = [v * sc * w for v, w in zip(row, norm)]
    return [sum(last[c] * lm[vv * 4 + c] for c in range(4)) for vv in range(8)]


def run_fixture_chain(ids):
    """Gather -> RmsNorm -> MatMulNT -> LastToken through the oracle kernels."""
    embed, norm, lm_head = fixture_weights()
    seq = len(ids)
    x = orc.gather(embed, ids, 8, 4, seq)
    h = orc.rms_norm(x, norm, seq, 4, 1e-5)
    mm = orc.matmul_nt(h, lm_head, 1, seq, 4, 8)
    return orc.last_token(mm, 1, seq, 8, seq)


@pytest.mark.parametrize("ids", [[1, 2], [7]])
def test_end_to_end_fixture_matches_f64(ids):  # end_to_end.rs:113-152, :184-217
    got = run_fixture_chain(ids)
    want = expected_fixture_logits(ids)
    assert np.all(np.abs(got.astype(np.float64) - np.array(want)) <= 1e-5)
