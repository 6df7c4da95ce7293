"""The symmetric grouped INT4/INT8 weight format, on CPU. The reference's
quantizer (the sl-precision crate) is absent from the checkout, so the format
is this project's definition (oracle/quant.c); these tests pin the oracle's
implementation of it against the written rules:

- an independent numpy restatement (per-row groups along K, the last one
  ragged; scale = max|w| / qmax in f32; code = w / scale in f32 rounded half
  away from zero and clamped; zero scale -> code 0; INT4 two's-complement
  nibbles with the even k in the low nibble; INT8 one signed byte) agrees
  with the oracle bit for bit, payload and scales;
- hand-worked known answers (rounding ties, packing bytes, a ragged group,
  an all-zero group);
- properties: codes within [-qmax, qmax], the largest |w| of every nonzero
  group quantized to +-qmax, dequantization ((float)code * scale) within half
  a step of w, and dequantize(quantize(dequantize(.))) a fixed point."""
import numpy as np
import pytest

from oracle import pyoracle as orc

QMAX = {orc.INT4: 7, orc.INT8: 127}


def np_quantize(fmt, w, group):
    """The format's rules restated with numpy (f32 arithmetic throughout)."""
    n, k = w.shape
    qmax = np.float32(QMAX[fmt])
    groups = -(-k // group)
    scales = np.zeros((n, groups), np.float32)
    codes = np.zeros((n, k), np.int32)
    for g in range(groups):
        b, e = g * group, min(k, (g + 1) * group)
        seg = w[:, b:e].astype(np.float32)
        s = (np.max(np.abs(seg), axis=1) / qmax).astype(np.float32)
        scales[:, g] = s
        safe = np.where(s == 0, np.float32(1), s).astype(np.float32)
        q = (seg / safe[:, None]).astype(np.float32)
        t = np.trunc(q)
        r = t + np.sign(q) * (np.abs(q - t) >= np.float32(0.5))  # half away from zero
        r = np.clip(r, -qmax, qmax)
        codes[:, b:e] = np.where(s[:, None] == 0, 0, r).astype(np.int32)
    return codes, scales


def np_pack(fmt, codes):
    n, k = codes.shape
    if fmt == orc.INT8:
        return codes.astype(np.int8).view(np.uint8).ravel()
    rb = (k + 1) // 2
    out = np.zeros((n, rb), np.uint8)
    nib = (codes & 0xF).astype(np.uint8)
    out[:, :] = nib[:, 0::2][:, :rb]
    out[:, : k // 2] |= (nib[:, 1::2] << 4).astype(np.uint8)
    return out.ravel()


def _weights(rng, n, k, zero_group=None, group=None):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if zero_group is not None:
        w[:, zero_group * group:(zero_group + 1) * group] = 0
    return w


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("n,k,group", [(4, 256, 128), (3, 688, 32), (5, 33, 8), (2, 7, 4),
                                       (1, 4096, 128)])
def test_oracle_matches_numpy_restatement(fmt, n, k, group):
    rng = np.random.default_rng(k * 31 + n)
    w = _weights(rng, n, k, zero_group=1 if k > 2 * group else None, group=group)
    codes, scales = orc.quantize(fmt, w.ravel(), n, k, group)
    want_codes, want_scales = np_quantize(fmt, w, group)
    assert np.array_equal(scales.view(np.uint32), want_scales.ravel().view(np.uint32))
    assert np.array_equal(codes, np_pack(fmt, want_codes))
    assert np.array_equal(orc.codes_as_int(fmt, codes, n, k), want_codes)


def test_known_answer_int4_packing_and_ties():
    w = np.array([[0.7, -0.35, 0.05, -0.7]], np.float32)
    codes, scales = orc.quantize(orc.INT4, w.ravel(), 1, 4, 4)
    assert scales[0] == np.float32(0.7) / np.float32(7)
    # codes 7, -4 (-3.5 rounds away from zero), 1 (0.5 away from zero), -7:
    # nibbles 0x7, 0xC | 0x1, 0x9, even k low.
    assert list(codes) == [0xC7, 0x91]


def test_known_answer_exact_ties_round_away_from_zero():
    # scale 1.0 exactly: max 7.0 / 7; every quotient is exact.
    w = np.array([[7.0, 2.5, -2.5, 0.5, -0.5, 1.5, -1.5, 6.5]], np.float32)
    codes, scales = orc.quantize(orc.INT4, w.ravel(), 1, 8, 8)
    assert scales[0] == 1.0
    assert list(orc.codes_as_int(orc.INT4, codes, 1, 8).ravel()) == [7, 3, -3, 1, -1, 2, -2, 7]


def test_known_answer_int8_ragged_and_zero_group():
    # k = 6, group 4: groups [0, 4) and the ragged [4, 6); a zero group gives
    # scale 0 and codes 0.
    w = np.array([[1.27, -0.635, 0.01, 0.0, 0.0, 0.0],
                  [0.0, 0.0, 0.0, 0.0, -2.54, 1.27]], np.float32)
    codes, scales = orc.quantize(orc.INT8, w.ravel(), 2, 6, 4)
    s = scales.reshape(2, 2)
    assert s[0, 0] == np.float32(1.27) / np.float32(127) and s[0, 1] == 0
    assert s[1, 0] == 0 and s[1, 1] == np.float32(2.54) / np.float32(127)
    c = orc.codes_as_int(orc.INT8, codes, 2, 6)
    assert list(c[0]) == [127, -64, 1, 0, 0, 0]
    assert list(c[1]) == [0, 0, 0, 0, -127, 64]


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_properties(fmt, seed):
    rng = np.random.default_rng(seed)
    n, k, group = 6, 300, 64
    w = (rng.standard_normal((n, k)) * rng.uniform(0.001, 3.0)).astype(np.float32)
    w[2, 64:128] = 0  # one zero group
    codes, scales = orc.quantize(fmt, w.ravel(), n, k, group)
    c = orc.codes_as_int(fmt, codes, n, k)
    s = scales.reshape(n, -1)
    qmax = QMAX[fmt]
    assert c.min() >= -qmax and c.max() <= qmax
    for r in range(n):
        for g in range(s.shape[1]):
            seg = slice(g * group, min(k, (g + 1) * group))
            if s[r, g] == 0:
                assert not c[r, seg].any()
                continue
            j = int(np.argmax(np.abs(w[r, seg])))
            assert abs(int(c[r, seg][j])) == qmax
    deq = orc.dequantize(fmt, codes, scales, n, k, group).reshape(n, k)
    step = np.repeat(s, group, axis=1)[:, :k]
    assert np.all(np.abs(deq - w) <= 0.5 * step * (1 + 1e-5) + 1e-30)
    # Dequantized weights are a fixed point of quantize -> dequantize.
    codes2, scales2 = orc.quantize(fmt, deq.ravel(), n, k, group)
    deq2 = orc.dequantize(fmt, codes2, scales2, n, k, group)
    assert np.array_equal(codes2, codes)
    assert np.array_equal(deq2.view(np.uint32), deq.ravel().view(np.uint32))
