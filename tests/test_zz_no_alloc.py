"""slc_qmatmul_noalloc, the quantized matmul whose scratch is a fixed array in
the library, against the existing entry point (slc_dispatch of MatMulNT on a
GroupwiseQuantized weight): two calls in a row on the same inputs must each
match it within the matmul tolerance of tests/gpu_util.py, and a problem
whose scratch would not fit is rejected before anything is launched.

The file name sorts last so that it also runs after every other GPU test in
the same process; it passes alone as well."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as orc
from oracle.pyoracle import Lcg
from starlight_b200 import device as D
from starlight_b200.device import BufferRef, CudaDevice, Op, OpCode, QuantFormat, Status, Value
from tests.gpu_util import assert_reduction, get, new_f32, put_f32, put_quant

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 << 20  # SLC_NOALLOC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def dev():
    d = CudaDevice(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def noalloc():
    lib = C.CDLL(D.library_path())
    fn = lib.slc_qmatmul_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64,
                   C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.POINTER(C.c_char_p)]

    def call(x, m, codes, scales, n, k, fmt, group, out, stream):
        msg = C.c_char_p()
        rc = fn(x, m, codes, scales, n, k, int(fmt), group, out, stream, C.byref(msg))
        return rc, (msg.value.decode() if msg.value else None)

    return call


def _setup(dev, fmt, m, k, n, group, seed):
    lcg = Lcg(seed)
    w = lcg.normal(n * k, 0.0, 0.02)
    x = lcg.normal(m * k, 0.0, 1.0)
    codes, scales = orc.quantize(fmt, w, n, k, group)
    qf = QuantFormat.Int4 if fmt == orc.INT4 else QuantFormat.Int8
    cb, sb, words = put_quant(dev, codes, scales, qf, group)
    xr = put_f32(dev, x)
    return qf, xr, cb, sb, words


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("m,k,n,group", [(1, 4096, 4096, 128), (8, 4096, 1024, 128),
                                         (32, 4096, 4096, 128), (40, 1024, 4096, 128),
                                         (3, 100, 48, 7), (100, 512, 256, 64)])
def test_noalloc_matches_dispatch_twice(dev, noalloc, fmt, m, k, n, group):
    qf, xr, cb, sb, words = _setup(dev, fmt, m, k, n, group, seed=m * 7 + k + n + group)
    want = new_f32(dev, m * n)
    dev.dispatch(Op(OpCode.MatMulNT), [xr, BufferRef(cb, 0, words)],
                 [Value.f32((1, m, k)), Value.quantized((n, k), qf, group)], [want],
                 [Value.f32((1, m, n))])
    ref = get(dev, want)

    outs = [new_f32(dev, m * n, fill=np.nan), new_f32(dev, m * n, fill=np.nan)]
    dev.synchronize()
    stream = dev.stream()
    for out in outs:  # two calls in a row, no synchronize between them
        rc, msg = noalloc(dev.device_ptr(xr.buffer), m, dev.device_ptr(cb), dev.device_ptr(sb),
                          n, k, qf, group, dev.device_ptr(out.buffer), stream)
        assert rc == Status.Ok, msg
    first, second = get(dev, outs[0]), get(dev, outs[1])
    assert_reduction(first, ref)
    assert_reduction(second, ref)
    # The reduction order is fixed, so both calls agree exactly.
    assert np.array_equal(first, second)


def test_noalloc_rejects_scratch_beyond_the_array(dev, noalloc):
    # m = 32, k = 256 (two groups of 128), n = 295 * 128 rows: the decode GEMV
    # splits K in two, so the partial sums alone need 2 * 32 * n * 4 bytes.
    m, k, n, group = 32, 256, 295 * 128, 128
    assert 2 * m * n * 4 > SCRATCH_BYTES
    qf, xr, cb, sb, words = _setup(dev, orc.INT4, m, k, n, group, seed=3)
    out = new_f32(dev, m * n, fill=7.0)
    dev.synchronize()
    rc, msg = noalloc(dev.device_ptr(xr.buffer), m, dev.device_ptr(cb), dev.device_ptr(sb), n, k,
                      qf, group, dev.device_ptr(out.buffer), dev.stream())
    assert rc == Status.OutOfMemory
    assert "SLC_NOALLOC_SCRATCH_BYTES" in msg
    assert np.all(get(dev, out) == 7.0)  # nothing was launched


def test_noalloc_argument_errors(dev, noalloc):
    qf, xr, cb, sb, words = _setup(dev, orc.INT8, 1, 64, 16, 32, seed=4)
    out = new_f32(dev, 16)
    args = (dev.device_ptr(xr.buffer), 1, dev.device_ptr(cb), dev.device_ptr(sb), 16, 64)
    rc, msg = noalloc(*args, 9, 32, dev.device_ptr(out.buffer), dev.stream())
    assert rc == Status.Unimplemented and "format" in msg
    rc, msg = noalloc(*args, qf, 0, dev.device_ptr(out.buffer), dev.stream())
    assert rc == Status.Execution and "group" in msg
    rc, msg = noalloc(*args, qf, 32, None, dev.stream())
    assert rc == Status.Execution and "null" in msg
    rc, msg = noalloc(args[0], 0, args[2], args[3], 16, 64, qf, 32, None, dev.stream())
    assert rc == Status.Ok and msg is None  # m = 0: nothing to compute
