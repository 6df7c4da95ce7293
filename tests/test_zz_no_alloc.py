"""slc_qmatmul_noalloc, the quantized matmul for callers that cannot allocate
device memory (a host whose own pool or caching allocator owns the GPU, a
fixed memory budget, a latency loop in which cudaMalloc would synchronize the
device). Its scratch is a fixed array inside the library, so the test checks:

  * two calls in a row on the same inputs each match the CPU oracle
    (dequantize, then an f64 matmul) within the matmul tolerance of
    tests/gpu_util.py, and agree with each other bit for bit;
  * decode-sized (m <= 64, split-K tickets and partial sums in the array)
    and prefill-sized (m > 64, the tcgen05 GEMM's activation planes in the
    array) problems, and a prefill-sized call between two decode calls;
  * the caller's error word stays zero (no bounded wait gave up);
  * a problem whose scratch would not fit is rejected before anything runs.

The file name sorts last so that, in a run that stops at the first failure,
every other test has already run; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as orc
from oracle.pyoracle import Lcg
from starlight_b200 import device as D
from starlight_b200.device import CudaDevice, QuantFormat, Status
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
                   C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                   C.POINTER(C.c_char_p)]

    def call(x, m, codes, scales, n, k, fmt, group, out, stream, err_word=None):
        msg = C.c_char_p()
        rc = fn(x, m, codes, scales, n, k, int(fmt), group, out, stream, err_word, C.byref(msg))
        return rc, (msg.value.decode() if msg.value else None)

    return call


class Case:
    """Seeded weights and activations on the device, plus the oracle result."""

    def __init__(self, dev, fmt, m, k, n, group, seed):
        lcg = Lcg(seed)
        w = lcg.normal(n * k, 0.0, 0.02)
        x = lcg.normal(m * k, 0.0, 1.0)
        codes, scales = orc.quantize(fmt, w, n, k, group)
        self.qf = QuantFormat.Int4 if fmt == orc.INT4 else QuantFormat.Int8
        self.cb, self.sb, _ = put_quant(dev, codes, scales, self.qf, group)
        self.xr = put_f32(dev, x)
        self.m, self.k, self.n, self.group = m, k, n, group
        wd = orc.dequantize(fmt, codes, scales, n, k, group).reshape(n, k)
        self.want = (x.reshape(m, k).astype(np.float64) @ wd.astype(np.float64).T).ravel()

    def run(self, dev, noalloc, out, err_word):
        return noalloc(dev.device_ptr(self.xr.buffer), self.m, dev.device_ptr(self.cb),
                       dev.device_ptr(self.sb), self.n, self.k, self.qf, self.group,
                       dev.device_ptr(out.buffer), dev.stream(), err_word)


def _error_word(dev):
    """A zeroed 4-byte word in device memory for the kernels' error code."""
    ref = new_f32(dev, 1, fill=0.0)
    return ref, dev.device_ptr(ref.buffer)


def _error_code(dev, ref):
    return int(get(dev, ref).view(np.uint32)[0])


@pytest.mark.parametrize("fmt", [orc.INT4, orc.INT8])
@pytest.mark.parametrize("m,k,n,group", [(1, 4096, 4096, 128), (8, 4096, 1024, 128),
                                         (32, 4096, 4096, 128), (40, 1024, 4096, 128),
                                         (3, 100, 48, 7), (100, 512, 256, 64),
                                         (300, 1024, 512, 128)])
def test_noalloc_matches_oracle_twice(dev, noalloc, fmt, m, k, n, group):
    case = Case(dev, fmt, m, k, n, group, seed=m * 7 + k + n + group)
    err_ref, err_ptr = _error_word(dev)
    outs = [new_f32(dev, m * n, fill=np.nan), new_f32(dev, m * n, fill=np.nan)]
    dev.synchronize()
    for out in outs:  # two calls in a row, no synchronize between them
        rc, msg = case.run(dev, noalloc, out, err_ptr)
        assert rc == Status.Ok, msg
    first, second = get(dev, outs[0]), get(dev, outs[1])
    assert_reduction(first, case.want)
    assert_reduction(second, case.want)
    # The reduction order is fixed, so both calls agree exactly.
    assert np.array_equal(first, second)
    assert _error_code(dev, err_ref) == 0


def test_noalloc_prefill_call_between_decode_calls(dev, noalloc):
    """A prefill-sized call fills the array behind the tickets with activation
    planes; decode calls before and after it (split-K partial sums in the
    same bytes) still match the oracle."""
    dec = Case(dev, orc.INT4, 4, 4096, 1024, 128, seed=11)
    pre = Case(dev, orc.INT4, 256, 4096, 1024, 128, seed=12)
    err_ref, err_ptr = _error_word(dev)
    o1, o2 = new_f32(dev, 4 * 1024, fill=np.nan), new_f32(dev, 4 * 1024, fill=np.nan)
    op = new_f32(dev, 256 * 1024, fill=np.nan)
    dev.synchronize()
    before = dev.launch_count()
    assert dec.run(dev, noalloc, o1, err_ptr)[0] == Status.Ok
    mid = dev.launch_count()
    assert pre.run(dev, noalloc, op, err_ptr)[0] == Status.Ok
    # The prefill-sized call runs the tcgen05 GEMM: one activation split and
    # one GEMM launch (one pass: 256 rows of 16 KiB of planes fit the array).
    assert dev.launch_count() - mid == 2
    assert dec.run(dev, noalloc, o2, err_ptr)[0] == Status.Ok
    assert mid > before
    assert_reduction(get(dev, o1), dec.want)
    assert_reduction(get(dev, op), pre.want)
    assert np.array_equal(get(dev, o1), get(dev, o2))
    assert _error_code(dev, err_ref) == 0


def test_noalloc_rejects_scratch_beyond_the_array(dev, noalloc):
    # m = 32, k = 256 (two groups of 128), n = 295 * 128 rows: the decode GEMV
    # splits K in two, so the partial sums alone need 2 * 32 * n * 4 bytes.
    m, k, n, group = 32, 256, 295 * 128, 128
    assert 2 * m * n * 4 > SCRATCH_BYTES
    case = Case(dev, orc.INT4, m, k, n, group, seed=3)
    out = new_f32(dev, m * n, fill=7.0)
    dev.synchronize()
    rc, msg = case.run(dev, noalloc, out, None)
    assert rc == Status.OutOfMemory
    assert "SLC_NOALLOC_SCRATCH_BYTES" in msg
    assert np.all(get(dev, out) == 7.0)  # nothing was launched


def test_noalloc_argument_errors(dev, noalloc):
    case = Case(dev, orc.INT8, 1, 64, 16, 32, seed=4)
    out = new_f32(dev, 16)
    args = (dev.device_ptr(case.xr.buffer), 1, dev.device_ptr(case.cb), dev.device_ptr(case.sb),
            16, 64)
    rc, msg = noalloc(*args, 9, 32, dev.device_ptr(out.buffer), dev.stream())
    assert rc == Status.Unimplemented and "format" in msg
    rc, msg = noalloc(*args, case.qf, 0, dev.device_ptr(out.buffer), dev.stream())
    assert rc == Status.Execution and "group" in msg
    rc, msg = noalloc(*args, case.qf, 32, None, dev.stream())
    assert rc == Status.Execution and "null" in msg
    rc, msg = noalloc(args[0], 0, args[2], args[3], 16, 64, case.qf, 32, None, dev.stream())
    assert rc == Status.Ok and msg is None  # m = 0: nothing to compute
