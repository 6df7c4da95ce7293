"""Helpers shared by the GPU parity tests (not collected as tests).

Tolerances:
  * bit-exact: quantized codes, scales, dequantized weights, copies, KV-cache
    indexing, gathers;
  * f32 elementwise ops: |gpu - ref| <= 1e-5 * |ref| (with a 1e-6 absolute
    floor for results that round to ~0);
  * reductions, matmul and attention: |gpu - ref| <= max(1e-3, 2e-3 * |ref|),
    the looser of 2e-3 relative and 1e-3 absolute.
"""
import numpy as np

from starlight_b200.device import BufferRef, CudaDevice, Op, OpCode, Value, ValueRole

ELEMENTWISE_REL = 1e-5
ELEMENTWISE_ABS = 1e-6
REDUCTION_REL = 2e-3
REDUCTION_ABS = 1e-3


def assert_elementwise(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    err = np.abs(got - want)
    tol = np.maximum(ELEMENTWISE_ABS, ELEMENTWISE_REL * np.abs(want))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first {bad[:4]}: {got[bad[:4]]} vs {want[bad[:4]]}"


def assert_reduction(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    err = np.abs(got - want)
    tol = np.maximum(REDUCTION_ABS, REDUCTION_REL * np.abs(want))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, (f"{bad.size} mismatches, first {bad[:4]}: {got[bad[:4]]} vs "
                           f"{want[bad[:4]]}, max err {err.max()}")
    return float(err.max()) if err.size else 0.0


def put_f32(dev: CudaDevice, arr) -> BufferRef:
    a = np.ascontiguousarray(arr, np.float32).ravel()
    b = dev.allocate_f32(a.size)
    if a.size:
        dev.upload_f32(b, a)
    return BufferRef(b, 0, a.size)


def put_u32(dev: CudaDevice, arr) -> BufferRef:
    a = np.ascontiguousarray(arr, np.uint32).ravel()
    b = dev.allocate_u32(a.size)
    if a.size:
        dev.upload_u32(b, a)
    return BufferRef(b, 0, a.size)


def new_f32(dev: CudaDevice, n: int, fill=None) -> BufferRef:
    b = dev.allocate_f32(n)
    if fill is not None and n:
        dev.upload_f32(b, np.full(n, fill, np.float32))
    return BufferRef(b, 0, n)


def get(dev: CudaDevice, ref: BufferRef) -> np.ndarray:
    dev.synchronize()
    if ref.len == 0:
        return np.zeros(0, np.float32)
    full = dev.download_f32(ref.buffer)
    return full[ref.offset:ref.offset + ref.len]


def put_quant(dev: CudaDevice, codes: np.ndarray, scales: np.ndarray, fmt, group):
    """Uploads a payload (bytes) and scales; returns (codes_buffer, scales_buffer, words)."""
    raw = np.ascontiguousarray(codes, np.uint8).ravel()
    words = (raw.size + 3) // 4
    padded = np.zeros(words * 4, np.uint8)
    padded[:raw.size] = raw
    cb = dev.allocate_u32(words)
    dev.upload_u32(cb, padded.view(np.uint32))
    sb = dev.allocate_f32(scales.size)
    dev.upload_f32(sb, scales)
    dev.bind_quant(cb, sb, fmt, group)
    return cb, sb, words
