"""Python view of backend-cuda's C ABI (include/starlight_cuda.h).

`CudaDevice` mirrors the `sl_device::Device` trait (docs/ARCH-0007 section
3.1; CPU implementation crates/backends/backend-cpu/src/device.rs:114-213):
allocate_f32/u32, upload_*/download_*, dispatch, synchronize, with the same
argument meaning. Errors raise `DeviceError` carrying the DeviceError variant
and payload. The types `DType`, `ValueRole`, `Value`, `Op`, `BufferRef`
mirror sl-ir (docs/ARCH-0004 sections 3 and 5).

This module loads the compiled library and nothing else: there is no CPU
fallback. Without the library (or without a CUDA device) every entry point
fails loudly.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libslc.so")

MAX_RANK = 8
MIN_BUFFER_ALIGN = 64
IR_VERSION = 2


class DType(enum.IntEnum):  # docs/ARCH-0004:82
    F32 = 0
    F16 = 1
    BF16 = 2
    U32 = 3
    I32 = 4
    U8 = 5
    I8 = 6


class ValueRole(enum.IntEnum):  # docs/ARCH-0004:104-111
    Input = 0
    Scalar = 1
    Output = 2
    Param = 3
    State = 4
    Temp = 5


class Encoding(enum.IntEnum):  # docs/ARCH-0004:120-131
    Dense = 0
    Groupwise = 1
    Opaque = 2


class QuantFormat(enum.IntEnum):
    Int4 = 0
    Int8 = 1


class OpCode(enum.IntEnum):  # docs/ARCH-0004:226-235, #[repr(u16)] order
    MatMulNT = 0
    MatMulNN = 1
    Softmax = 2
    SoftmaxCausal = 3
    RmsNorm = 4
    Rope = 5
    Silu = 6
    Mul = 7
    Add = 8
    Scale = 9
    Gather = 10
    LastToken = 11
    KvAppend = 12
    SplitHeads = 13
    MergeHeads = 14
    CausalAttention = 15
    SwiGlu = 16
    RmsNormMatMul = 17
    AllReduce = 0x8000  # extension: tensor-parallel sum
    AllGather = 0x8001  # extension: tensor-parallel gather of column blocks
    AddBias = 0x8002  # extension: (a + b) + bias[col], bias broadcast over rows


class RopeVariant(enum.IntEnum):
    Neox = 0
    GptJ = 1


class Status(enum.IntEnum):  # DeviceError variants, docs/ARCH-0007:63-71
    Ok = 0
    OutOfMemory = 1
    InvalidBuffer = 2
    InvalidRange = 3
    UnsupportedOp = 4
    ShapeOverflow = 5
    Execution = 6
    Unimplemented = 7


# ---------------------------------------------------------------- structs --

class _Value(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("role", C.c_uint32), ("rank", C.c_uint32),
                ("dims", C.c_uint32 * MAX_RANK), ("encoding", C.c_uint32),
                ("quant_format", C.c_uint32), ("group_size", C.c_uint32)]


class _BufferRef(C.Structure):
    _fields_ = [("buffer", C.c_uint32), ("reserved", C.c_uint32), ("offset", C.c_uint64),
                ("len", C.c_uint64)]


class _Op(C.Structure):
    _fields_ = [("code", C.c_uint16), ("rope_variant", C.c_uint16), ("layer", C.c_uint32),
                ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("eps", C.c_float), ("theta", C.c_float), ("scale", C.c_float),
                ("factor", C.c_float)]


class _Error(C.Structure):
    _fields_ = [("status", C.c_int32), ("buffer", C.c_uint32), ("offset", C.c_uint64),
                ("len", C.c_uint64), ("requested", C.c_uint64), ("opcode", C.c_uint32),
                ("message", C.c_char_p)]


class _Caps(C.Structure):
    _fields_ = [("ir_version", C.c_uint32), ("core_ops", C.c_uint64),
                ("composite_ops", C.c_uint64), ("dtypes", C.c_uint32),
                ("min_buffer_align", C.c_uint32), ("max_scratchpad_bytes", C.c_uint64),
                ("max_value_bytes", C.c_uint64), ("head_dim_multiple_of", C.c_uint32),
                ("matmul_k_multiple_of", C.c_uint32), ("max_heads", C.c_uint32),
                ("quant_formats", C.c_uint32)]


class _CaptureInfo(C.Structure):
    _fields_ = [("captures", C.c_uint64), ("replays", C.c_uint64),
                ("replayed_commands", C.c_uint64), ("eager_commands", C.c_uint64)]


class _FusionInfo(C.Structure):
    _fields_ = [("launched", C.c_uint64), ("refused", C.c_uint64), ("last_ms", C.c_float),
                ("reserved", C.c_float)]


class _Options(C.Structure):
    _fields_ = [("workspace_bytes", C.c_uint64), ("staging_bytes", C.c_uint64)]


# ------------------------------------------------------------ public types --

@dataclass(frozen=True)
class BufferRef:
    """sl_device::BufferRef: `len` elements at element `offset` of `buffer`."""
    buffer: int
    offset: int
    len: int


@dataclass(frozen=True)
class Value:
    """sl_ir::Value with a constant shape."""
    dtype: DType
    shape: tuple
    role: ValueRole
    encoding: Encoding = Encoding.Dense
    quant_format: QuantFormat = QuantFormat.Int4
    group_size: int = 0

    @staticmethod
    def f32(shape, role=ValueRole.Temp):
        return Value(DType.F32, tuple(shape), role)

    @staticmethod
    def u32(shape, role=ValueRole.Input):
        return Value(DType.U32, tuple(shape), role)

    @staticmethod
    def quantized(shape, fmt: QuantFormat, group: int):
        return Value(DType.F32, tuple(shape), ValueRole.Param, Encoding.Groupwise, fmt, group)

    def element_count(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    def _c(self) -> _Value:
        v = _Value()
        v.dtype = int(self.dtype)
        v.role = int(self.role)
        v.rank = len(self.shape)
        for i, d in enumerate(self.shape[:MAX_RANK]):
            v.dims[i] = int(d)
        v.encoding = int(self.encoding)
        v.quant_format = int(self.quant_format)
        v.group_size = int(self.group_size)
        return v


@dataclass(frozen=True)
class Op:
    """sl_ir::Op: opcode plus the attributes of its variant."""
    code: OpCode
    layer: int = 0
    heads: int = 0
    kv_heads: int = 0
    head_dim: int = 0
    eps: float = 0.0
    theta: float = 0.0
    scale: float = 0.0
    factor: float = 0.0
    variant: RopeVariant = RopeVariant.Neox

    def _c(self) -> _Op:
        o = _Op()
        o.code = int(self.code)
        o.rope_variant = int(self.variant)
        o.layer, o.heads, o.kv_heads, o.head_dim = self.layer, self.heads, self.kv_heads, self.head_dim
        o.eps, o.theta, o.scale, o.factor = self.eps, self.theta, self.scale, self.factor
        return o


class DeviceError(Exception):
    """sl_device::DeviceError (docs/ARCH-0007:63-71)."""

    def __init__(self, status: int, message: str | None = None, buffer=None, offset=None,
                 length=None, requested=None, opcode=None):
        self.status = Status(status) if status in Status._value2member_map_ else status
        self.message = message
        self.buffer, self.offset, self.len = buffer, offset, length
        self.requested, self.opcode = requested, opcode
        super().__init__(f"{getattr(self.status, 'name', self.status)}: {message}")


# ------------------------------------------------------------------- lib --

_lib = None


def library_path() -> str:
    return LIB_PATH


def load_library():
    """Loads libslc.so (built in-tree by starlight_b200.build). Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"backend-cuda library not built: {LIB_PATH} "
                           "(run python -m starlight_b200.build)")
    lib = C.CDLL(LIB_PATH)
    P = C.c_void_p
    sig = {
        "slc_device_create": (C.c_int, [C.c_int, C.POINTER(P)]),
        "slc_device_create_ex": (C.c_int, [C.c_int, C.POINTER(_Options), C.POINTER(P)]),
        "slc_device_destroy": (None, [P]),
        "slc_last_error": (C.c_int, [P, C.POINTER(_Error)]),
        "slc_get_capabilities": (C.c_int, [P, C.POINTER(_Caps)]),
        "slc_status_name": (C.c_char_p, [C.c_int]),
        "slc_allocate_f32": (C.c_int, [P, C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32)]),
        "slc_allocate_u32": (C.c_int, [P, C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32)]),
        "slc_upload_f32": (C.c_int, [P, C.c_uint32, P, C.c_uint64]),
        "slc_upload_u32": (C.c_int, [P, C.c_uint32, P, C.c_uint64]),
        "slc_download_f32": (C.c_int, [P, C.c_uint32, P, C.c_uint64]),
        "slc_download_u32": (C.c_int, [P, C.c_uint32, P, C.c_uint64]),
        "slc_dispatch": (C.c_int, [P, C.POINTER(_Op), C.POINTER(_BufferRef), C.POINTER(_Value),
                                   C.c_uint64, C.POINTER(_BufferRef), C.POINTER(_Value),
                                   C.c_uint64, C.POINTER(C.c_uint32), C.c_uint64]),
        "slc_synchronize": (C.c_int, [P]),
        "slc_bind_quant": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
        "slc_quantize": (C.c_int, [P, _BufferRef, C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32,
                                   C.c_uint32, C.c_uint32]),
        "slc_dequantize": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint64,
                                     C.c_uint32, C.c_uint32, _BufferRef]),
        "slc_copy_f32_from_device": (C.c_int, [P, C.c_uint32, C.c_uint64, P, C.c_uint64]),
        "slc_buffer_device_ptr": (C.c_int, [P, C.c_uint32, C.POINTER(P)]),
        "slc_release": (C.c_int, [P, C.c_uint32]),
        "slc_fill_normal": (C.c_int, [P, _BufferRef, C.c_uint64, C.c_uint64, C.c_float,
                                      C.c_float]),
        "slc_device_stream": (C.c_int, [P, C.POINTER(P)]),
        "slc_kernel_launch_count": (C.c_uint64, [P]),
        "slc_set_capture": (C.c_int, [P, C.c_int]),
        "slc_flush": (C.c_int, [P]),
        "slc_capture_stats": (C.c_int, [P, C.POINTER(_CaptureInfo)]),
        "slc_decode_fusion_stats": (C.c_int, [P, C.POINTER(_FusionInfo)]),
        "slc_comm_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
        "slc_comm_init": (C.c_int, [P, C.POINTER(C.c_uint8), C.c_int, C.c_int]),
        "slc_comm_world": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "slc_comm_peer_status": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "slc_comm_async_error": (C.c_int, [P]),
        "slc_comm_abort": (C.c_int, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols():
    """Names of the C entry points this module binds (all declared in include/*.h)."""
    return ["slc_device_create", "slc_device_create_ex", "slc_device_destroy", "slc_last_error",
            "slc_get_capabilities", "slc_status_name", "slc_allocate_f32", "slc_allocate_u32",
            "slc_upload_f32", "slc_upload_u32", "slc_download_f32", "slc_download_u32",
            "slc_dispatch", "slc_synchronize", "slc_bind_quant", "slc_quantize",
            "slc_dequantize", "slc_copy_f32_from_device", "slc_buffer_device_ptr", "slc_release",
            "slc_fill_normal",
            "slc_device_stream", "slc_kernel_launch_count", "slc_set_capture", "slc_flush",
            "slc_capture_stats", "slc_decode_fusion_stats",
            "slc_comm_unique_id", "slc_comm_init", "slc_comm_world", "slc_comm_peer_status",
            "slc_comm_async_error", "slc_comm_abort"]


def _ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data) if a.size else None


class CudaDevice:
    """backend-cuda device on one GPU (the `impl Device` of the ABI)."""

    def __init__(self, ordinal: int = 0, workspace_bytes: int = 0, staging_bytes: int = 0):
        self._lib = load_library()
        self._d = C.c_void_p()
        opt = _Options(workspace_bytes, staging_bytes)
        rc = self._lib.slc_device_create_ex(ordinal, C.byref(opt), C.byref(self._d))
        if rc != 0:
            raise DeviceError(rc, f"slc_device_create({ordinal}) failed")
        self._sizes = {}

    @property
    def handle(self):
        return self._d

    def close(self):
        if self._d:
            self._lib.slc_device_destroy(self._d)
            self._d = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc == 0:
            return
        e = _Error()
        self._lib.slc_last_error(self._d, C.byref(e))
        raise DeviceError(rc, e.message.decode() if e.message else None, e.buffer, e.offset,
                          e.len, e.requested, e.opcode)

    # -- Device trait ------------------------------------------------------
    def allocate_f32(self, elements: int, align: int = MIN_BUFFER_ALIGN) -> int:
        out = C.c_uint32()
        self._check(self._lib.slc_allocate_f32(self._d, elements, align, C.byref(out)))
        self._sizes[out.value] = (elements, np.float32)
        return out.value

    def allocate_u32(self, elements: int, align: int = MIN_BUFFER_ALIGN) -> int:
        out = C.c_uint32()
        self._check(self._lib.slc_allocate_u32(self._d, elements, align, C.byref(out)))
        self._sizes[out.value] = (elements, np.uint32)
        return out.value

    def upload_f32(self, buffer: int, data) -> None:
        a = np.ascontiguousarray(data, np.float32).ravel()
        self._check(self._lib.slc_upload_f32(self._d, buffer, _ptr(a), a.size))

    def upload_u32(self, buffer: int, data) -> None:
        a = np.ascontiguousarray(data, np.uint32).ravel()
        self._check(self._lib.slc_upload_u32(self._d, buffer, _ptr(a), a.size))

    def download_f32(self, buffer: int, length: int | None = None) -> np.ndarray:
        n = self._sizes[buffer][0] if length is None else length
        out = np.empty(n, np.float32)
        self._check(self._lib.slc_download_f32(self._d, buffer, _ptr(out), n))
        return out

    def download_u32(self, buffer: int, length: int | None = None) -> np.ndarray:
        n = self._sizes[buffer][0] if length is None else length
        out = np.empty(n, np.uint32)
        self._check(self._lib.slc_download_u32(self._d, buffer, _ptr(out), n))
        return out

    def dispatch(self, op: Op, inputs: Sequence[BufferRef], input_values: Sequence[Value],
                 outputs: Sequence[BufferRef], output_values: Sequence[Value],
                 scalars: Sequence[int] = ()) -> None:
        ni, no, ns = len(inputs), len(outputs), len(scalars)
        if ni != len(input_values) or no != len(output_values):
            raise DeviceError(Status.Execution, "inputs and input_values have different lengths")
        ir = (_BufferRef * max(ni, 1))(*[_BufferRef(r.buffer, 0, r.offset, r.len) for r in inputs])
        iv = (_Value * max(ni, 1))(*[v._c() for v in input_values])
        orf = (_BufferRef * max(no, 1))(*[_BufferRef(r.buffer, 0, r.offset, r.len) for r in outputs])
        ov = (_Value * max(no, 1))(*[v._c() for v in output_values])
        sc = (C.c_uint32 * max(ns, 1))(*[int(s) for s in scalars])
        o = op._c()
        self._check(self._lib.slc_dispatch(self._d, C.byref(o), ir, iv, ni, orf, ov, no, sc, ns))

    def synchronize(self) -> None:
        self._check(self._lib.slc_synchronize(self._d))

    # -- extensions --------------------------------------------------------
    def capabilities(self) -> dict:
        c = _Caps()
        self._check(self._lib.slc_get_capabilities(self._d, C.byref(c)))
        return {f: getattr(c, f) for f, _ in _Caps._fields_}

    def bind_quant(self, codes_buffer: int, scales_buffer: int, fmt: QuantFormat, group: int):
        self._check(self._lib.slc_bind_quant(self._d, codes_buffer, scales_buffer, int(fmt), group))

    def quantize(self, weights: BufferRef, rows: int, k: int, fmt: QuantFormat, group: int,
                 codes_buffer: int, scales_buffer: int):
        self._check(self._lib.slc_quantize(self._d, _BufferRef(weights.buffer, 0, weights.offset,
                                                               weights.len), rows, k, int(fmt),
                                           group, codes_buffer, scales_buffer))

    def dequantize(self, codes_buffer: int, scales_buffer: int, rows: int, k: int,
                   fmt: QuantFormat, group: int, out: BufferRef):
        self._check(self._lib.slc_dequantize(self._d, codes_buffer, scales_buffer, rows, k,
                                             int(fmt), group,
                                             _BufferRef(out.buffer, 0, out.offset, out.len)))

    def copy_f32_from_device(self, buffer: int, offset: int, device_ptr: int, length: int):
        self._check(self._lib.slc_copy_f32_from_device(self._d, buffer, offset,
                                                       C.c_void_p(device_ptr), length))

    def fill_normal(self, ref: BufferRef, seed: int, offset: int = 0, mean: float = 0.0,
                    std: float = 1.0):
        """Fills an F32 ref with N(mean, std) draws (synthetic data on the device)."""
        self._check(self._lib.slc_fill_normal(self._d, _BufferRef(ref.buffer, 0, ref.offset, ref.len),
                                              seed, offset, mean, std))

    def release(self, buffer: int):
        """Frees a buffer's device memory (its BufferId becomes invalid)."""
        self._check(self._lib.slc_release(self._d, buffer))

    def device_ptr(self, buffer: int) -> int:
        p = C.c_void_p()
        self._check(self._lib.slc_buffer_device_ptr(self._d, buffer, C.byref(p)))
        return p.value or 0

    def stream(self) -> int:
        p = C.c_void_p()
        self._check(self._lib.slc_device_stream(self._d, C.byref(p)))
        return p.value or 0

    def launch_count(self) -> int:
        return int(self._lib.slc_kernel_launch_count(self._d))

    def set_capture(self, enabled: bool):
        """Command capture and CUDA-graph replay (include/starlight_cuda.h)."""
        self._check(self._lib.slc_set_capture(self._d, 1 if enabled else 0))

    def flush(self):
        """Submits deferred (captured) work without waiting for it."""
        self._check(self._lib.slc_flush(self._d))

    def capture_stats(self) -> dict:
        info = _CaptureInfo()
        self._check(self._lib.slc_capture_stats(self._d, C.byref(info)))
        return {f: int(getattr(info, f)) for f, _ in _CaptureInfo._fields_}

    def decode_fusion_stats(self) -> dict:
        """Persistent decode-layer launches enqueued / refused and the device
        time (ms, from the kernel's global-timer stamps) of the latest one;
        waits for the device stream."""
        info = _FusionInfo()
        self._check(self._lib.slc_decode_fusion_stats(self._d, C.byref(info)))
        return {"launched": int(info.launched), "refused": int(info.refused),
                "last_ms": float(info.last_ms)}

    def peer_status(self) -> dict:
        """Peer-memory paths agreed by all ranks at comm_init: the fused
        all-reduce + Add + RmsNorm kernel and persistent decode-layer fusion."""
        a, b = C.c_int(0), C.c_int(0)
        self._check(self._lib.slc_comm_peer_status(self._d, C.byref(a), C.byref(b)))
        return {"peer_allreduce": bool(a.value), "decode_fusion": bool(b.value)}

    def comm_check(self):
        """Raises DeviceError if the communicator reported an asynchronous
        error or was aborted."""
        self._check(self._lib.slc_comm_async_error(self._d))

    def comm_abort(self):
        """Tears the communicator down without the other ranks (a peer left):
        later collectives fail instead of waiting."""
        self._check(self._lib.slc_comm_abort(self._d))

    def comm_init(self, unique_id: bytes, rank: int, world: int):
        buf = (C.c_uint8 * 128)(*unique_id)
        self._check(self._lib.slc_comm_init(self._d, buf, rank, world))


def comm_unique_id() -> bytes:
    lib = load_library()
    buf = (C.c_uint8 * 128)()
    rc = lib.slc_comm_unique_id(buf)
    if rc != 0:
        raise DeviceError(rc, "slc_comm_unique_id failed")
    return bytes(buf)


def quant_storage_words(rows: int, k: int, fmt: QuantFormat) -> int:
    """u32 words of a packed payload [rows, k] (INT4: ceil(k/2) bytes per row)."""
    row_bytes = (k + 1) // 2 if fmt == QuantFormat.Int4 else k
    return (rows * row_bytes + 3) // 4


def quant_groups(k: int, group: int) -> int:
    return (k + group - 1) // group
