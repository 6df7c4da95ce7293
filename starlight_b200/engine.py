"""Python view of the llama-dense engine (include/starlight_engine.h).

`Llama` wraps slc_llama_*: the sl-core::Engine contract (docs/ARCH-0007
section 3.2) over backend-cuda, with the llama-dense lowering of
docs/ARCH-0006. All computation happens in libslc.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from .device import (BufferRef, CudaDevice, DeviceError, DType, Encoding, QuantFormat, Value,
                     ValueRole, _BufferRef, _Value, load_library)

ROLES = ("embed", "attn_norm", "q", "k", "v", "o", "mlp_norm", "gate", "up", "down",
         "final_norm", "lm_head")
LAYER_ROLES = ROLES[1:10]
PREFILL, DECODE = 0, 1


# Tensor-parallel layout of every weight role (the engine's add_weight in
# starlight_b200/csrc/engine.cpp): 0 replicated, 1 split by output rows
# (q, k, v, gate, up, lm_head: column-parallel matmuls), 2 split by input
# columns (o, down: row-parallel matmuls followed by an all-reduce).
SHARDING = {"embed": 0, "attn_norm": 0, "q": 1, "k": 1, "v": 1, "o": 2, "mlp_norm": 0,
            "gate": 1, "up": 1, "down": 2, "final_norm": 0, "lm_head": 1}


def full_shape(cfg: "LlamaConfig", role: str) -> tuple:
    """Unsharded [rows, cols] of a weight role."""
    H, D = cfg.hidden, cfg.head_dim
    return {"embed": (cfg.vocab, H), "attn_norm": (1, H), "q": (cfg.heads * D, H),
            "k": (cfg.kv_heads * D, H), "v": (cfg.kv_heads * D, H), "o": (H, cfg.heads * D),
            "mlp_norm": (1, H), "gate": (cfg.inter, H), "up": (cfg.inter, H),
            "down": (H, cfg.inter), "final_norm": (1, H), "lm_head": (cfg.vocab, H)}[role]


def shard_plan(cfg: "LlamaConfig", role: str, rank: int, world: int) -> tuple:
    """(row0, rows, col0, cols) of `rank`'s shard of a weight role."""
    fr, fc = full_shape(cfg, role)
    kind = SHARDING[role]
    rows = fr // world if kind == 1 else fr
    cols = fc // world if kind == 2 else fc
    return (rank * rows if kind == 1 else 0, rows, rank * cols if kind == 2 else 0, cols)


class _Config(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("hidden", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("inter", C.c_uint32),
                ("vocab", C.c_uint32), ("batch", C.c_uint32), ("prefill_len", C.c_uint32),
                ("max_seq", C.c_uint32), ("eps", C.c_float), ("theta", C.c_float),
                ("quant_format", C.c_int32), ("group_size", C.c_uint32), ("tp_rank", C.c_int32),
                ("tp_world", C.c_int32), ("decompose_swiglu", C.c_uint32)]


@dataclass
class LlamaConfig:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    batch: int = 1
    prefill_len: int = 16
    max_seq: int = 32
    eps: float = 1e-5
    theta: float = 10000.0
    quant: QuantFormat | None = QuantFormat.Int4
    group_size: int = 32
    tp_rank: int = 0
    tp_world: int = 1
    decompose_swiglu: bool = False

    def _c(self) -> _Config:
        return _Config(self.layers, self.hidden, self.heads, self.kv_heads, self.head_dim,
                       self.inter, self.vocab, self.batch, self.prefill_len, self.max_seq,
                       self.eps, self.theta, -1 if self.quant is None else int(self.quant),
                       self.group_size, self.tp_rank, self.tp_world,
                       1 if self.decompose_swiglu else 0)

    def role_shape(self, role: str):
        H, Q, KV = self.hidden, self.heads * self.head_dim, self.kv_heads * self.head_dim
        return {"embed": (self.vocab, H), "attn_norm": (H,), "mlp_norm": (H,), "final_norm": (H,),
                "q": (Q, H), "k": (KV, H), "v": (KV, H), "o": (H, Q), "gate": (self.inter, H),
                "up": (self.inter, H), "down": (H, self.inter), "lm_head": (self.vocab, H)}[role]


# The BASELINE configurations.
FIXTURE = LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=4, head_dim=64, inter=688,
                      vocab=1024, prefill_len=16, max_seq=32, theta=10000.0,
                      quant=QuantFormat.Int4, group_size=32)
LLAMA3_8B = LlamaConfig(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336,
                        vocab=128256, prefill_len=1024, max_seq=1280, theta=500000.0,
                        quant=QuantFormat.Int4, group_size=128)
LLAMA2_70B = LlamaConfig(layers=80, hidden=8192, heads=64, kv_heads=8, head_dim=128, inter=28672,
                         vocab=32000, prefill_len=2048, max_seq=2176, theta=10000.0,
                         quant=QuantFormat.Int8, group_size=128)


def _bind(lib):
    if getattr(lib, "_llama_bound", False):
        return
    P = C.c_void_p
    sig = {
        "slc_llama_create": (C.c_int, [P, C.POINTER(_Config), C.POINTER(P)]),
        "slc_llama_destroy": (None, [P]),
        "slc_llama_set_weight": (C.c_int, [P, C.c_int, C.c_uint32, P, C.c_uint64]),
        "slc_llama_set_quant_weight": (C.c_int, [P, C.c_int, C.c_uint32, P, C.c_uint64, P,
                                                 C.c_uint64]),
        "slc_llama_init_random": (C.c_int, [P, C.c_uint64, C.c_float]),
        "slc_llama_step": (C.c_int, [P, C.c_int, P, P, C.c_uint32, C.c_uint32, P, C.c_uint64]),
        "slc_llama_generate": (C.c_int, [P, P, C.c_uint32, P, P]),
        "slc_llama_kv_buffer": (C.c_int, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)]),
        "slc_llama_command_count": (C.c_int, [P, C.c_int, C.POINTER(C.c_uint64)]),
        "slc_llama_weight_bytes": (C.c_int, [P, C.POINTER(C.c_uint64)]),
        "slc_llama_weight_ref": (C.c_int, [P, C.c_int, C.c_uint32, P, P]),
        "slc_llama_last_step_ms": (C.c_int, [P, C.POINTER(C.c_float)]),
        "slc_llama_memo_steps": (C.c_int, [P, C.POINTER(C.c_uint64)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    lib._llama_bound = True


class Llama:
    """A llama-dense model on one backend-cuda device (one tensor-parallel rank)."""

    def __init__(self, device: CudaDevice, config: LlamaConfig):
        self.dev = device
        self.cfg = config
        self._lib = load_library()
        _bind(self._lib)
        self._m = C.c_void_p()
        c = config._c()
        self._check(self._lib.slc_llama_create(device.handle, C.byref(c), C.byref(self._m)))

    def _check(self, rc):
        if rc != 0:
            self.dev._check(rc)

    def close(self):
        if self._m:
            self._lib.slc_llama_destroy(self._m)
            self._m = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_weight(self, role: str, layer: int, full: np.ndarray):
        a = np.ascontiguousarray(full, np.float32).ravel()
        self._check(self._lib.slc_llama_set_weight(self._m, ROLES.index(role), layer,
                                                   C.c_void_p(a.ctypes.data), a.size))

    def set_quant_weight(self, role: str, layer: int, codes: np.ndarray, scales: np.ndarray):
        """The full (unsharded) weight of `role` as already quantized codes
        (uint8 rows of the payload) and f32 scales [N, groups] in the model's
        format and group size; stored as it is (no second quantization)."""
        c = np.ascontiguousarray(codes, np.uint8).ravel()
        sc = np.ascontiguousarray(scales, np.float32).ravel()
        self._check(self._lib.slc_llama_set_quant_weight(self._m, ROLES.index(role), layer,
                                                         C.c_void_p(c.ctypes.data), c.size,
                                                         C.c_void_p(sc.ctypes.data), sc.size))

    def init_random(self, seed: int, std: float = 0.02):
        self._check(self._lib.slc_llama_init_random(self._m, seed, std))

    def step(self, mode: int, ids, positions, seq_len: int, past_len: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32).ravel()
        pos = np.ascontiguousarray(positions, np.uint32).ravel()
        logits = np.empty(self.cfg.batch * self.cfg.vocab, np.float32)
        self._check(self._lib.slc_llama_step(self._m, mode, C.c_void_p(ids.ctypes.data),
                                             C.c_void_p(pos.ctypes.data), seq_len, past_len,
                                             C.c_void_p(logits.ctypes.data), logits.size))
        return logits.reshape(self.cfg.batch, self.cfg.vocab)

    def generate(self, prompt, steps: int):
        """Greedy generation; returns (ids [steps+1, batch], margins [steps+1, batch])."""
        prompt = np.ascontiguousarray(prompt, np.uint32).ravel()
        ids = np.empty((steps + 1) * self.cfg.batch, np.uint32)
        margins = np.empty((steps + 1) * self.cfg.batch, np.float32)
        self._check(self._lib.slc_llama_generate(self._m, C.c_void_p(prompt.ctypes.data), steps,
                                                 C.c_void_p(ids.ctypes.data),
                                                 C.c_void_p(margins.ctypes.data)))
        return ids.reshape(steps + 1, self.cfg.batch), margins.reshape(steps + 1, self.cfg.batch)

    def kv_buffer(self):
        b, n = C.c_uint32(), C.c_uint64()
        self._check(self._lib.slc_llama_kv_buffer(self._m, C.byref(b), C.byref(n)))
        return b.value, n.value

    def command_count(self, mode: int) -> int:
        n = C.c_uint64()
        self._check(self._lib.slc_llama_command_count(self._m, mode, C.byref(n)))
        return n.value

    def weight_bytes(self) -> int:
        n = C.c_uint64()
        self._check(self._lib.slc_llama_weight_bytes(self._m, C.byref(n)))
        return n.value

    def weight_ref(self, role: str, layer: int = 0):
        """(BufferRef, Value) of this rank's shard of a weight."""
        r, v = _BufferRef(), _Value()
        self._check(self._lib.slc_llama_weight_ref(self._m, ROLES.index(role), layer,
                                                   C.byref(r), C.byref(v)))
        val = Value(DType(v.dtype), tuple(int(v.dims[i]) for i in range(v.rank)),
                    ValueRole(v.role), Encoding(v.encoding), QuantFormat(v.quant_format),
                    int(v.group_size))
        return BufferRef(r.buffer, r.offset, r.len), val

    def last_step_ms(self) -> float:
        ms = C.c_float()
        self._check(self._lib.slc_llama_last_step_ms(self._m, C.byref(ms)))
        return float(ms.value)

    def memo_steps(self) -> int:
        """Steps that relaunched their program's captured graph directly."""
        n = C.c_uint64()
        self._check(self._lib.slc_llama_memo_steps(self._m, C.byref(n)))
        return int(n.value)
