"""Quantized weights in a Safetensors file, and their binding to a model.

The reference's `sl-quantize` tool (`README.md` section 8.3) writes a
Safetensors file in which every quantized tensor becomes its payload and its
scales, stored as tensors, with the recovery information in the file's
`starlight.quantization` metadata entry; it is not a file ordinary loaders
can use as weights. Its exact schema belongs to the sl-precision crate, which
is an empty submodule in the reference checkout, so this module defines it
(the format is this project's, not pinned to a reference file):

- `<name>.qweight`: U8 [N, row_bytes], the payload rows of the quantization
  format (INT4: ceil(K / 2) bytes a row, two's-complement nibbles, even k in
  the low nibble; INT8: K bytes);
- `<name>.scales`: F32 [N, ceil(K / group)], one scale per group along K;
- tensors that are not quantized (norm weights, ...) are kept as they are;
- metadata `starlight.quantization`: JSON
  `{"version": 1, "tensors": {name: {"format": "int4"|"int8",
  "group_size": g, "shape": [N, K], "payload": "<name>.qweight",
  "scales": "<name>.scales"}}}`.

`quantize_file` makes such a file from an F32 Safetensors file with the
device's quantizer (`CudaDevice.quantize`, the sl-precision rounding), and
`load` / `QuantTensor` give the codes and scales that
`Llama.set_quant_weight` binds without quantizing again.
"""
from __future__ import annotations

import json
from dataclasses import dataclass

import numpy as np

from .device import BufferRef, CudaDevice, QuantFormat

METADATA_KEY = "starlight.quantization"
_FORMATS = {"int4": QuantFormat.Int4, "int8": QuantFormat.Int8}


def row_bytes(fmt: QuantFormat, k: int) -> int:
    return (k + 1) // 2 if fmt == QuantFormat.Int4 else k


@dataclass
class QuantTensor:
    """One quantized matrix of logical shape [N, K]."""
    codes: np.ndarray   # uint8 [N, row_bytes]
    scales: np.ndarray  # float32 [N, ceil(K / group)]
    fmt: QuantFormat
    group_size: int
    shape: tuple

    def check(self, name: str = "tensor"):
        n, k = self.shape
        groups = -(-k // self.group_size)
        if self.codes.dtype != np.uint8 or self.codes.shape != (n, row_bytes(self.fmt, k)):
            raise ValueError(f"{name}: payload must be uint8 [{n}, {row_bytes(self.fmt, k)}]")
        if self.scales.dtype != np.float32 or self.scales.shape != (n, groups):
            raise ValueError(f"{name}: scales must be float32 [{n}, {groups}]")


def save(path: str, quantized: dict, plain: dict | None = None):
    """Writes quantized tensors (name -> QuantTensor) and plain arrays."""
    from safetensors.numpy import save_file
    tensors, meta = {}, {}
    for name, q in quantized.items():
        q.check(name)
        tensors[name + ".qweight"] = np.ascontiguousarray(q.codes)
        tensors[name + ".scales"] = np.ascontiguousarray(q.scales)
        meta[name] = {"format": "int4" if q.fmt == QuantFormat.Int4 else "int8",
                      "group_size": int(q.group_size), "shape": [int(d) for d in q.shape],
                      "payload": name + ".qweight", "scales": name + ".scales"}
    for name, a in (plain or {}).items():
        if name in tensors:
            raise ValueError(f"{name}: name taken by a quantized tensor's part")
        tensors[name] = np.ascontiguousarray(a)
    save_file(tensors, path, metadata={METADATA_KEY: json.dumps({"version": 1, "tensors": meta})})


def load(path: str):
    """Returns (quantized: name -> QuantTensor, plain: name -> array)."""
    from safetensors import safe_open
    with safe_open(path, framework="numpy") as f:
        raw = (f.metadata() or {}).get(METADATA_KEY)
        if raw is None:
            raise ValueError(f"{path}: no {METADATA_KEY} metadata (not a quantized file)")
        meta = json.loads(raw)
        if meta.get("version") != 1:
            raise ValueError(f"{path}: unsupported {METADATA_KEY} version {meta.get('version')}")
        quantized, used = {}, set()
        for name, m in meta["tensors"].items():
            if m["format"] not in _FORMATS:
                raise ValueError(f"{name}: unknown quantization format {m['format']!r}")
            q = QuantTensor(f.get_tensor(m["payload"]), f.get_tensor(m["scales"]),
                            _FORMATS[m["format"]], int(m["group_size"]), tuple(m["shape"]))
            q.check(name)
            quantized[name] = q
            used.update((m["payload"], m["scales"]))
        plain = {k: f.get_tensor(k) for k in f.keys() if k not in used}
    return quantized, plain


def quantize_file(dev: CudaDevice, src: str, dst: str, fmt: QuantFormat, group_size: int,
                  select=None):
    """Quantizes the 2-D F32 tensors of `src` (those `select(name, array)`
    accepts; default: all) on the device and writes `dst`; the others are
    copied unchanged."""
    from safetensors.numpy import load_file
    tensors = load_file(src)
    quantized, plain = {}, {}
    for name, a in tensors.items():
        if a.ndim == 2 and a.dtype == np.float32 and (select is None or select(name, a)):
            quantized[name] = quantize_array(dev, a, fmt, group_size)
        else:
            plain[name] = a
    save(dst, quantized, plain)


def quantize_array(dev: CudaDevice, w: np.ndarray, fmt: QuantFormat, group_size: int) -> QuantTensor:
    """One F32 [N, K] matrix through the device's quantizer."""
    n, k = w.shape
    rb, groups = row_bytes(fmt, k), -(-k // group_size)
    words = -(-(n * rb) // 4)
    src = dev.allocate_f32(n * k)
    dev.upload_f32(src, np.ascontiguousarray(w, np.float32).ravel())
    codes, scales = dev.allocate_u32(words), dev.allocate_f32(n * groups)
    dev.quantize(BufferRef(src, 0, n * k), n, k, fmt, group_size, codes, scales)
    payload = dev.download_u32(codes).view(np.uint8)[: n * rb].reshape(n, rb).copy()
    sc = dev.download_f32(scales).reshape(n, groups).copy()
    for b in (src, codes, scales):
        dev.release(b)
    return QuantTensor(payload, sc, fmt, group_size, (n, k))
