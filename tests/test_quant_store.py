"""The quantized Safetensors store (starlight_b200/quant_store.py), on CPU:
payload, scales and plain tensors round-trip bit for bit with the
`starlight.quantization` metadata, and malformed files or tensors are
rejected with a message. (Quantizing with the device and binding the stored
weights to a model: tests/test_gpu_quant_store.py.)"""
import json

import numpy as np
import pytest

from starlight_b200.device import QuantFormat
from starlight_b200.quant_store import METADATA_KEY, QuantTensor, load, save


def _qt(rng, n, k, fmt, g):
    rb = (k + 1) // 2 if fmt == QuantFormat.Int4 else k
    return QuantTensor(rng.integers(0, 256, (n, rb), dtype=np.uint8),
                       rng.random((n, -(-k // g)), dtype=np.float32), fmt, g, (n, k))


def test_round_trip_is_bit_exact(tmp_path):
    rng = np.random.default_rng(3)
    q = {"layers.0.q": _qt(rng, 64, 256, QuantFormat.Int4, 128),
         "layers.0.down": _qt(rng, 32, 96, QuantFormat.Int8, 32),
         "odd": _qt(rng, 5, 33, QuantFormat.Int4, 7)}
    plain = {"layers.0.attn_norm": rng.random(256, dtype=np.float32)}
    path = str(tmp_path / "m.safetensors")
    save(path, q, plain)
    got, got_plain = load(path)
    assert set(got) == set(q) and set(got_plain) == set(plain)
    for name, t in q.items():
        g = got[name]
        assert g.fmt == t.fmt and g.group_size == t.group_size and g.shape == t.shape
        assert np.array_equal(g.codes, t.codes) and np.array_equal(g.scales, t.scales)
    assert np.array_equal(got_plain["layers.0.attn_norm"], plain["layers.0.attn_norm"])


def test_metadata_records_recovery_information(tmp_path):
    from safetensors import safe_open
    path = str(tmp_path / "m.safetensors")
    save(path, {"w": _qt(np.random.default_rng(1), 16, 256, QuantFormat.Int4, 128)})
    with safe_open(path, framework="numpy") as f:
        meta = json.loads(f.metadata()[METADATA_KEY])
        assert meta == {"version": 1, "tensors": {"w": {
            "format": "int4", "group_size": 128, "shape": [16, 256],
            "payload": "w.qweight", "scales": "w.scales"}}}
        assert f.get_tensor("w.qweight").dtype == np.uint8
        assert f.get_tensor("w.scales").shape == (16, 2)


def test_rejects_malformed_tensors_and_files(tmp_path):
    from safetensors.numpy import save_file
    rng = np.random.default_rng(2)
    bad = _qt(rng, 8, 64, QuantFormat.Int4, 32)
    bad.codes = bad.codes[:, :-1]
    with pytest.raises(ValueError, match="payload must be uint8"):
        save(str(tmp_path / "a.safetensors"), {"w": bad})
    bad = _qt(rng, 8, 64, QuantFormat.Int8, 32)
    bad.scales = bad.scales.astype(np.float64)
    with pytest.raises(ValueError, match="scales must be float32"):
        save(str(tmp_path / "b.safetensors"), {"w": bad})
    plain = str(tmp_path / "plain.safetensors")
    save_file({"w": np.zeros((2, 2), np.float32)}, plain)
    with pytest.raises(ValueError, match="not a quantized file"):
        load(plain)
    wrong = str(tmp_path / "wrong.safetensors")
    save_file({"w.qweight": np.zeros((2, 3), np.uint8), "w.scales": np.zeros((2, 1), np.float32)},
              wrong, metadata={METADATA_KEY: json.dumps({"version": 1, "tensors": {"w": {
                  "format": "int4", "group_size": 8, "shape": [2, 8],
                  "payload": "w.qweight", "scales": "w.scales"}}})})
    with pytest.raises(ValueError, match="payload must be uint8"):
        load(wrong)
