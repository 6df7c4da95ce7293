"""Parity of the path bench.py times: the Llama-3-8B-shaped llama-dense model
(hidden 4096, 32/8 heads of 128, FFN 14336, the full 128256-entry vocabulary,
INT4 group 128, theta 5e5) with command capture on, so that decode steps run
as CUDA-graph replays through the capture-time fusions (grouped q/k/v and
gate/up GEMVs, the fused decode attention block, residual Add + RmsNorm) and
the production decode GEMVs. Two layers keep the CPU oracle within seconds.

Every step's logits (prefill, then greedy decode) must match the oracle
(restated backend-cpu kernels on the dequantized weights) within the
reduction/matmul tolerance, and every greedy id must match bit for bit. The
top-1 minus top-2 margin of the oracle's logits is recorded with each id so a
failure can be told apart from a near tie."""
import numpy as np
import pytest

from oracle import pyoracle as orc
from starlight_b200.device import CudaDevice, QuantFormat
from starlight_b200.engine import DECODE, PREFILL, ROLES, Llama, LlamaConfig
from tests.gpu_util import assert_reduction

pytestmark = pytest.mark.gpu

LAYERS, VOCAB = 2, 128256


def _configs(batch, prefill, steps):
    ocfg = orc.LlamaConfig(layers=LAYERS, hidden=4096, heads=32, kv_heads=8, head_dim=128,
                           inter=14336, vocab=VOCAB, max_seq=prefill + steps + 1, batch=batch,
                           eps=1e-5, theta=500000.0, quant_format=orc.INT4, group_size=128)
    cfg = LlamaConfig(layers=LAYERS, hidden=4096, heads=32, kv_heads=8, head_dim=128,
                      inter=14336, vocab=VOCAB, batch=batch, prefill_len=prefill,
                      max_seq=prefill + steps + 1, theta=500000.0, quant=QuantFormat.Int4,
                      group_size=128)
    return ocfg, cfg


def _margin(row):
    top = np.partition(np.asarray(row, np.float64), -2)[-2:]
    return float(top[1] - top[0])


@pytest.mark.parametrize("batch,prefill,steps", [(1, 64, 16), (8, 16, 8)])
def test_benchmark_shape_with_capture_matches_oracle(batch, prefill, steps):
    ocfg, cfg = _configs(batch, prefill, steps)
    ref = orc.Llama(ocfg)
    ref.init_random(2024, 0.02)
    dev = CudaDevice(0)
    model = None
    try:
        dev.set_capture(True)
        model = Llama(dev, cfg)
        for role in ROLES:
            for layer in (range(LAYERS) if role in orc.LAYER_ROLES else [0]):
                model.set_weight(role, layer, ref.weight_source(role, layer))
        prompt = orc.Lcg(2025).fill(batch * prefill, 0, VOCAB - 1).astype(np.uint32)
        pos = np.tile(np.arange(prefill, dtype=np.uint32), batch)
        ref.reset()
        got = model.step(PREFILL, prompt, pos, prefill, 0)
        want = ref.step(prompt, pos, prefill, 0).reshape(batch, VOCAB)
        records = []
        for s in range(steps + 1):
            assert_reduction(got.ravel(), want.ravel())
            ids = np.array([int(np.argmax(r)) for r in got], np.uint32)
            want_ids = np.array([orc.argmax(r) for r in want], np.uint32)
            records.append([(int(i), _margin(r)) for i, r in zip(want_ids, want)])
            assert np.array_equal(ids, want_ids), (s, ids, want_ids, records[-1])
            if s == steps:
                break
            past = prefill + s
            got = model.step(DECODE, ids, np.full(batch, past, np.uint32), 1, past)
            want = ref.step(want_ids, np.full(batch, past, np.uint32), 1, past).reshape(batch, VOCAB)
        stats = dev.capture_stats()
        # Decode steps 3.. replay one captured graph each.
        assert stats["replays"] >= steps - 2, stats
    finally:
        if model is not None:  # the model refers to the device: close it first
            model.close()
        dev.close()
