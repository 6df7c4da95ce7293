"""The persistent decode-layer kernel (starlight_b200/csrc/kernels/
decode_layers.cu), reached the way the engine reaches it: command capture on,
batch 1, one token per step, every layer's sixteen commands fused into one
cooperative launch.

For several model shapes (GQA groups 1, 2, 4 and 8; INT4 and INT8; rows of
more and of fewer than 1 KiB of codes, and rows whose last 1 KiB chunk is
ragged; a short and a long context, so that the key
chunks per kv head vary) every decode step's logits must match the CPU oracle
(restated backend-cpu kernels on the dequantized weights) within the
reduction/matmul tolerance, every greedy id must match bit for bit, and the
KV cache the kernel appended must match the oracle's cache within the same
tolerance. The same steps with the fusion switched off (SLC_DECODE_FUSION=0)
must launch one kernel per command (or fused pair) again, and the fused steps
at most a handful."""
import os

import numpy as np
import pytest

from oracle import pyoracle as orc
from starlight_b200.device import CudaDevice, QuantFormat
from starlight_b200.engine import DECODE, PREFILL, ROLES, Llama, LlamaConfig
from tests.gpu_util import assert_reduction

pytestmark = pytest.mark.gpu

SHAPES = {
    # name: hidden, heads, kv_heads, inter, format, layers
    "g4_int4": (2048, 16, 4, 6144, orc.INT4, 3),
    "g8_int8": (2048, 16, 2, 4096, orc.INT8, 2),
    "g1_int4_short_rows": (1024, 8, 8, 2048, orc.INT4, 3),
    # down rows of 1536 code bytes: a 1 KiB chunk and a ragged 512-byte one
    "g2_int4_ragged_down": (2048, 16, 8, 3072, orc.INT4, 2),
}


def _configs(shape, prefill, steps, vocab=2048):
    H, Hq, Hkv, I, fmt, L = SHAPES[shape]
    max_seq = prefill + steps + 2
    ocfg = orc.LlamaConfig(layers=L, hidden=H, heads=Hq, kv_heads=Hkv, head_dim=128, inter=I,
                           vocab=vocab, max_seq=max_seq, batch=1, eps=1e-5, theta=500000.0,
                           quant_format=fmt, group_size=128)
    cfg = LlamaConfig(layers=L, hidden=H, heads=Hq, kv_heads=Hkv, head_dim=128, inter=I,
                      vocab=vocab, batch=1, prefill_len=prefill, max_seq=max_seq,
                      theta=500000.0,
                      quant=QuantFormat.Int4 if fmt == orc.INT4 else QuantFormat.Int8,
                      group_size=128)
    return ocfg, cfg


def _run(shape, prefill, steps, fused, ref):
    os.environ["SLC_DECODE_FUSION"] = "1" if fused else "0"
    ocfg, cfg = _configs(shape, prefill, steps)
    dev = CudaDevice(0)
    model = None
    try:
        dev.set_capture(True)
        model = Llama(dev, cfg)
        for role in ROLES:
            for layer in (range(cfg.layers) if role in orc.LAYER_ROLES else [0]):
                model.set_weight(role, layer, ref.weight_source(role, layer))
        prompt = orc.Lcg(prefill + 7).fill(prefill, 0, cfg.vocab - 1).astype(np.uint32)
        ref.reset()
        got = model.step(PREFILL, prompt, np.arange(prefill), prefill, 0).ravel()
        want = ref.step(prompt, np.arange(prefill, dtype=np.uint32), prefill, 0)
        logits, launches = [], []
        for s in range(steps + 1):
            assert_reduction(got, want)
            nxt = orc.argmax(want)
            assert int(np.argmax(got)) == nxt, (shape, s)
            logits.append(got)
            if s == steps:
                break
            past = prefill + s
            before = dev.launch_count()
            got = model.step(DECODE, [nxt], [past], 1, past).ravel()
            launches.append(dev.launch_count() - before)
            want = ref.step(np.array([nxt], np.uint32), np.array([past], np.uint32), 1, past)
        kb, kn = model.kv_buffer()
        cache = dev.download_f32(kb, kn)
        return logits, launches, cache, ocfg
    finally:
        if model is not None:  # the model refers to the device: close it first
            model.close()
        dev.close()
        os.environ.pop("SLC_DECODE_FUSION", None)


@pytest.mark.parametrize("shape,prefill", [("g4_int4", 37), ("g4_int4", 300), ("g8_int8", 90),
                                           ("g1_int4_short_rows", 20),
                                           ("g2_int4_ragged_down", 50)])
def test_fused_decode_layers_match_oracle(shape, prefill):
    steps = 6
    ocfg, _ = _configs(shape, prefill, steps)
    ref = orc.Llama(ocfg)
    ref.init_random(1000 + prefill, 0.02)
    logits, launches, cache, ocfg = _run(shape, prefill, steps, True, ref)
    # Replayed steps: gather, the fused layers, final norm, last token,
    # vocabulary projection.
    assert max(launches[2:]) <= 6, launches
    # The appended keys / values (prefill by the per-command kernels, decode
    # positions by the fused kernel) against the oracle's cache.
    want = ref.cache()
    L, Hkv, D, ms = ocfg.layers, ocfg.kv_heads, 128, ocfg.max_seq
    got5 = cache.reshape(1, L, 2, ms, Hkv, D)[:, :, :, :prefill + steps]
    want5 = want.reshape(1, L, 2, ms, Hkv, D)[:, :, :, :prefill + steps]
    assert_reduction(got5.ravel(), want5.ravel())


def test_fusion_off_restores_per_command_launches():
    shape, prefill, steps = "g4_int4", 37, 4
    ocfg, _ = _configs(shape, prefill, steps)
    ref = orc.Llama(ocfg)
    ref.init_random(77, 0.02)
    on, launches_on, _, _ = _run(shape, prefill, steps, True, ref)
    off, launches_off, _, _ = _run(shape, prefill, steps, False, ref)
    assert max(launches_on[2:]) <= 6
    assert min(launches_off[2:]) >= 8 * ocfg.layers
    for a, b in zip(on, off):
        assert_reduction(a, b)
