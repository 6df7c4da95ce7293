"""Quantized weights through the Safetensors store on a B200: a file of F32
weights quantized by the device (`quantize_file`) holds exactly the codes
and scales of the quantization format's CPU definition (oracle), and a model
bound to the stored codes (`Llama.set_quant_weight`, no second
quantization) gives the same logits, bit for bit, as the model quantizing
the same F32 weights on upload (`Llama.set_weight`)."""
import numpy as np
import pytest

from oracle import pyoracle as orc
from starlight_b200.device import CudaDevice, QuantFormat
from starlight_b200.engine import DECODE, PREFILL, ROLES, Llama
from starlight_b200.quant_store import load, quantize_file
from tests.golden.make_golden import WEIGHT_SEED, fixture_config, fixture_prompt
from tests.test_gpu_engine import engine_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("quant,group", [(orc.INT4, 32), (orc.INT8, 64)])
def test_quantized_file_and_binding(tmp_path, quant, group):
    from safetensors.numpy import save_file
    qf = QuantFormat.Int4 if quant == orc.INT4 else QuantFormat.Int8
    ref = orc.Llama(fixture_config(quant=quant, group=group, batch=1))
    ref.init_random(WEIGHT_SEED, 0.02)
    cfg = engine_config(quant, group)
    # The matrices of the quantized roles (the embedding and norms stay F32).
    mats = {}
    for role in ("q", "k", "v", "o", "gate", "up", "down", "lm_head"):
        for layer in (range(cfg.layers) if role in orc.LAYER_ROLES else [0]):
            n, k = _shape(cfg, role)
            mats[f"{role}.{layer}"] = np.asarray(ref.weight_source(role, layer),
                                                 np.float32).reshape(n, k)
    src, dst = str(tmp_path / "f32.safetensors"), str(tmp_path / "q.safetensors")
    save_file(mats, src)
    dev = CudaDevice(0)
    try:
        quantize_file(dev, src, dst, qf, group)
        stored, plain = load(dst)
        assert not plain and set(stored) == set(mats)
        for name, q in stored.items():
            n, k = mats[name].shape
            codes, scales = orc.quantize(quant, mats[name].ravel(), n, k, group)
            rb = q.codes.shape[1]
            assert np.array_equal(q.codes.ravel(), np.asarray(codes).view(np.uint8)[: n * rb]), name
            assert np.array_equal(q.scales.ravel(), np.asarray(scales, np.float32)), name
        logits = []
        for bind_stored in (False, True):
            model = Llama(dev, cfg)
            for role in ROLES:
                for layer in (range(cfg.layers) if role in orc.LAYER_ROLES else [0]):
                    key = f"{role}.{layer}"
                    if bind_stored and key in stored:
                        model.set_quant_weight(role, layer, stored[key].codes, stored[key].scales)
                    else:
                        model.set_weight(role, layer, ref.weight_source(role, layer))
            prompt = fixture_prompt(1)
            T = cfg.prefill_len
            out = [model.step(PREFILL, prompt, np.arange(T, dtype=np.uint32), T, 0)]
            for s in range(3):
                nxt = int(np.argmax(out[-1]))
                out.append(model.step(DECODE, [nxt], [T + s], 1, T + s))
            logits.append(np.stack(out))
            model.close()
        assert np.array_equal(logits[0], logits[1])
    finally:
        dev.close()


def _shape(cfg, role):
    H, D = cfg.hidden, cfg.head_dim
    return {"q": (cfg.heads * D, H), "k": (cfg.kv_heads * D, H), "v": (cfg.kv_heads * D, H),
            "o": (H, cfg.heads * D), "gate": (cfg.inter, H), "up": (cfg.inter, H),
            "down": (H, cfg.inter), "lm_head": (cfg.vocab, H)}[role]
