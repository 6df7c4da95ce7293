"""End-to-end parity of the llama-dense engine on backend-cuda against the CPU
oracle: BASELINE configs[0] (the llama-dense fixture), prefill + 16 greedy
decode steps. Greedy token ids must match bit for bit; logits of every step
within the reduction/matmul tolerance (tests/gpu_util.py)."""
import json
import os

import numpy as np
import pytest

from oracle import pyoracle as orc
from starlight_b200.device import CudaDevice, QuantFormat
from starlight_b200.engine import DECODE, PREFILL, ROLES, Llama, LlamaConfig
from tests.golden.make_golden import WEIGHT_SEED, fixture_config, fixture_prompt
from tests.gpu_util import assert_reduction

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fixture_greedy.json")


@pytest.fixture(scope="module")
def dev():
    d = CudaDevice(0)
    yield d
    d.close()


def engine_config(quant, group, batch=1, decompose=False):
    q = None if quant is None else (QuantFormat.Int4 if quant == orc.INT4 else QuantFormat.Int8)
    return LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=4, head_dim=64, inter=688,
                       vocab=1024, batch=batch, prefill_len=16, max_seq=32, eps=1e-5,
                       theta=10000.0, quant=q, group_size=group, decompose_swiglu=decompose)


def load_from_oracle(model: Llama, ref: orc.Llama, layers=2):
    for role in ROLES:
        for layer in (range(layers) if role in orc.LAYER_ROLES else [0]):
            model.set_weight(role, layer, ref.weight_source(role, layer))


def run_pair(dev, quant, group, batch=1, decompose=False, steps=16):
    ref = orc.Llama(fixture_config(quant=-1 if quant is None else quant, group=group, batch=batch))
    ref.init_random(WEIGHT_SEED, 0.02)
    model = Llama(dev, engine_config(quant, group, batch, decompose))
    load_from_oracle(model, ref)
    prompt = fixture_prompt(batch)
    ids, margins = model.generate(prompt, steps)
    # Oracle run (batch rows are independent sequences).
    ref.reset()
    t = 16
    pos = np.tile(np.arange(t, dtype=np.uint32), batch)
    want_logits = [ref.step(prompt, pos, t, 0).reshape(batch, -1)]
    want_ids = [want_logits[0].argmax(axis=1).astype(np.uint32)]
    for s in range(steps):
        nxt = want_ids[-1]
        lg = ref.step(nxt, np.full(batch, t + s, np.uint32), 1, t + s).reshape(batch, -1)
        want_logits.append(lg)
        want_ids.append(np.array([orc.argmax(r) for r in lg], np.uint32))
    return model, ids, margins, np.stack(want_ids), want_logits


def test_fixture_greedy_ids_match_oracle_and_golden(dev):
    model, ids, margins, want_ids, want_logits = run_pair(dev, orc.INT4, 32)
    g = json.load(open(GOLDEN))
    assert [int(v) for v in ids[:, 0]] == g["greedy_ids"]
    assert np.array_equal(ids, want_ids)
    # Logits of the prefill and of every decode step, re-run step by step.
    prompt = fixture_prompt()
    lg = model.step(PREFILL, prompt, np.arange(16), 16, 0)
    assert_reduction(lg.ravel(), want_logits[0].ravel())
    for s in range(16):
        lg = model.step(DECODE, [int(want_ids[s][0])], [16 + s], 1, 16 + s)
        assert_reduction(lg.ravel(), want_logits[s + 1].ravel())


@pytest.mark.parametrize("quant,group", [(None, 32), (orc.INT8, 32), (orc.INT4, 64),
                                         (orc.INT4, 128), (orc.INT8, 64)])
def test_fixture_variants_match_oracle(dev, quant, group):
    _, ids, _, want_ids, _ = run_pair(dev, quant, group, steps=8)
    assert np.array_equal(ids, want_ids)


def test_fixture_decomposed_swiglu_matches_oracle(dev):
    _, ids, _, want_ids, _ = run_pair(dev, orc.INT4, 32, decompose=True, steps=8)
    assert np.array_equal(ids, want_ids)


def test_fixture_batch_of_two(dev):
    _, ids, _, want_ids, _ = run_pair(dev, orc.INT4, 32, batch=2, steps=8)
    assert np.array_equal(ids, want_ids)


def test_engine_rejects_a_full_cache(dev):
    model = Llama(dev, engine_config(orc.INT4, 32))
    with pytest.raises(Exception):
        model.step(DECODE, [1], [40], 1, 40)


def test_llama8b_layer_shapes_match_oracle(dev):
    """One decoder layer with the Llama-3-8B shapes (GQA 32/8, head_dim 128,
    FFN 14336, theta 5e5, INT4 g128) and a 1024-entry vocabulary: exercises the
    tensor-core GEMV fast path, GQA split-K attention and the 4096-wide norms
    end to end against the oracle."""
    ocfg = orc.LlamaConfig(layers=1, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336,
                           vocab=1024, max_seq=16, batch=1, eps=1e-5, theta=500000.0,
                           quant_format=orc.INT4, group_size=128)
    ref = orc.Llama(ocfg)
    ref.init_random(77, 0.02)
    cfg = LlamaConfig(layers=1, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336,
                      vocab=1024, batch=1, prefill_len=8, max_seq=16, theta=500000.0,
                      quant=QuantFormat.Int4, group_size=128)
    model = Llama(dev, cfg)
    load_from_oracle(model, ref, layers=1)
    prompt = orc.Lcg(78).fill(8, 0, 1023).astype(np.uint32)
    ids, _ = model.generate(prompt, 3)
    ref.reset()
    want = [ref.step(prompt, np.arange(8, dtype=np.uint32), 8, 0)]
    got = [model.step(PREFILL, prompt, np.arange(8), 8, 0).ravel()]
    nxt = orc.argmax(want[0])
    for s in range(3):
        want.append(ref.step(np.array([nxt], np.uint32), np.array([8 + s], np.uint32), 1, 8 + s))
        got.append(model.step(DECODE, [nxt], [8 + s], 1, 8 + s).ravel())
        nxt = orc.argmax(want[-1])
    for g, w in zip(got, want):
        assert_reduction(g, w)
    assert [int(v) for v in ids[:, 0]] == [orc.argmax(w) for w in want]
