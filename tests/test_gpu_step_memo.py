"""The engine's step memo (command capture on). Once a program's commands
have run as one captured graph, later steps of that program relaunch the
graph with their own seq_len / past_len instead of dispatching every
command again. The logits of memo steps must match a model that dispatches
every step (SLC_STEP_MEMO=0) on the same device, weights and ids. The memo
is dropped whenever the device's graphs are (here: capture switched off and
on again) and is rebuilt once the program has been captured again."""
import numpy as np
import pytest

from tests.gpu_util import assert_reduction

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, hidden=1024, heads=8, kv_heads=8, head_dim=128, inter=2048, vocab=1024,
           batch=1, prefill_len=20, max_seq=40, eps=1e-5, theta=500000.0, group_size=128)
STEPS = 10


def _run(dev, monkeypatch, memo, reset_at=None):
    from starlight_b200.device import QuantFormat
    from starlight_b200.engine import DECODE, PREFILL, Llama, LlamaConfig
    monkeypatch.setenv("SLC_STEP_MEMO", "1" if memo else "0")
    model = Llama(dev, LlamaConfig(**CFG, quant=QuantFormat.Int4))
    counts = []
    try:
        model.init_random(seed=7, std=0.02)
        T = CFG["prefill_len"]
        rng = np.random.default_rng(5)
        prompt = rng.integers(0, CFG["vocab"], size=T, dtype=np.uint32)
        out = [model.step(PREFILL, prompt, np.arange(T, dtype=np.uint32), T, 0)]
        ids = rng.integers(0, CFG["vocab"], size=STEPS, dtype=np.uint32)
        for s in range(STEPS):
            if s == reset_at:
                dev.set_capture(False)
                dev.set_capture(True)
            out.append(model.step(DECODE, ids[s:s + 1], np.array([T + s], np.uint32), 1, T + s))
            counts.append(model.memo_steps())
    finally:
        model.close()
    return out, counts


@pytest.fixture
def dev():
    from starlight_b200.device import CudaDevice
    d = CudaDevice(0)
    d.set_capture(True)
    yield d
    d.close()


def test_memo_steps_match_dispatched_steps(dev, monkeypatch):
    ref, ref_counts = _run(dev, monkeypatch, memo=False)
    got, counts = _run(dev, monkeypatch, memo=True)
    assert ref_counts == [0] * STEPS
    # Step 0 runs eagerly (first sight of the key), step 1 is captured and
    # fills the memo, steps 2.. relaunch the graph from it.
    assert counts == [0, 0] + list(range(1, STEPS - 1)), counts
    for a, b in zip(got, ref):
        assert_reduction(a.ravel(), b.ravel())
        assert int(np.argmax(a)) == int(np.argmax(b))


def test_memo_is_dropped_with_the_graphs_and_rebuilt(dev, monkeypatch):
    ref, _ = _run(dev, monkeypatch, memo=False)
    got, counts = _run(dev, monkeypatch, memo=True, reset_at=5)
    # Steps 2-4 from the memo; capture reset before step 5: step 5 eager,
    # step 6 captured again, steps 7-9 from the new memo.
    assert counts == [0, 0, 1, 2, 3, 3, 3, 4, 5, 6], counts
    for a, b in zip(got, ref):
        assert_reduction(a.ravel(), b.ravel())
