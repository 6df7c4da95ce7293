"""Generates tests/golden/fixture_greedy.json with the CPU oracle.

The fixture is BASELINE configs[0]: llama-dense, 2 layers, hidden 256,
4 heads x 64 (MHA), FFN 688 SiLU-gated, vocab 1024, RMSNorm eps 1e-5, RoPE
theta 10000, weights N(0, 0.02) (norm weights N(1, 0.1)) drawn from the
reference LCG (crates/backends/backend-cpu/src/reference/mod.rs:118-148) with
a Box-Muller transform, symmetric INT4 group 32; batch 1; a 16-token prompt of
ids uniform in [0, 1024); 16 greedy decode steps.

Run from the repository root:  python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import pyoracle as orc  # noqa: E402

WEIGHT_SEED = 20260001
PROMPT_SEED = 20260002


def fixture_config(quant=orc.INT4, group=32, batch=1):
    return orc.LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=4, head_dim=64, inter=688,
                           vocab=1024, max_seq=32, batch=batch, eps=1e-5, theta=10000.0,
                           quant_format=quant, group_size=group)


def fixture_prompt(batch=1):
    lcg = orc.Lcg(PROMPT_SEED)
    return np.array([lcg.below(1024) for _ in range(16 * batch)], np.uint32)


def main():
    model = orc.Llama(fixture_config())
    model.init_random(WEIGHT_SEED, 0.02)
    prompt = fixture_prompt()
    ids, logits = model.generate(prompt, 16)
    margins = []
    for lg in logits:
        top = np.sort(lg)[-2:]
        margins.append(float(top[1] - top[0]))
    out = {
        "config": "BASELINE configs[0] llama-dense fixture, INT4 g32, batch 1",
        "weight_seed": WEIGHT_SEED,
        "prompt_seed": PROMPT_SEED,
        "prompt": [int(v) for v in prompt],
        "greedy_ids": [int(v) for v in ids],
        "top2_margins": margins,
        "prefill_logits_head": [float(v) for v in logits[0][:8]],
        "logits_sha256": [hashlib.sha256(lg.tobytes()).hexdigest() for lg in logits],
    }
    with open(os.path.join(HERE, "fixture_greedy.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps({k: out[k] for k in ("prompt", "greedy_ids")}))
    print("min margin", min(margins))


if __name__ == "__main__":
    main()
