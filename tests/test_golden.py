"""The committed golden fixture (tests/golden/fixture_greedy.json) is
reproduced bit for bit by the CPU oracle: same greedy ids, same logits bytes."""
import hashlib
import json
import os

import numpy as np

from oracle import pyoracle as orc
from tests.golden.make_golden import WEIGHT_SEED, fixture_config, fixture_prompt

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fixture_greedy.json")


def test_oracle_reproduces_golden_fixture():
    g = json.load(open(GOLDEN))
    model = orc.Llama(fixture_config())
    model.init_random(WEIGHT_SEED, 0.02)
    prompt = fixture_prompt()
    assert [int(v) for v in prompt] == g["prompt"]
    ids, logits = model.generate(prompt, 16)
    assert ids == g["greedy_ids"]
    assert [hashlib.sha256(lg.tobytes()).hexdigest() for lg in logits] == g["logits_sha256"]


def test_oracle_result_independent_of_thread_count():
    a = orc.Llama(fixture_config())
    a.init_random(WEIGHT_SEED, 0.02)
    orc.set_threads(1)
    ids1, lg1 = a.generate(fixture_prompt(), 3)
    orc.set_threads(4)
    ids4, lg4 = a.generate(fixture_prompt(), 3)
    assert ids1 == ids4 and all(np.array_equal(x, y) for x, y in zip(lg1, lg4))
