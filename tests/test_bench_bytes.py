"""The algorithmic byte counts behind the bench's roofline numbers, on CPU,
against independent closed forms of the model shapes:

- one 8B-shaped INT4 g128 layer streams 218,103,808 weights as 4-bit codes
  (109,051,904 bytes) plus one f32 scale per 128 weights (6,815,744 bytes),
  reads 2 x past x 8 KV heads x 128 f32 of cache, writes one position, and
  reads two norm weight vectors;
- the vocabulary projection is 128256 x 4096 codes plus its scales, and the
  final norm weight;
- under tensor parallelism every rank's weight bytes are 1/N of the whole
  (the shards hold whole groups), and its KV bytes those of its heads;
- the 70B-shaped INT8 model the same way, with one byte a weight."""
import bench
from starlight_b200.engine import LLAMA2_70B, LLAMA3_8B, LlamaConfig


def _with(cfg, **kw):
    return LlamaConfig(**{**cfg.__dict__, **kw})


def test_8b_layer_bytes_closed_form():
    params = 4096 * (4096 + 1024 + 1024 + 4096) + 3 * 4096 * 14336
    assert params == 218_103_808
    weights = params // 2 + params // 128 * 4
    assert weights == 115_867_648
    for past in (0, 1, 1024, 1152):
        kv = 2 * past * 8 * 128 * 4 + 2 * 8 * 128 * 4
        assert bench.fused_layer_bytes(LLAMA3_8B, past) == weights + kv + 2 * 4096 * 4


def test_8b_step_bytes_match_the_reported_launch():
    # The bench's 32-layer launch at the timed steps' mean past (1044 after
    # 4 warm-up steps from a 1024-token prompt, 32 timed steps) is 3.98 GB.
    pasts = range(1028, 1060)
    per_launch = sum(32 * bench.fused_layer_bytes(LLAMA3_8B, p) for p in pasts) / len(pasts)
    assert abs(per_launch - 3_982_622_720) < 1


def test_lm_head_and_streamed_bytes():
    lm = 128256 * 4096 // 2 + 128256 * 32 * 4 + 4096 * 4
    assert bench.model_lm_bytes(LLAMA3_8B) == lm
    assert bench.streamed_weight_bytes(LLAMA3_8B) == 32 * 115_867_648 + lm


def test_tp_shards_divide_the_weights():
    full = bench.fused_layer_bytes(LLAMA3_8B, 0) - 2 * 8 * 128 * 4 - 2 * 4096 * 4
    for world in (2, 4, 8):
        cfg = _with(LLAMA3_8B, tp_world=world)
        rank = bench.fused_layer_bytes(cfg, 0) - 2 * (8 // world) * 128 * 4 - 2 * 4096 * 4
        assert rank * world == full
        # KV bytes of a rank: its kv heads only.
        d = bench.fused_layer_bytes(cfg, 100) - bench.fused_layer_bytes(cfg, 0)
        assert d == 2 * 100 * (8 // world) * 128 * 4


def test_70b_int8_layer_bytes():
    params = 8192 * (8192 + 1024 + 1024 + 8192) + 3 * 8192 * 28672
    weights = params + params // 128 * 4
    assert bench.fused_layer_bytes(LLAMA2_70B, 0) == weights + 2 * 8 * 128 * 4 + 2 * 8192 * 4
    lm = 32000 * 8192 + 32000 * 64 * 4 + 8192 * 4
    assert bench.model_lm_bytes(LLAMA2_70B) == lm
