"""The bench's algorithmic bytes (the roofline numerator), derived independently from the
pinned model's tensor shapes (the synthetic checkpoint's own specification)."""
from tests.conftest import load_synth

import bench


def _shapes():
    synth = load_synth()
    return dict(synth.tensor_specs(synth.PINNED)), synth.PINNED


def _numel(shape):
    n = 1
    for v in shape:
        n *= v
    return n


def test_layer_head_and_kv_bytes_match_the_tensor_shapes():
    specs, d = _shapes()
    layer = [name for name in specs if name.startswith("model.layers.0.") and name.endswith("proj.weight")]
    assert len(layer) == 7  # q, k, v, o, gate, up, down
    assert bench.LAYER_BYTES == sum(_numel(specs[n]) for n in layer) * 2
    norms = [n for n in specs if n.endswith("norm.weight")]
    assert bench.NORM_BYTES == sum(_numel(specs[n]) for n in norms) * 2
    # The semantic phase projects rows [151852, 151853 + 32768): 32,769 head rows.
    assert bench.HEAD_BYTES == 32769 * d.hidden * 2
    assert bench.EMBED_BYTES == d.hidden * 2
    # K and V of every layer at one position.
    assert bench.KV_BYTES_PER_POS == d.layers * 2 * d.kv_heads * d.head_dim * 2


def test_step_bytes_at_the_config2_average_position():
    # Prompt 512, 400 decoded tokens: the average visible length is 712.
    L = bench.PROMPT + bench.DECODE // 2
    assert bench.step_bytes(L) == 28 * bench.LAYER_BYTES + bench.NORM_BYTES + bench.HEAD_BYTES + \
        bench.EMBED_BYTES + bench.KV_BYTES_PER_POS * (L + 1)
    assert bench.step_bytes(712) == 3_034_818_560


def test_kv_bytes_grow_by_one_position_per_step():
    assert bench.step_bytes(1001) - bench.step_bytes(1000) == bench.KV_BYTES_PER_POS
