"""The product-side input generator is bit-identical to the oracle's."""
import numpy as np

import oracle as O
from firewing_b200 import synth


def test_input_generator_matches_oracle():
    for seed, rows, hidden in ((0, 3, 2048), (17, 5, 256), (1001, 2, 3072)):
        assert np.array_equal(synth.synth_input(seed, rows, hidden), O.synth_input(seed, rows, hidden))


def test_weight_stream_matches_oracle():
    key = synth.stream_key(5, O.T_DOWN)
    assert int(key) == O.lib().fwo_splitmix64_key(5, O.T_DOWN)
    ih = synth.irwin_hall(key, 12345, 64)
    w = synth.f32_to_bf16(ih.astype(np.float32) * synth.scale_for(0.02))
    assert np.array_equal(w, O.synth_bf16(5, O.T_DOWN, 12345, 64, 0.02))


def test_zipf_bias_matches_oracle():
    assert np.array_equal(synth.zipf_bias(512), O.zipf_bias(512))
