"""The synthetic workloads have the shapes and statistics the benchmark configurations name."""
import numpy as np

import oracle
from airllm_b200 import workloads as W


def test_layer_shapes_and_scale_range():
    layer = W.small_layer(hidden=64, intermediate=128, experts=4, top_k=2, seed=1)
    H, I, E = 64, 128, 4
    assert layer["gate_up"].size == E * 2 * I * (H // 32) * 17
    assert layer["down"].size == E * H * (I // 32) * 17
    scales = layer["gate_up"].reshape(-1, 17)[:, 0]
    assert scales.min() >= 119 and scales.max() <= 123


def test_seeded_generation_is_reproducible():
    a = W.make_layer(W.MoEShape(64, 64, 4, 2), 7)
    b = W.make_layer(W.MoEShape(64, 64, 4, 2), 7)
    for key in a:
        if isinstance(a[key], np.ndarray):
            assert np.array_equal(a[key], b[key])


def test_prefill_config_zipf_skew_is_about_three_times_mean():
    layer = W.config_layer(1)
    x = W.config_tokens(1)
    _, idx, _ = oracle.route(layer, x)
    counts = np.bincount(idx.ravel(), minlength=32)
    ratio = counts.max() / counts.mean()
    assert 2.7 <= ratio <= 3.3, ratio


def test_adversarial_config_hot_experts():
    b0 = W.make_layer(W.GPTOSS_120B, 4)["router_b"]
    b = W.config_layer(4)["router_b"]
    assert np.allclose(b[:8] - b0[:8], 4.0) and np.array_equal(b[8:], b0[8:])
