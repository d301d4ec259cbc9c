"""Seeded synthetic MoE-layer workloads with GPT-OSS shapes.

No checkpoint or dataset is involved: every tensor is drawn from a seeded
numpy PCG64 stream with the distributions below, in the GGUF storage layout
that the reference reads (internal/model/gptoss/weights.go:52-116):

  norm gain        ones                         [H]
  router weight    N(0, 0.02)  f32              [E x H]  (ffn_gate_inp.weight)
  router bias      N(0, 0.01)  f32              [E]
  gate_up          MXFP4, E x 2I rows x H/32 blocks x 17 B (ffn_gate_up_exps.weight)
  gate_up bias     N(0, 0.01)  f32              [E x 2I]
  down             MXFP4, E x H rows x I/32 blocks x 17 B  (ffn_down_exps.weight)
  down bias        N(0, 0.01)  f32              [E x H]
  MXFP4 nibbles are uniform over the 16 E2M1 codes and the E8M0 scale byte is
  uniform over 119..123 (2^-8 .. 2^-4).
  Token rows (the block's residual input) are N(0, 1) f32.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class MoEShape:
    hidden: int
    intermediate: int
    experts: int
    top_k: int
    eps: float = 1e-5

    @property
    def gate_up_bytes_per_expert(self) -> int:
        return 2 * self.intermediate * (self.hidden // 32) * 17

    @property
    def down_bytes_per_expert(self) -> int:
        return self.hidden * (self.intermediate // 32) * 17


GPTOSS_20B = MoEShape(hidden=2880, intermediate=2880, experts=32, top_k=4)
GPTOSS_120B = MoEShape(hidden=2880, intermediate=2880, experts=128, top_k=4)


def _streams(seed: int, n: int):
    return [np.random.Generator(np.random.PCG64(s)) for s in np.random.SeedSequence(seed).spawn(n)]


def _mxfp4_bytes(rng, rows: int, cols: int, scale_lo=119, scale_hi=123) -> np.ndarray:
    nblk = cols // 32
    data = np.frombuffer(rng.bytes(rows * nblk * 17), dtype=np.uint8).copy()
    blocks = data.reshape(rows * nblk, 17)
    blocks[:, 0] = rng.integers(scale_lo, scale_hi + 1, size=rows * nblk, dtype=np.uint8)
    return data


def make_layer(shape: MoEShape, seed) -> dict:
    """One MoE layer (weights only) drawn from `seed` (an int or a tuple of ints)."""
    H, I, E = shape.hidden, shape.intermediate, shape.experts
    r = _streams(seed, 6)
    return {
        "hidden": H, "intermediate": I, "experts": E, "top_k": shape.top_k, "eps": shape.eps,
        "norm_gain": np.ones(H, np.float32),
        "router_w": r[0].normal(0.0, 0.02, size=(E, H)).astype(np.float32),
        "router_b": r[1].normal(0.0, 0.01, size=E).astype(np.float32),
        "gate_up": _mxfp4_bytes(r[2], E * 2 * I, H),
        "gate_up_b": r[3].normal(0.0, 0.01, size=(E, 2 * I)).astype(np.float32),
        "down": _mxfp4_bytes(r[4], E * H, I),
        "down_b": r[5].normal(0.0, 0.01, size=(E, H)).astype(np.float32),
    }


def make_tokens(shape: MoEShape, T: int, seed: int) -> np.ndarray:
    """T residual rows ~ N(0, 1), drawn from a stream independent of the weights."""
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 0x70C3])))
    return rng.standard_normal(size=(T, shape.hidden), dtype=np.float32)


# Zipf(s=1.1) rank-order router-bias offset: expert of rank r (0-based, drawn as a
# seeded permutation) gets ZIPF_SCALE * log(1 / (r + 1)^1.1), centred.  With the
# N(0, 0.02) router this makes the busiest expert take ~3x the mean load at
# T=4096, top-4 of 32 (checked by tests/test_workloads.py).
ZIPF_S = 1.1
ZIPF_SCALE = 0.33


def zipf_bias_offset(experts: int, seed: int, scale: float = ZIPF_SCALE) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 0x21F])))
    rank = rng.permutation(experts)
    off = scale * (-ZIPF_S * np.log(rank + 1.0))
    return (off - off.mean()).astype(np.float32)


HOT_EXPERTS = 8
HOT_BIAS = 4.0


def config_layer(config: int) -> dict:
    """Layer of one of the five benchmark configurations (router bias adjusted)."""
    if config == 0:
        return make_layer(GPTOSS_20B, 0)
    if config == 1:
        layer = make_layer(GPTOSS_20B, 1)
        layer["router_b"] = (layer["router_b"] + zipf_bias_offset(GPTOSS_20B.experts, 1)).astype(np.float32)
        return layer
    if config == 2:
        return make_layer(GPTOSS_20B, 2)
    if config == 3:
        return make_layer(GPTOSS_120B, 3)
    if config == 4:
        layer = make_layer(GPTOSS_120B, 4)
        b = layer["router_b"].copy()
        b[:HOT_EXPERTS] += HOT_BIAS  # the hot experts 0..7 all live on expert-parallel rank 0
        layer["router_b"] = b.astype(np.float32)
        return layer
    raise ValueError(f"no workload configuration {config}")


STREAM_LAYERS = 24
STREAM_DECODE_TOKENS = 64


def stream_layer(index: int) -> dict:
    """Layer `index` of the 24-layer streamed stack: config-0 statistics, seed (2, index)."""
    return make_layer(GPTOSS_20B, (2, index))


CONFIG_TOKENS = {0: 1, 1: 4096, 2: 1, 3: 256, 4: 16384}
CONFIG_SHAPE = {0: GPTOSS_20B, 1: GPTOSS_20B, 2: GPTOSS_20B, 3: GPTOSS_120B, 4: GPTOSS_120B}


def config_tokens(config: int, T: int | None = None) -> np.ndarray:
    return make_tokens(CONFIG_SHAPE[config], CONFIG_TOKENS[config] if T is None else T, config)


def small_layer(hidden=64, intermediate=128, experts=8, top_k=4, seed=0, scale_lo=119, scale_hi=123) -> dict:
    """Tiny layer for fast exact checks.  The CUDA path needs hidden and
    intermediate to be multiples of 64 (the oracle only needs 32)."""
    shape = MoEShape(hidden, intermediate, experts, top_k)
    layer = make_layer(shape, seed)
    if (scale_lo, scale_hi) != (119, 123):
        r = np.random.Generator(np.random.PCG64(seed + 99))
        layer["gate_up"] = _mxfp4_bytes(r, experts * 2 * intermediate, hidden, scale_lo, scale_hi)
        layer["down"] = _mxfp4_bytes(r, experts * hidden, intermediate, scale_lo, scale_hi)
    return layer
