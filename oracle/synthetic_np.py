"""Seeded numpy inputs for oracle tests and golden vectors (test
infrastructure only). Shapes and distributions follow the BASELINE configs:
router and shared gate BF16 ~ N(0, 0.02), expert weights FP32 ~ N(0, 0.02)
quantised with the oracle's NVFP4 quantiser, tokens BF16 ~ N(0, 1). Each
(seed, layer, kind, expert, projection) has its own numpy stream, so any
subset of experts can be generated on its own."""

from __future__ import annotations

import numpy as np

from .nvfp4_oracle import BankHost, QuantizedMatrix, bf16_bits_from_f32, bf16_bits_to_f32, quantize_nvfp4


def _rng(seed: int, layer: int, kind: int, *rest: int) -> np.random.Generator:
    return np.random.default_rng([seed, layer, kind, *rest])


def router_bf16(experts: int, hidden: int, seed: int, layer: int = 0) -> np.ndarray:
    w = _rng(seed, layer, 1).standard_normal((experts, hidden), dtype=np.float32) * np.float32(0.02)
    return bf16_bits_from_f32(w)


def shared_gate_bf16(hidden: int, seed: int, layer: int = 0) -> np.ndarray:
    w = _rng(seed, layer, 2).standard_normal(hidden, dtype=np.float32) * np.float32(0.02)
    return bf16_bits_from_f32(w)


def expert_projection(expert: int, projection: int, hidden: int, intermediate: int, seed: int,
                      layer: int = 0) -> QuantizedMatrix:
    shape = (intermediate, hidden) if projection < 2 else (hidden, intermediate)
    w = _rng(seed, layer, 3, expert, projection).standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return quantize_nvfp4(w)


def tokens_bf16(tokens: int, hidden: int, seed: int) -> np.ndarray:
    return bf16_bits_from_f32(_rng(seed, 0, 4).standard_normal((tokens, hidden), dtype=np.float32))


def skew_bias(experts: int, seed: int, layer: int = 0) -> np.ndarray:
    rank = (_rng(seed, layer, 5).permutation(experts) + 1).astype(np.float64)
    return (2.0 * np.log(1.0 / rank**1.2)).astype(np.float32)


def make_bank(experts: int, hidden: int, intermediate: int, seed: int, layer: int = 0,
              which: list[int] | None = None, skew: bool = False) -> BankHost:
    """BankHost with the listed experts (default: all routed + shared)."""
    bank = BankHost(experts, hidden, intermediate, router_bf16(experts, hidden, seed, layer),
                    shared_gate_bf16(hidden, seed, layer))
    if skew:
        bank.router_bias = skew_bias(experts, seed, layer)
    ids = range(experts + 1) if which is None else which
    for e in ids:
        for p in range(3):
            bank.projections[p][e] = expert_projection(e, p, hidden, intermediate, seed, layer)
    return bank


def tokens_f32(tokens: int, hidden: int, seed: int) -> np.ndarray:
    return bf16_bits_to_f32(tokens_bf16(tokens, hidden, seed))
