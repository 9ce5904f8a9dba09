"""Seeded synthetic MoE-layer inputs with the shapes and distributions of the benchmark.

There is no checkpoint on the machines this runs on, so every weight and
activation is drawn from a seeded generator: expert and shared weights
N(0, 0.02) rounded to bf16 (round to nearest even), the router gate N(0, 0.02)
kept in float32, activations N(0, 1) rounded to bf16.  Each tensor has its own
PCG64 stream keyed by (seed, layer, role, expert), so one expert can be rebuilt
without drawing the rest.

Layouts match the reference's safetensors tensors (src/DeepSeekRunner.cpp:157-177):
gate/up [experts, inter, hidden], down [experts, hidden, inter], the shared FFN
as one block of width inter * n_shared (src/DeepSeekRunner.cpp:217-222).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

ROLE_ROUTER, ROLE_GATE, ROLE_UP, ROLE_DOWN, ROLE_SHARED_GATE, ROLE_SHARED_UP, ROLE_SHARED_DOWN, \
    ROLE_TOKENS, ROLE_BIAS, ROLE_NORM = range(10)


@dataclass(frozen=True)
class MoeShape:
    """One MoE layer's sizes; defaults are DeepSeek-V2-Lite (include/Config.hpp:43-71)."""

    hidden: int = 2048
    inter: int = 1408
    n_routed_experts: int = 64
    n_shared_experts: int = 2
    top_k: int = 6

    @property
    def shared_width(self) -> int:
        return self.inter * self.n_shared_experts

    @property
    def expert_bytes(self) -> int:
        return 3 * self.inter * self.hidden * 2

    @property
    def shared_bytes(self) -> int:
        return 3 * self.shared_width * self.hidden * 2

    @property
    def router_bytes(self) -> int:
        return self.n_routed_experts * self.hidden * 4


V2_LITE = MoeShape()


def _rng(seed: int, *key: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, *key])))


def bf16_round(values: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (as the checkpoint writer does)."""
    bits = np.ascontiguousarray(values, np.float32).view(np.uint32)
    rounded = bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed: int, key: tuple, shape, std: float) -> np.ndarray:
    g = _rng(seed, *key)
    v = g.standard_normal(int(np.prod(shape)), dtype=np.float32)
    if std != 1.0:
        v *= np.float32(std)
    return bf16_round(v).reshape(shape)


def layer_weights(shape: MoeShape = V2_LITE, seed: int = 0, layer: int = 0, std: float = 0.02) -> dict:
    """All weights of one MoE layer as host arrays (bf16 as uint16 bits)."""
    E, I, H, S = shape.n_routed_experts, shape.inter, shape.hidden, shape.shared_width
    gate = np.empty((E, I, H), np.uint16)
    up = np.empty((E, I, H), np.uint16)
    down = np.empty((E, H, I), np.uint16)

    def fill(e: int) -> None:
        gate[e] = normal_bf16(seed, (layer, ROLE_GATE, e), (I, H), std)
        up[e] = normal_bf16(seed, (layer, ROLE_UP, e), (I, H), std)
        down[e] = normal_bf16(seed, (layer, ROLE_DOWN, e), (H, I), std)

    # numpy's generators release the GIL while filling, so threads scale.
    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as pool:
        list(pool.map(fill, range(E)))
    router = _rng(seed, layer, ROLE_ROUTER).standard_normal(E * H, dtype=np.float32).reshape(E, H)
    router *= np.float32(std)
    return {
        "router": np.ascontiguousarray(router),
        "gate": gate,
        "up": up,
        "down": down,
        "shared_gate": normal_bf16(seed, (layer, ROLE_SHARED_GATE), (S, H), std),
        "shared_up": normal_bf16(seed, (layer, ROLE_SHARED_UP), (S, H), std),
        "shared_down": normal_bf16(seed, (layer, ROLE_SHARED_DOWN), (H, S), std),
    }


def tokens(shape: MoeShape, T: int, seed: int, stream: int = 0) -> np.ndarray:
    """Activations [T, hidden] drawn N(0, 1) and rounded to bf16 (uint16 bits)."""
    return normal_bf16(seed, (stream, ROLE_TOKENS), (T, shape.hidden), 1.0)


def zipf_bias(shape: MoeShape, seed: int, s: float = 1.2) -> np.ndarray:
    """Per-expert logit bias b_e = ln(r_e ** -s) over a seeded permutation of ranks.

    Added to the router logits before the softmax, it skews expert load towards a
    Zipf(s) profile (the prefill configuration's load skew)."""
    ranks = _rng(seed, 0, ROLE_BIAS).permutation(shape.n_routed_experts) + 1
    return (-s * np.log(ranks.astype(np.float64))).astype(np.float32)
