"""Seeded synthetic networks and input boxes.

Every workload is generated from numpy's PCG64 generator with a fixed seed so
the engine, the oracle and the reference see bit-identical fp32 weights and
boxes.  Weights are He-normal (N(0, 2/fan_in)); biases are N(0, 0.01^2).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .abi import NODE_INPUT, NODE_LINEAR, NODE_RELU, Graph, Node


def mlp(widths, seed: int, bias_std: float = 0.01) -> Graph:
    """Input -> (Linear -> ReLU) * (len(widths)-2) -> Linear, He-normal weights.

    Node ids follow the order a Luna ModelBuilder would assign
    (tests/fixtures/model_builders.cpp: input 0, then one id per layer)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], (widths[0], 1, 1))]
    for li in range(1, len(widths)):
        fan_in, fan_out = widths[li - 1], widths[li]
        w = (rng.standard_normal((fan_out, fan_in)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
        b = (rng.standard_normal(fan_out) * bias_std).astype(np.float32)
        nodes.append(Node(NODE_LINEAR, [len(nodes) - 1], (fan_out, 1, 1), weight=w, bias=b))
        if li != len(widths) - 1:
            nodes.append(Node(NODE_RELU, [len(nodes) - 1], (fan_out, 1, 1)))
    return Graph(nodes, 0, len(nodes) - 1)


@dataclass
class Boxes:
    """A batch of L-infinity input boxes plus one specification matrix per box."""
    lower: np.ndarray   # [B, n_in] fp32
    upper: np.ndarray   # [B, n_in] fp32
    C: np.ndarray       # [B or 1, nspec, n_out] fp32

    @property
    def n(self) -> int:
        return self.lower.shape[0]

    def slice(self, a: int, b: int) -> "Boxes":
        c = self.C if self.C.shape[0] == 1 else self.C[a:b]
        return Boxes(self.lower[a:b].copy(), self.upper[a:b].copy(), np.ascontiguousarray(c))


def margin_spec(true_class: np.ndarray, n_out: int) -> np.ndarray:
    """Rows y_t - y_j for every j != t, per box: [B, n_out-1, n_out]."""
    B = true_class.shape[0]
    C = np.zeros((B, n_out - 1, n_out), np.float32)
    for b in range(B):
        t = int(true_class[b])
        r = 0
        for j in range(n_out):
            if j == t:
                continue
            C[b, r, t] = 1.0
            C[b, r, j] = -1.0
            r += 1
    return C


def mlp_5_50x6_5(n_boxes: int = 1024, seed: int = 0):
    """MLP 5->50x6->5 (ReLU after each hidden layer), weights from seed 0;
    centres U[-1,1]^5, per-dim radius U[0.01,0.1]; spec rows y0 - yi, i=1..4."""
    g = mlp([5, 50, 50, 50, 50, 50, 50, 5], seed)
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    c = rng.uniform(-1.0, 1.0, (n_boxes, 5)).astype(np.float32)
    r = rng.uniform(0.01, 0.1, (n_boxes, 5)).astype(np.float32)
    C = np.zeros((1, 4, 5), np.float32)
    for i in range(1, 5):
        C[0, i - 1, 0] = 1.0
        C[0, i - 1, i] = -1.0
    return g, Boxes((c - r).astype(np.float32), (c + r).astype(np.float32), C)


def mlp_784_256x4_10(n_boxes: int = 512, seed: int = 1, eps: float = 0.02):
    """MLP 784->256x4->10, He-normal weights from seed 1; centres U[0,1]^784,
    eps 0.02 clipped to [0,1]; 9 margin rows y_t - y_j, t ~ U{0..9} per box."""
    g = mlp([784, 256, 256, 256, 256, 10], seed)
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    c = rng.uniform(0.0, 1.0, (n_boxes, 784)).astype(np.float32)
    t = rng.integers(0, 10, n_boxes)
    lo = np.clip(c - np.float32(eps), 0.0, 1.0).astype(np.float32)
    hi = np.clip(c + np.float32(eps), 0.0, 1.0).astype(np.float32)
    return g, Boxes(lo, hi, margin_spec(t, 10))


def random_mlp_case(seed: int, n_boxes: int = 8, depth: int = 3, width: int = 12,
                    n_in: int = 6, n_out: int = 4, eps: float = 0.3):
    """Small random MLP and boxes for parity fuzzing."""
    rng = np.random.Generator(np.random.PCG64(seed))
    widths = [n_in] + [int(rng.integers(max(2, width // 2), width + 1)) for _ in range(depth)] + [n_out]
    g = mlp(widths, seed + 7, bias_std=0.1)
    c = rng.uniform(-1.0, 1.0, (n_boxes, n_in)).astype(np.float32)
    r = rng.uniform(0.2 * eps, eps, (n_boxes, n_in)).astype(np.float32)
    t = rng.integers(0, n_out, n_boxes)
    return g, Boxes((c - r).astype(np.float32), (c + r).astype(np.float32), margin_spec(t, n_out))
