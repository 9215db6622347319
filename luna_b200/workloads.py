"""Seeded synthetic networks and input boxes.

Every workload is generated from numpy's PCG64 generator with a fixed seed so
the engine, the oracle and the reference see bit-identical fp32 weights and
boxes.  Weights are He-normal (N(0, 2/fan_in)); biases are N(0, 0.01^2).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .abi import (NODE_ADD, NODE_BATCHNORM, NODE_CONCAT, NODE_CONV, NODE_CONVTRANSPOSE, NODE_FLATTEN,
                  NODE_IDENTITY, NODE_RESHAPE, NODE_SLICE, NODE_SUB,
                  NODE_INPUT, NODE_LINEAR, NODE_RELU, NODE_SIGMOID, Graph, Node)


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


def conv_out(h: int, k: int, s: int, p: int) -> int:
    return (h + 2 * p - k) // s + 1


def cnn(input_shape, layers, seed: int, bias_std: float = 0.01) -> Graph:
    """Input (C, H, W) -> layers -> output, ReLU after every layer but the last.

    `layers` items are ("conv", C_out, k, stride, pad), ("convbn", C_out, k,
    stride, pad) -- a conv followed by BatchNorm --, ("convT", C_out, k,
    stride, pad) -- a transposed conv -- or ("linear", n_out); a
    Flatten node is inserted where a conv feeds a linear layer.  Weights are
    He-normal over the fan-in (C_in k k for a conv), biases N(0, bias_std^2);
    BatchNorm gamma ~ U[0.5, 1.5], beta ~ N(0, 0.1^2), running mean ~ N(0,
    0.1^2), running var ~ U[0.5, 2]; drawn layer by layer from one PCG64
    stream."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], tuple(input_shape))]
    shape = tuple(input_shape)
    for li, spec in enumerate(layers):
        last = li == len(layers) - 1
        if spec[0] in ("conv", "convbn"):
            _, co, k, s, p = spec
            ci, h, w = shape
            fan_in = ci * k * k
            wt = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
            b = (rng.standard_normal(co) * bias_std).astype(np.float32)
            shape = (co, conv_out(h, k, s, p), conv_out(w, k, s, p))
            nodes.append(Node(NODE_CONV, [len(nodes) - 1], shape, weight=wt, bias=b,
                              kernel=(k, k), stride=(s, s), padding=(p, p)))
            if spec[0] == "convbn":
                gamma = rng.uniform(0.5, 1.5, co).astype(np.float32)
                beta = (rng.standard_normal(co) * 0.1).astype(np.float32)
                mean = (rng.standard_normal(co) * 0.1).astype(np.float32)
                var = rng.uniform(0.5, 2.0, co).astype(np.float32)
                nodes.append(Node(NODE_BATCHNORM, [len(nodes) - 1], shape, weight=gamma, bias=beta,
                                  running_mean=mean, running_var=var, eps=1e-5))
        elif spec[0] == "convT":
            # Transposed conv, weight [C_in, C_out, k, k] (He-normal over C_in k k).
            _, co, k, s, p = spec
            ci, h, w = shape
            fan_in = ci * k * k
            wt = (rng.standard_normal((ci, co, k, k)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
            b = (rng.standard_normal(co) * bias_std).astype(np.float32)
            shape = (co, (h - 1) * s - 2 * p + k, (w - 1) * s - 2 * p + k)
            nodes.append(Node(NODE_CONVTRANSPOSE, [len(nodes) - 1], shape, weight=wt, bias=b,
                              kernel=(k, k), stride=(s, s), padding=(p, p)))
        elif spec[0] == "linear":
            n_out = spec[1]
            if shape[1] != 1 or shape[2] != 1:
                shape = (int(np.prod(shape)), 1, 1)
                nodes.append(Node(NODE_FLATTEN, [len(nodes) - 1], shape))
            fan_in = shape[0]
            wt = (rng.standard_normal((n_out, fan_in)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
            b = (rng.standard_normal(n_out) * bias_std).astype(np.float32)
            shape = (n_out, 1, 1)
            nodes.append(Node(NODE_LINEAR, [len(nodes) - 1], shape, weight=wt, bias=b))
        else:
            raise ValueError(spec)
        if not last:
            nodes.append(Node(NODE_RELU, [len(nodes) - 1], shape))
    return Graph(nodes, 0, len(nodes) - 1)


def image_boxes(rng, n_boxes: int, n_in: int, eps: float, n_out: int):
    """Centres U[0,1]^n_in, radius eps clipped to [0,1], margin spec with a
    uniformly drawn true class per box."""
    c = rng.uniform(0.0, 1.0, (n_boxes, n_in)).astype(np.float32)
    t = rng.integers(0, n_out, n_boxes)
    lo = np.clip(c - np.float32(eps), 0.0, 1.0).astype(np.float32)
    hi = np.clip(c + np.float32(eps), 0.0, 1.0).astype(np.float32)
    return Boxes(lo, hi, margin_spec(t, n_out))


def cnn_cifar(n_boxes: int = 256, seed: int = 2, eps: float = 2.0 / 255.0):
    """CIFAR-shaped CNN 3x32x32 -> conv3->32 k3s1p1 -> conv32->64 k4s2p1 ->
    conv64->64 k4s2p1 -> flatten 4096 -> 512 -> 10, He-normal weights from
    seed 2; centres U[0,1], eps 2/255 clipped; 9 margin rows."""
    g = cnn((3, 32, 32), [("conv", 32, 3, 1, 1), ("conv", 64, 4, 2, 1), ("conv", 64, 4, 2, 1),
                          ("linear", 512), ("linear", 10)], seed)
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    return g, image_boxes(rng, n_boxes, 3 * 32 * 32, eps, 10)


def small_cnn_case(seed: int, n_boxes: int = 4, eps: float = 0.02, big_first: bool = True):
    """Small CNN for parity tests.  With big_first the first conv output has
    more than 4096 features, so Luna's CPU path starts it in patches mode
    (CROWNAnalysis.cpp:257-272); the second conv start stays dense."""
    rng = np.random.Generator(np.random.PCG64(seed))
    hw = 24 if big_first else 10
    g = cnn((3, hw, hw), [("conv", 8, 3, 1, 1), ("conv", 16, 4, 2, 1), ("conv", 8, 3, 1, 1),
                          ("linear", 24), ("linear", 5)], seed + 7, bias_std=0.1)
    return g, image_boxes(rng, n_boxes, 3 * hw * hw, eps, 5)


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


def sigmoid_mlp_case(seed: int, n_boxes: int = 4, widths=(6, 14, 12, 4), acts=(NODE_SIGMOID, NODE_SIGMOID),
                     eps: float = 0.5):
    """Small MLP with Sigmoid (and ReLU) activations for parity tests:
    weights 1.5x He-normal and biases N(0, 0.3^2) so that pre-activations
    cover the convex, concave and crossing regions of the sigmoid."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], (widths[0], 1, 1))]
    for i in range(1, len(widths)):
        w = (rng.standard_normal((widths[i], widths[i - 1])) * np.sqrt(2.0 / widths[i - 1]) * 1.5).astype(np.float32)
        b = (rng.standard_normal(widths[i]) * 0.3).astype(np.float32)
        nodes.append(Node(NODE_LINEAR, [len(nodes) - 1], (widths[i], 1, 1), weight=w, bias=b))
        if i < len(widths) - 1:
            nodes.append(Node(acts[i - 1], [len(nodes) - 1], (widths[i], 1, 1)))
    g = Graph(nodes, 0, len(nodes) - 1)
    c = rng.uniform(-1, 1, (n_boxes, widths[0])).astype(np.float32)
    r = rng.uniform(0.2 * eps, eps, (n_boxes, widths[0])).astype(np.float32)
    t = rng.integers(0, widths[-1], n_boxes)
    return g, Boxes((c - r).astype(np.float32), (c + r).astype(np.float32), margin_spec(t, widths[-1]))


def random_cnn_case(seed: int, n_boxes: int = 4, eps: float = 0.05, bn: bool = False):
    """Small random CNN (kernel 2..5, stride 1..2, padding 0..2, 1-3 convs,
    1-2 linear layers; with bn every conv is followed by BatchNorm) and boxes
    for parity fuzzing."""
    rng = np.random.Generator(np.random.PCG64(seed))
    c, h = int(rng.integers(1, 4)), int(rng.integers(7, 13))
    layers = []
    hh = h
    for _ in range(int(rng.integers(1, 4))):
        k = int(rng.integers(2, 6))
        s = int(rng.integers(1, 3))
        p = int(rng.integers(0, min(3, k)))
        if conv_out(hh, k, s, p) < 2:
            break
        layers.append(("convbn" if bn else "conv", int(rng.integers(2, 7)), k, s, p))
        hh = conv_out(hh, k, s, p)
    if not layers:
        layers.append(("convbn" if bn else "conv", 3, 3, 1, 1))
    for _ in range(int(rng.integers(1, 3))):
        layers.append(("linear", int(rng.integers(4, 17))))
    layers.append(("linear", 3))
    g = cnn((c, h, h), layers, seed + 11, bias_std=0.1)
    return g, image_boxes(rng, n_boxes, c * h * h, eps, 3)


def cnn_wide_case(seed: int, n_boxes: int = 3, eps: float = 0.01, hw: int = 12):
    """Small CNN whose strided convs have 32 / 64 channels (the shapes the
    tensor-core conv path takes), for parity tests: 3 x hw x hw -> conv32 k3
    -> conv32 k4s2p1 -> conv64 k4s2p1 -> 16 -> 4."""
    rng = np.random.Generator(np.random.PCG64(seed))
    g = cnn((3, hw, hw), [("conv", 32, 3, 1, 1), ("conv", 32, 4, 2, 1), ("conv", 64, 4, 2, 1),
                          ("linear", 16), ("linear", 4)], seed + 5, bias_std=0.05)
    return g, image_boxes(rng, n_boxes, 3 * hw * hw, eps, 4)


def small_cnn_bn_case(seed: int, n_boxes: int = 3, eps: float = 0.02, big_first: bool = True):
    """Small CNN with BatchNorm after every conv; with big_first the first
    BatchNorm output has more than 4096 features (a patches start on Luna's
    CPU path)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    hw = 24 if big_first else 10
    g = cnn((3, hw, hw), [("convbn", 8, 3, 1, 1), ("convbn", 16, 4, 2, 1), ("convbn", 8, 3, 1, 1),
                          ("linear", 24), ("linear", 5)], seed + 7, bias_std=0.1)
    return g, image_boxes(rng, n_boxes, 3 * hw * hw, eps, 5)


def convt_cnn_case(seed: int, n_boxes: int = 3, eps: float = 0.02, hw: int = 10, conv_after: bool = False,
                   wide: bool = False, tc: bool = False):
    """Small CNN with a strided transposed conv (conv -> conv s2 -> convT s2
    [-> conv] -> linear head) for parity tests; with wide the transposed conv
    maps 16 to 8 channels (the register-blocked kernels' shapes), with tc 32
    to 32 channels (the tensor-core transposed-conv steps' shapes)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if tc:
        layers = [("conv", 8, 3, 1, 1), ("conv", 32, 4, 2, 1), ("convT", 32, 4, 2, 1)]
    elif wide:
        layers = [("conv", 8, 3, 1, 1), ("conv", 16, 4, 2, 1), ("convT", 8, 4, 2, 1)]
    else:
        layers = [("conv", 6, 3, 1, 1), ("conv", 8, 4, 2, 1), ("convT", 5, 4, 2, 1)]
    if conv_after:
        layers.append(("conv", 4, 3, 1, 1))
    g = cnn((3, hw, hw), layers + [("linear", 12), ("linear", 4)], seed + 9, bias_std=0.1)
    return g, image_boxes(rng, n_boxes, 3 * hw * hw, eps, 4)


def _lin(rng, nodes, src, n_in, n_out, bias_std=0.1):
    w = (rng.standard_normal((n_out, n_in)) * np.sqrt(2.0 / n_in)).astype(np.float32)
    b = (rng.standard_normal(n_out) * bias_std).astype(np.float32)
    nodes.append(Node(NODE_LINEAR, [src], (n_out, 1, 1), weight=w, bias=b))
    return len(nodes) - 1


def _conv(rng, nodes, src, shape, co, k, s, p, bias_std=0.1):
    ci, h, w = shape
    wt = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    b = (rng.standard_normal(co) * bias_std).astype(np.float32)
    out = (co, conv_out(h, k, s, p), conv_out(w, k, s, p))
    nodes.append(Node(NODE_CONV, [src], out, weight=wt, bias=b, kernel=(k, k), stride=(s, s), padding=(p, p)))
    return len(nodes) - 1, out


def _act(nodes, src, shape):
    nodes.append(Node(NODE_RELU, [src], shape))
    return len(nodes) - 1


def flat_boxes(rng, n_boxes: int, n_in: int, eps: float, n_out: int):
    """Centres U[-1, 1]^n_in, radius U[0.2 eps, eps] per feature, margin spec."""
    c = rng.uniform(-1.0, 1.0, (n_boxes, n_in)).astype(np.float32)
    r = rng.uniform(0.2 * eps, eps, (n_boxes, n_in)).astype(np.float32)
    t = rng.integers(0, n_out, n_boxes)
    return Boxes((c - r).astype(np.float32), (c + r).astype(np.float32), margin_spec(t, n_out))


def sub_mlp_case(seed: int, n_boxes: int = 6, where: str = "input", constant_second: int = 1, eps: float = 0.3):
    """MLP 6 -> 12 -> 10 -> 4 with a Sub of a constant (BoundedSubNode):
    on the input (an input normalisation), or on the first Linear's output
    (where="linear"); constant_second = 0 gives constant - x."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], (6, 1, 1))]
    src, n = 0, 6
    if where == "input":
        c = rng.normal(0.3, 0.4, 6).astype(np.float32)
        nodes.append(Node(NODE_SUB, [0], (6, 1, 1), constant=c, constant_second=constant_second))
        src = 1
    h = _lin(rng, nodes, src, n, 12)
    if where == "linear":
        c = rng.normal(0.1, 0.3, 12).astype(np.float32)
        nodes.append(Node(NODE_SUB, [h], (12, 1, 1), constant=c, constant_second=constant_second))
        h = len(nodes) - 1
    h = _act(nodes, h, (12, 1, 1))
    h = _act(nodes, _lin(rng, nodes, h, 12, 10), (10, 1, 1))
    _lin(rng, nodes, h, 10, 4)
    return Graph(nodes, 0, len(nodes) - 1), flat_boxes(rng, n_boxes, 6, eps, 4)


def slice_mlp_case(seed: int, n_boxes: int = 6, eps: float = 0.3, reverse: bool = False):
    """MLP with Slices of flat vectors (BoundedSliceNode): 6 -> Linear 16 ->
    Slice [2:14] -> ReLU -> Linear 10 -> ReLU -> Slice [1:9] (or, reversed,
    start 8, end 0, step -1: features 8 down to 0, as Luna's
    BoundedSliceNode::_fixup_params reads it) -> Linear 4."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], (6, 1, 1))]
    h = _lin(rng, nodes, 0, 6, 16)
    nodes.append(Node(NODE_SLICE, [h], (12, 1, 1), axis=1, start=2, end=14, step=1))
    h = _act(nodes, len(nodes) - 1, (12, 1, 1))
    h = _act(nodes, _lin(rng, nodes, h, 12, 10), (10, 1, 1))
    k = 9 if reverse else 8
    if reverse:
        nodes.append(Node(NODE_SLICE, [h], (k, 1, 1), axis=1, start=8, end=0, step=-1))
    else:
        nodes.append(Node(NODE_SLICE, [h], (k, 1, 1), axis=1, start=1, end=-1, step=1))
    _lin(rng, nodes, len(nodes) - 1, k, 4)
    return Graph(nodes, 0, len(nodes) - 1), flat_boxes(rng, n_boxes, 6, eps, 4)


def concat_mlp_case(seed: int, n_boxes: int = 6, eps: float = 0.3):
    """Two Linear branches of the input concatenated (BoundedConcatNode,
    axis 1): 6 -> [Linear 8, Linear 6] -> Concat 14 -> ReLU -> Linear 10 ->
    ReLU -> Linear 4."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], (6, 1, 1))]
    a = _lin(rng, nodes, 0, 6, 8)
    b = _lin(rng, nodes, 0, 6, 6)
    nodes.append(Node(NODE_CONCAT, [a, b], (14, 1, 1), axis=1))
    h = _act(nodes, len(nodes) - 1, (14, 1, 1))
    h = _act(nodes, _lin(rng, nodes, h, 14, 10), (10, 1, 1))
    _lin(rng, nodes, h, 10, 4)
    return Graph(nodes, 0, len(nodes) - 1), flat_boxes(rng, n_boxes, 6, eps, 4)


def concat_cnn_case(seed: int, n_boxes: int = 3, eps: float = 0.02, hw: int = 8):
    """Two conv branches of the input concatenated along the channels: 3 x hw x
    hw -> [conv 4 k3 p1, conv 3 k3 p1] -> Concat 7 -> ReLU -> conv 6 k4 s2 p1
    -> ReLU -> Reshape (flatten) -> Linear 12 -> ReLU -> Linear 4."""
    rng = np.random.Generator(np.random.PCG64(seed))
    shape = (3, hw, hw)
    nodes = [Node(NODE_INPUT, [], shape)]
    a, sa = _conv(rng, nodes, 0, shape, 4, 3, 1, 1)
    b, sb = _conv(rng, nodes, 0, shape, 3, 3, 1, 1)
    cat = (sa[0] + sb[0], sa[1], sa[2])
    nodes.append(Node(NODE_CONCAT, [a, b], cat, axis=1))
    h = _act(nodes, len(nodes) - 1, cat)
    c, sc = _conv(rng, nodes, h, cat, 6, 4, 2, 1)
    h = _act(nodes, c, sc)
    n = int(np.prod(sc))
    nodes.append(Node(NODE_RESHAPE, [h], (n, 1, 1)))
    h = _act(nodes, _lin(rng, nodes, len(nodes) - 1, n, 12), (12, 1, 1))
    _lin(rng, nodes, h, 12, 4)
    return Graph(nodes, 0, len(nodes) - 1), image_boxes(rng, n_boxes, 3 * hw * hw, eps, 4)


def sub_cnn_case(seed: int, n_boxes: int = 3, eps: float = 0.02, hw: int = 8, constant_second: int = 1):
    """Input normalisation on a CNN: 3 x hw x hw -> Sub (per-pixel constant)
    -> conv 5 k3 p1 -> ReLU -> conv 6 k4 s2 p1 -> ReLU -> Reshape -> Linear 10
    -> ReLU -> Linear 4 (starts small enough for dense A on Luna's path)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    shape = (3, hw, hw)
    nodes = [Node(NODE_INPUT, [], shape)]
    c = rng.normal(0.45, 0.1, 3 * hw * hw).astype(np.float32)
    nodes.append(Node(NODE_SUB, [0], shape, constant=c, constant_second=constant_second))
    a, sa = _conv(rng, nodes, 1, shape, 5, 3, 1, 1)
    h = _act(nodes, a, sa)
    b, sb = _conv(rng, nodes, h, sa, 6, 4, 2, 1)
    h = _act(nodes, b, sb)
    n = int(np.prod(sb))
    nodes.append(Node(NODE_RESHAPE, [h], (n, 1, 1)))
    h = _act(nodes, _lin(rng, nodes, len(nodes) - 1, n, 10), (10, 1, 1))
    _lin(rng, nodes, h, 10, 4)
    return Graph(nodes, 0, len(nodes) - 1), image_boxes(rng, n_boxes, 3 * hw * hw, eps, 4)


def cnn_convt_cifar(n_boxes: int = 256, seed: int = 5, eps: float = 8.0 / 255.0):
    """3x32x32 -> conv3->32 k3s1p1 -> conv32->64 k4s2p1 -> convT64->32 k4s2p1 ->
    flatten 32768 -> 512 -> 10: the transposed-conv variant of the CIFAR CNN."""
    g = cnn((3, 32, 32), [("conv", 32, 3, 1, 1), ("conv", 64, 4, 2, 1), ("convT", 32, 4, 2, 1),
                          ("linear", 512), ("linear", 10)], seed)
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    return g, image_boxes(rng, n_boxes, 3 * 32 * 32, eps, 10)


def resnet(input_shape, stem: int, blocks, head, seed: int, bias_std: float = 0.01,
           head_act: int = NODE_SIGMOID, bn_mean_std: float = 0.0) -> Graph:
    """Small ResNet: Input (C, H, W) -> conv stem k3 s1 p1 -> ReLU -> residual
    blocks -> Flatten -> Linear head.

    Each block (C_out, stride) is conv k3 (stride) p1 -> BatchNorm -> ReLU ->
    conv k3 s1 p1 -> BatchNorm -> Add(skip) -> ReLU; the skip is the block
    input when the shape is unchanged, else a 1x1 projection conv with the
    block's stride (node order as a torchvision BasicBlock exports: conv1,
    bn1, relu, conv2, bn2, projection, add, relu).  `head` lists the Linear
    widths; every head layer but the last is followed by `head_act` (ReLU or
    Sigmoid).  Weights He-normal over the fan-in, biases N(0, bias_std^2);
    BatchNorm gamma ~ U[0.5, 1.5], beta ~ N(0, 0.1^2), running mean ~
    N(0, bn_mean_std^2) (0 by default), running var ~ U[0.5, 2]; one PCG64
    stream, drawn node by node."""
    rng = np.random.Generator(np.random.PCG64(seed))
    nodes = [Node(NODE_INPUT, [], tuple(input_shape))]

    def conv(src, shape, co, k, s, p):
        ci, h, w = shape
        wt = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
        b = (rng.standard_normal(co) * bias_std).astype(np.float32)
        out = (co, conv_out(h, k, s, p), conv_out(w, k, s, p))
        nodes.append(Node(NODE_CONV, [src], out, weight=wt, bias=b, kernel=(k, k), stride=(s, s), padding=(p, p)))
        return len(nodes) - 1, out

    def bn(src, shape):
        co = shape[0]
        gamma = rng.uniform(0.5, 1.5, co).astype(np.float32)
        beta = (rng.standard_normal(co) * 0.1).astype(np.float32)
        mean = (rng.standard_normal(co) * bn_mean_std).astype(np.float32)
        var = rng.uniform(0.5, 2.0, co).astype(np.float32)
        nodes.append(Node(NODE_BATCHNORM, [src], shape, weight=gamma, bias=beta, running_mean=mean,
                          running_var=var, eps=1e-5))
        return len(nodes) - 1

    def act(src, shape, kind=NODE_RELU):
        nodes.append(Node(kind, [src], shape))
        return len(nodes) - 1

    cur, shape = conv(0, tuple(input_shape), stem, 3, 1, 1)
    cur = act(cur, shape)
    for co, s in blocks:
        x, xshape = cur, shape
        h, shape = conv(x, xshape, co, 3, s, 1)
        h = act(bn(h, shape), shape)
        h, shape = conv(h, shape, co, 3, 1, 1)
        h = bn(h, shape)
        skip = x
        if s != 1 or co != xshape[0]:
            skip, _ = conv(x, xshape, co, 1, s, 0)
        nodes.append(Node(NODE_ADD, [h, skip], shape))
        cur = act(len(nodes) - 1, shape)
    shape = (int(np.prod(shape)), 1, 1)
    nodes.append(Node(NODE_FLATTEN, [cur], shape))
    cur = len(nodes) - 1
    for li, n_out in enumerate(head):
        fan_in = shape[0]
        wt = (rng.standard_normal((n_out, fan_in)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
        b = (rng.standard_normal(n_out) * bias_std).astype(np.float32)
        shape = (n_out, 1, 1)
        nodes.append(Node(NODE_LINEAR, [cur], shape, weight=wt, bias=b))
        cur = len(nodes) - 1
        if li != len(head) - 1:
            cur = act(cur, shape, head_act)
    return Graph(nodes, 0, len(nodes) - 1)


def resnet_cifar(n_boxes: int = 128, seed: int = 3, eps: float = 1.0 / 255.0):
    """Small CIFAR ResNet: stem conv3->16 k3, blocks (16, s1), (16, s1), (32, s2
    with a 1x1 projection skip), (32, s1), BatchNorm with running mean 0,
    flatten 8192 -> 100 -> Sigmoid -> 10; seed 3; centres U[0,1], eps 1/255
    clipped; 9 margin rows."""
    g = resnet((3, 32, 32), 16, [(16, 1), (16, 1), (32, 2), (32, 1)], [100, 10], seed)
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    return g, image_boxes(rng, n_boxes, 3 * 32 * 32, eps, 10)


def small_resnet_case(seed: int, n_boxes: int = 3, eps: float = 0.01, hw: int = 8, head_act: int = NODE_RELU,
                      big: bool = False):
    """Small ResNet for parity tests: stem 4 channels, an identity block and a
    strided block with a projection skip, head 12 -> 4.  With big the maps are
    20 x 20 with 12 channels, so the block convs have more than 4096 output
    features (patches starts on Luna's CPU path)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    c = 12 if big else 4
    hw = 20 if big else hw
    g = resnet((3, hw, hw), c, [(c, 1), (2 * c, 2)], [12, 4], seed + 13, bias_std=0.05, head_act=head_act,
               bn_mean_std=0.1)
    return g, image_boxes(rng, n_boxes, 3 * hw * hw, eps, 4)


def graph_forward(graph, x):
    """Plain forward of a graph on a batch of flat CHW inputs (torch, CPU);
    used to rank input pixels when splitting a box, not on the bounding path."""
    import torch
    import torch.nn.functional as F
    f = lambda a: torch.from_numpy(np.asarray(a, np.float32))
    deg = [len(n.inputs) for n in graph.nodes]
    users = [[] for _ in graph.nodes]
    for i, n in enumerate(graph.nodes):
        for p in n.inputs:
            users[p].append(i)
    order, q = [], [i for i, d in enumerate(deg) if d == 0]
    while q:
        c = q.pop(0)
        order.append(c)
        for u in users[c]:
            deg[u] -= 1
            if deg[u] == 0:
                q.append(u)
    val = {}
    for i in order:
        n = graph.nodes[i]
        ins = [val[p] for p in n.inputs]
        if n.type == NODE_INPUT:
            y = x.reshape(x.shape[0], *n.out_shape)
        elif n.type == NODE_LINEAR:
            y = ins[0].reshape(x.shape[0], -1) @ (f(n.weight) * n.scale).T + (f(n.bias) if n.bias is not None else 0)
        elif n.type == NODE_CONV:
            y = F.conv2d(ins[0], f(n.weight), f(n.bias) if n.bias is not None else None, stride=n.stride,
                         padding=n.padding)
        elif n.type == NODE_CONVTRANSPOSE:
            y = F.conv_transpose2d(ins[0], f(n.weight), f(n.bias) if n.bias is not None else None,
                                   stride=n.stride, padding=n.padding)
        elif n.type == NODE_BATCHNORM:
            w = f(n.weight) / torch.sqrt(f(n.running_var) + n.eps)
            b = f(n.bias) - f(n.running_mean) * w
            y = ins[0] * w.view(1, -1, 1, 1) + b.view(1, -1, 1, 1)
        elif n.type == NODE_RELU:
            y = torch.relu(ins[0])
        elif n.type == NODE_SIGMOID:
            y = torch.sigmoid(ins[0])
        elif n.type == NODE_ADD:
            y = ins[0] + ins[1]
        elif n.type in (NODE_FLATTEN, NODE_IDENTITY):
            y = ins[0].reshape(x.shape[0], -1) if n.type == NODE_FLATTEN else ins[0]
        else:
            raise NotImplementedError(n.type)
        val[i] = y
    return val[graph.output_index].reshape(x.shape[0], -1)


@dataclass
class SubdomainSplit:
    """A box split into 2^(groups) sub-domains: sub-domain `sid` takes, for
    every group g, the lower half of the box on the group's pixels when bit g
    of sid is 0 and the upper half when it is 1 (all other pixels keep the
    whole box).  A group is bisected as a unit, so the sub-domains cover the
    points whose pixels in each group lie on one side of the midpoint."""
    lower: np.ndarray    # [n_in] the box
    upper: np.ndarray
    centre: np.ndarray   # [n_in] the point the pixels were ranked at
    C: np.ndarray        # [1, nspec, n_out]
    groups: np.ndarray   # [n_groups, group_size] input indices (CHW)

    @property
    def count(self) -> int:
        return 1 << len(self.groups)

    def boxes(self, first: int, n: int) -> Boxes:
        """Sub-domains first .. first + n - 1 as a batch of boxes."""
        ids = np.arange(first, first + n, dtype=np.int64)
        if n and (ids[0] < 0 or ids[-1] >= self.count):
            raise ValueError("sub-domain id out of range")
        lo = np.repeat(self.lower[None], n, 0)
        hi = np.repeat(self.upper[None], n, 0)
        mid = ((self.lower + self.upper) / np.float32(2)).astype(np.float32)
        for g, idx in enumerate(self.groups):
            bit = ((ids >> g) & 1).astype(bool)
            lo[np.ix_(bit, idx)] = mid[idx]
            hi[np.ix_(~bit, idx)] = mid[idx]
        return Boxes(lo, hi, self.C)


def subdomain_split(graph, seed: int, eps: float, n_groups: int = 16, group_size: int = 4,
                    n_in_shape=(3, 32, 32)) -> SubdomainSplit:
    """Split one seeded eps-box (centre U[0,1], clipped to [0, 1], 9 margin rows
    for a uniformly drawn true class) along its widest-gradient pixels: rank
    the input coordinates by |d margin / d x| * width at the centre (margin =
    the sum of the specification rows), take the top n_groups * group_size,
    and group them in rank order into n_groups groups of group_size; each
    bit of a sub-domain id bisects one group."""
    import torch
    rng = np.random.Generator(np.random.PCG64(seed))
    n_in = int(np.prod(n_in_shape))
    n_out = graph.nodes[graph.output_index].out_shape[0]
    c = rng.uniform(0.0, 1.0, n_in).astype(np.float32)
    t = int(rng.integers(0, n_out))
    lo = np.clip(c - np.float32(eps), 0.0, 1.0).astype(np.float32)
    hi = np.clip(c + np.float32(eps), 0.0, 1.0).astype(np.float32)
    C = margin_spec(np.array([t]), n_out)
    x = torch.from_numpy(c[None]).requires_grad_(True)
    y = graph_forward(graph, x)
    (y @ torch.from_numpy(C[0]).T).sum().backward()
    score = np.abs(x.grad.numpy()[0]) * (hi - lo)
    top = np.argsort(-score, kind="stable")[: n_groups * group_size]
    return SubdomainSplit(lo, hi, c, C, top.reshape(n_groups, group_size).astype(np.int64))


def convt_sweep(seed: int = 5, eps: float = 8.0 / 255.0):
    """The transposed-conv CIFAR CNN and its eps = 8/255 box split into
    65,536 sub-domains (16 groups of 4 widest-gradient pixels)."""
    g, _ = cnn_convt_cifar(1, seed=seed)
    return g, subdomain_split(g, seed + 2000, eps)


_SWEEP = {}


def convt_sweep_boxes(n_boxes: int, seed: int = 5):
    """The first n_boxes sub-domains of convt_sweep (cached split)."""
    if seed not in _SWEEP:
        _SWEEP[seed] = convt_sweep(seed)
    g, split = _SWEEP[seed]
    return g, split.boxes(0, n_boxes)


def robustness_property(lower, upper, label: int, n_out: int) -> str:
    """VNN-LIB text of a local robustness property: the box [lower, upper] and
    the counterexample "some output j != label scores at least as high as
    the label" (an OR over j of Y_label - Y_j <= 0)."""
    lines = [f"; robustness of output {label} on a box of {len(lower)} inputs"]
    lines += [f"(declare-const X_{k} Real)" for k in range(len(lower))]
    lines += [f"(declare-const Y_{k} Real)" for k in range(n_out)]
    for k, (a, b) in enumerate(zip(lower, upper)):
        lines.append(f"(assert (>= X_{k} {float(a):.9g}))")
        lines.append(f"(assert (<= X_{k} {float(b):.9g}))")
    branches = " ".join(f"(and (<= (- Y_{label} Y_{j}) 0))" for j in range(n_out) if j != label)
    lines.append(f"(assert (or {branches}))")
    return "\n".join(lines) + "\n"


_PROPERTY = {}


def mlp_property_split(seed: int = 21, eps: float = 0.00317, n_groups: int = 9, group_size: int = 8):
    """The MLP 784->256x4->10 (seed 1) and a robustness property around one
    seeded point: the box centre U[0,1]^784, eps clipped to [0, 1], the label
    the network's own prediction at the centre; the box is split into
    2^n_groups sub-domains along its widest-gradient pixels
    (subdomain_split).  Returns (graph, split, property text)."""
    key = (seed, eps, n_groups, group_size)
    if key not in _PROPERTY:
        import torch
        g = mlp([784, 256, 256, 256, 256, 10], 1)
        split = subdomain_split(g, seed, eps, n_groups, group_size, n_in_shape=(784,))
        y = graph_forward(g, torch.from_numpy(split.centre[None]))
        t = int(y.argmax())
        split.C = margin_spec(np.array([t]), 10)
        _PROPERTY[key] = (g, split, robustness_property(split.lower, split.upper, t, 10))
    return _PROPERTY[key]


def mlp_property_boxes(n_boxes: int = 512, seed: int = 21):
    """The first n_boxes sub-domains of mlp_property_split (C: the label's margins)."""
    g, split, _ = mlp_property_split(seed)
    return g, split.boxes(0, n_boxes)
