"""Generate the golden fixtures in tests/golden/ by running Luna itself.

Luna's own CPU implementation (compiled from the reference sources by
oracle/Makefile into oracle/_ref/libluna_ref.so) bounds every case below;
the inputs and Luna's outputs are stored as .npz files.  Network weights are
not stored: they are regenerated from the seeded generators in
luna_b200/workloads.py, and a checksum of them is stored to catch drift.

    make -C oracle && python tests/golden/make_golden.py [case names]
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from luna_b200 import abi, workloads as W  # noqa: E402
from oracle import luna_ref  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def weights_digest(graph) -> str:
    h = hashlib.sha256()
    for n in graph.nodes:
        for a in (n.weight, n.bias):
            if a is not None:
                h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def cases():
    """(name, generator, generator kwargs, box slice, method, option overrides)."""
    out = []
    out.append(("mlp5_ibp", "mlp_5_50x6_5", {"n_boxes": 32}, 32, abi.METHOD_IBP, {}))
    out.append(("mlp5_crown", "mlp_5_50x6_5", {"n_boxes": 32}, 32, abi.METHOD_CROWN, {}))
    out.append(("mlp5_alpha", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1}))
    out.append(("mlp784_crown", "mlp_784_256x4_10", {"n_boxes": 6}, 6, abi.METHOD_CROWN, {}))
    out.append(("mlp784_alpha", "mlp_784_256x4_10", {"n_boxes": 3}, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1}))
    for seed in range(6):
        kw = {"seed": 100 + seed, "n_boxes": 8, "depth": 2 + seed % 3, "width": 10 + 2 * seed}
        out.append((f"rand{seed}_crown", "random_mlp_case", kw, 8, abi.METHOD_CROWN, {}))
        out.append((f"rand{seed}_alpha", "random_mlp_case", kw, 8, abi.METHOD_ALPHA_CROWN,
                    {"alpha_lr": 0.5 if seed % 2 else 0.1, "alpha_iterations": 8 + seed}))
    # CNNs: all starts dense (conv outputs <= 4096 features) ...
    kw = {"seed": 3, "n_boxes": 4, "big_first": False}
    out.append(("cnn_dense_crown", "small_cnn_case", kw, 4, abi.METHOD_CROWN, {}))
    out.append(("cnn_dense_alpha", "small_cnn_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 8}))
    # ... and a first conv start in patches mode (4608 output features).
    kw = {"seed": 5, "n_boxes": 3, "big_first": True}
    out.append(("cnn_patch_crown", "small_cnn_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("cnn_patch_alpha", "small_cnn_case", kw, 2, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 5}))
    # BatchNorm after every conv: dense starts, and a patches start.
    kw = {"seed": 4, "n_boxes": 3, "big_first": False}
    out.append(("cnnbn_dense_crown", "small_cnn_bn_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("cnnbn_dense_alpha", "small_cnn_bn_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 6}))
    kw = {"seed": 6, "n_boxes": 2, "big_first": True}
    out.append(("cnnbn_patch_crown", "small_cnn_bn_case", kw, 2, abi.METHOD_CROWN, {}))
    out.append(("cnnbn_patch_alpha", "small_cnn_bn_case", kw, 2, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 4}))
    # A strided transposed conv below a linear head, and below another conv.
    kw = {"seed": 1, "n_boxes": 3}
    out.append(("convt_crown", "convt_cnn_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("convt_alpha", "convt_cnn_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 6}))
    kw = {"seed": 2, "n_boxes": 3, "conv_after": True}
    out.append(("convt2_crown", "convt_cnn_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("convt2_alpha", "convt_cnn_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 6}))
    # Residual blocks (identity and projection skips): dense starts, and
    # patches starts at the block convs.
    kw = {"seed": 7, "n_boxes": 3}
    out.append(("resnet_crown", "small_resnet_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("resnet_alpha", "small_resnet_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 6}))
    kw = {"seed": 8, "n_boxes": 2, "big": True}
    out.append(("resnetbig_crown", "small_resnet_case", kw, 2, abi.METHOD_CROWN, {}))
    out.append(("resnetbig_alpha", "small_resnet_case", kw, 1, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 3}))
    # Sigmoid activations (CROWN only: Luna's alpha-CROWN throws on any
    # Sigmoid node, AlphaCROWNAnalysis.cpp:264-272).
    out.append(("sig_crown", "sigmoid_mlp_case", {"seed": 0}, 4, abi.METHOD_CROWN, {}))
    out.append(("sigmix_crown", "sigmoid_mlp_case", {"seed": 1, "acts": (abi.NODE_RELU, abi.NODE_SIGMOID),
                                                      "eps": 1.0}, 4, abi.METHOD_CROWN, {}))
    out.append(("sigwide_crown", "sigmoid_mlp_case", {"seed": 3, "eps": 8.0}, 4, abi.METHOD_CROWN, {}))
    out.append(("resnetsig_crown", "small_resnet_case", {"seed": 9, "n_boxes": 3, "head_act": abi.NODE_SIGMOID},
                3, abi.METHOD_CROWN, {}))
    # The CIFAR-shaped CNN at full size, one box.
    out.append(("cnn_cifar_crown", "cnn_cifar", {"n_boxes": 1}, 1, abi.METHOD_CROWN, {}))
    return out


def make_case(gen: str, kw: dict):
    g, bx = getattr(W, gen)(**kw)
    if gen == "random_mlp_case":
        # Edge cases: a zero-width box and a box with some zero-width dimensions.
        bx.upper[0] = bx.lower[0]
        bx.upper[1, ::2] = bx.lower[1, ::2]
    return g, bx


def main(only=()):
    for name, gen, kw, nb, method, over in cases():
        if only and name not in only:
            continue
        g, bx = make_case(gen, kw)
        bx = bx.slice(0, nb)
        opt = abi.default_options(**over)
        res = luna_ref.compute_bounds(g, bx, method, opt, intermediate=method != abi.METHOD_IBP)
        payload = dict(lower=bx.lower, upper=bx.upper, C=bx.C, lb=res[0], ub=res[1],
                       method=np.int32(method), generator=np.str_(gen),
                       kwargs=np.str_(repr(kw)), options=np.str_(repr(over)),
                       weights_sha256=np.str_(weights_digest(g)))
        if method != abi.METHOD_IBP:
            payload["inter_lb"] = res[2]
            payload["inter_ub"] = res[3]
        np.savez_compressed(os.path.join(OUT, name + ".npz"), **payload)
        print(name, res[0].shape, float(res[0].min()), float(res[1].max()))


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
