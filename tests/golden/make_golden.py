"""Generate the golden fixtures in tests/golden/ by running Luna itself.

Luna's own CPU implementation (compiled from the reference sources by
oracle/Makefile into oracle/_ref/libluna_ref.so) bounds every case below;
the inputs and Luna's outputs are stored as .npz files.  Network weights are
not stored: they are regenerated from the seeded generators in
luna_b200/workloads.py, and a checksum of them is stored to catch drift.

    make -C oracle && python tests/golden/make_golden.py [--procs P] [case names]
    python tests/golden/make_golden.py --part K N case   # boxes of part K of N only
    python tests/golden/make_golden.py --merge N case    # assemble the N parts

Large cases run Luna on several host processes (one box range and one ATen
thread per process, as the CPU baseline does); their boxes are regenerated
from the seeded generator too and only a checksum is stored.  A case whose
Luna processes need too much host memory to run side by side is made in
parts (separate invocations, one box range each, results kept under
oracle/_ref/parts/) and then merged.
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


def boxes_digest(bx) -> str:
    h = hashlib.sha256()
    for a in (bx.lower, bx.upper, bx.C):
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


# Cases whose boxes are regenerated rather than stored, and that carry no
# intermediate bounds (their size would dominate the fixture directory).
LARGE = {"cfg2_alpha512", "cfg3_alpha"}


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
    # Sub (a constant on the input, or on a Linear output; x - c and c - x),
    # Slice of flat vectors (after a Linear, and feeding one, step 1 and -1),
    # Concat of Linear / Conv outputs, Reshape as a flatten.
    a6 = {"alpha_lr": 0.1, "alpha_iterations": 6}
    out.append(("sub_in_crown", "sub_mlp_case", {"seed": 1}, 6, abi.METHOD_CROWN, {}))
    out.append(("sub_in_alpha", "sub_mlp_case", {"seed": 1}, 6, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("sub_in_neg_alpha", "sub_mlp_case", {"seed": 2, "constant_second": 0}, 6, abi.METHOD_ALPHA_CROWN,
                a6))
    out.append(("sub_lin_alpha", "sub_mlp_case", {"seed": 3, "where": "linear"}, 6, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("sub_lin_neg_crown", "sub_mlp_case", {"seed": 4, "where": "linear", "constant_second": 0}, 6,
                abi.METHOD_CROWN, {}))
    out.append(("slice_crown", "slice_mlp_case", {"seed": 5}, 6, abi.METHOD_CROWN, {}))
    out.append(("slice_alpha", "slice_mlp_case", {"seed": 5}, 6, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("slice_rev_alpha", "slice_mlp_case", {"seed": 6, "reverse": True}, 6, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("concat_crown", "concat_mlp_case", {"seed": 7}, 6, abi.METHOD_CROWN, {}))
    out.append(("concat_alpha", "concat_mlp_case", {"seed": 7}, 6, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("concat_cnn_crown", "concat_cnn_case", {"seed": 8}, 3, abi.METHOD_CROWN, {}))
    out.append(("concat_cnn_alpha", "concat_cnn_case", {"seed": 8}, 3, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("sub_cnn_alpha", "sub_cnn_case", {"seed": 9}, 3, abi.METHOD_ALPHA_CROWN, a6))
    out.append(("sub_cnn_neg_crown", "sub_cnn_case", {"seed": 10, "constant_second": 0}, 3, abi.METHOD_CROWN, {}))
    # Strided 32/64-channel convs: the tensor-core (tcgen05) conv steps.
    kw = {"seed": 21, "n_boxes": 3}
    out.append(("cnnwide_crown", "cnn_wide_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("cnnwide_alpha", "cnn_wide_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 6}))
    # A 32 -> 32-channel transposed conv: the tensor-core transposed-conv steps.
    kw = {"seed": 11, "n_boxes": 3, "tc": True}
    out.append(("convttc_crown", "convt_cnn_case", kw, 3, abi.METHOD_CROWN, {}))
    out.append(("convttc_alpha", "convt_cnn_case", kw, 3, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 5}))
    # OPTIMIZE_UPPER: the upper side optimised first, then the lower side
    # (both), the upper side alone, and neither (runCROWN).
    up = {"alpha_lr": 0.1, "alpha_iterations": 6, "optimize_upper": 1}
    out.append(("mlp5_alpha_upper", "mlp_5_50x6_5", {"n_boxes": 8}, 8, abi.METHOD_ALPHA_CROWN, up))
    out.append(("mlp5_alpha_uponly", "mlp_5_50x6_5", {"n_boxes": 8}, 8, abi.METHOD_ALPHA_CROWN,
                dict(up, optimize_lower=0)))
    out.append(("mlp5_alpha_noopt", "mlp_5_50x6_5", {"n_boxes": 8}, 8, abi.METHOD_ALPHA_CROWN,
                dict(up, optimize_lower=0, optimize_upper=0)))
    out.append(("mlp784_alpha_upper", "mlp_784_256x4_10", {"n_boxes": 3}, 3, abi.METHOD_ALPHA_CROWN, up))
    out.append(("cnn_dense_alpha_upper", "small_cnn_case", {"seed": 3, "n_boxes": 4, "big_first": False}, 2,
                abi.METHOD_ALPHA_CROWN, up))
    out.append(("cnn_patch_alpha_upper", "small_cnn_case", {"seed": 5, "n_boxes": 3, "big_first": True}, 2,
                abi.METHOD_ALPHA_CROWN, dict(up, alpha_iterations=4)))
    out.append(("resnet_alpha_upper", "small_resnet_case", {"seed": 7, "n_boxes": 3}, 2, abi.METHOD_ALPHA_CROWN,
                dict(up, alpha_iterations=4)))
    out.append(("convt_alpha_upper", "convt_cnn_case", {"seed": 1, "n_boxes": 3}, 2, abi.METHOD_ALPHA_CROWN,
                dict(up, alpha_iterations=4)))
    # The MLP alpha-CROWN workload at its own size: all 512 boxes, 20 Adam
    # iterations at lr 0.1.
    out.append(("cfg2_alpha512", "mlp_784_256x4_10", {"n_boxes": 512}, 512, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.1, "alpha_iterations": 20}))
    # The CIFAR CNN alpha-CROWN workload (30 Adam iterations at Luna's default
    # lr 0.5), the first 4 of its 256 boxes.
    out.append(("cfg3_alpha", "cnn_cifar", {"n_boxes": 256}, 4, abi.METHOD_ALPHA_CROWN,
                {"alpha_lr": 0.5, "alpha_iterations": 30}))
    return out


# Cases with Luna's stabilised intermediate bounds switched off
# (STABILIZE_INTERMEDIATE_BOUNDS = false), written to tests/golden/nostab/:
# a random MLP on which one box's third layer, stable when its alphas are
# created, has an unstable neuron at the first Adam iteration.
def nostab_cases():
    kw = {"seed": 39, "n_boxes": 4, "depth": 3, "width": 12, "eps": 0.2}
    return [("rand39_alpha_nostab", "random_mlp_case", kw, 4, abi.METHOD_ALPHA_CROWN,
             {"alpha_lr": 0.5, "alpha_iterations": 10, "stabilize_intermediate_bounds": 0})]


# Result-affecting options at non-default values (the default runs above
# keep Luna's defaults), written to tests/golden/options/: early-stop
# patience short enough to end runs early, the best-alpha save window moved
# both ways, a faster learning-rate decay, CROWN with the first Linear layer
# back-substituted, and a large first conv concretised densely instead of in
# patches.
def option_cases():
    a = {"alpha_lr": 0.5, "alpha_iterations": 12}
    m5 = {"n_boxes": 8}
    return [
        # lr 1.0 over 30 steps: boxes 2, 3 and 6 stop early (at 16, 19, 21).
        ("mlp5_alpha_patience2", "mlp_5_50x6_5", m5, 8, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 1.0, "alpha_iterations": 30, "early_stop_patience": 2}),
        ("mlp5_alpha_save02", "mlp_5_50x6_5", m5, 8, abi.METHOD_ALPHA_CROWN, dict(a, start_save_best=0.2)),
        ("mlp5_alpha_save09", "mlp_5_50x6_5", m5, 8, abi.METHOD_ALPHA_CROWN, dict(a, start_save_best=0.9)),
        ("mlp5_alpha_decay09", "mlp_5_50x6_5", m5, 8, abi.METHOD_ALPHA_CROWN, dict(a, alpha_lr_decay=0.9)),
        ("mlp5_crown_nofirstibp", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_CROWN,
         {"enable_first_linear_ibp": 0}),
        ("cnn_patch_crown_dense", "small_cnn_case", {"seed": 5, "n_boxes": 3, "big_first": True}, 3,
         abi.METHOD_CROWN, {"use_patches_mode": 0}),
        ("cnn_patch_alpha_dense", "small_cnn_case", {"seed": 5, "n_boxes": 3, "big_first": True}, 2,
         abi.METHOD_ALPHA_CROWN, {"alpha_lr": 0.1, "alpha_iterations": 5, "use_patches_mode": 0}),
    ]


def make_case(gen: str, kw: dict):
    g, bx = getattr(W, gen)(**kw)
    if gen == "random_mlp_case":
        # Edge cases: a zero-width box and a box with some zero-width dimensions.
        bx.upper[0] = bx.lower[0]
        bx.upper[1, ::2] = bx.lower[1, ::2]
    return g, bx


_WORK = {}


def _luna_range(task):
    """One host process: Luna on boxes [a, b) of a case, one ATen thread."""
    gen, kw, a, b, method, over = task
    key = (gen, repr(kw))
    if _WORK.get("key") != key:
        _WORK["case"] = make_case(gen, kw)
        _WORK["key"] = key
    g, bx = _WORK["case"]
    return luna_ref.compute_bounds(g, bx.slice(a, b), method, abi.default_options(**over), num_threads=1)


def run_luna(g, bx, gen, kw, nb, method, over, procs, intermediate):
    if procs <= 1 or nb <= 1:
        return luna_ref.compute_bounds(g, bx, method, abi.default_options(**over), intermediate=intermediate)
    import multiprocessing as mp
    p = min(procs, nb)
    cuts = [nb * i // p for i in range(p + 1)]
    tasks = [(gen, kw, cuts[i], cuts[i + 1], method, over) for i in range(p)]
    with mp.get_context("spawn").Pool(p) as pool:
        parts = pool.map(_luna_range, tasks, chunksize=1)
    return np.concatenate([x[0] for x in parts]), np.concatenate([x[1] for x in parts])


PARTS = os.path.join(ROOT, "oracle", "_ref", "parts")


def part_path(name, k, n):
    return os.path.join(PARTS, f"{name}.part{k}of{n}.npz")


def main(only=(), procs=1, part=None, merge=0):
    nostab = {c[0] for c in nostab_cases()}
    options = {c[0] for c in option_cases()}
    for name, gen, kw, nb, method, over in cases() + nostab_cases() + option_cases():
        if only and name not in only:
            continue
        g, bx = make_case(gen, kw)
        bx = bx.slice(0, nb)
        large = name in LARGE
        inter = method != abi.METHOD_IBP and not large
        if part is not None:
            k, n = part
            a, b = nb * k // n, nb * (k + 1) // n
            res = run_luna(g, bx.slice(a, b), gen, kw, b - a, method, over, procs, False)
            os.makedirs(PARTS, exist_ok=True)
            np.savez(part_path(name, k, n), lb=res[0], ub=res[1], box_range=np.array([a, b]))
            print(name, f"part {k} of {n}: boxes [{a}, {b})", flush=True)
            continue
        if merge:
            zs = [np.load(part_path(name, k, merge)) for k in range(merge)]
            assert [int(z["box_range"][0]) for z in zs] == [nb * k // merge for k in range(merge)]
            res = (np.concatenate([z["lb"] for z in zs]), np.concatenate([z["ub"] for z in zs]))
        else:
            res = run_luna(g, bx, gen, kw, nb, method, over, procs, inter)
        payload = dict(lb=res[0], ub=res[1], method=np.int32(method), generator=np.str_(gen),
                       kwargs=np.str_(repr(kw)), options=np.str_(repr(over)),
                       weights_sha256=np.str_(weights_digest(g)))
        if large:
            payload.update(box_range=np.array([0, nb], np.int64), boxes_sha256=np.str_(boxes_digest(bx)))
        else:
            payload.update(lower=bx.lower, upper=bx.upper, C=bx.C)
        if inter:
            payload["inter_lb"] = res[2]
            payload["inter_ub"] = res[3]
        out_dir = os.path.join(OUT, "nostab") if name in nostab else (
            os.path.join(OUT, "options") if name in options else OUT)
        os.makedirs(out_dir, exist_ok=True)
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **payload)
        print(name, res[0].shape, float(res[0].min()), float(res[1].max()), flush=True)


if __name__ == "__main__":
    argv = list(sys.argv[1:])
    procs, part, merge = 1, None, 0
    if "--procs" in argv:
        k = argv.index("--procs")
        procs = int(argv[k + 1])
        del argv[k:k + 2]
    if "--part" in argv:
        k = argv.index("--part")
        part = (int(argv[k + 1]), int(argv[k + 2]))
        del argv[k:k + 3]
    if "--merge" in argv:
        k = argv.index("--merge")
        merge = int(argv[k + 1])
        del argv[k:k + 2]
    main(tuple(argv), procs, part, merge)
