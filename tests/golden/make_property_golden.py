"""Generate tests/golden/prop_*.npz: Luna bounding boxes against VNN-LIB
properties, the CLI's flow (TorchModel(onnx, vnnlib), compute_bounds with the
property's thresholds kept, evaluatePropertyStatus).

Each case writes a property text whose thresholds are quantiles of Luna's own
bounds over the boxes, so that some boxes are verified by the initial CROWN
pass (STOP_CROWN_ON_VERIFIED), some part-way through the alpha optimisation
(STOP_ALPHA_ON_VERIFIED) and some not at all.  The property is read by Luna's
parser (oracle/_ref/luna_ref_vnnlib) and bounded by Luna's engine
(oracle/_ref/libluna_ref.so); the text, the boxes and Luna's bounds and
verdicts are stored.

    make -C oracle && python tests/golden/make_property_golden.py [case names]
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from luna_b200 import abi, workloads as W  # noqa: E402
from luna_b200.workloads import Boxes  # noqa: E402
from oracle import luna_ref  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def margin_rows(n_out: int, label: int):
    """Rows Y_label - Y_j for j != label (the robustness margins)."""
    rows = []
    for j in range(n_out):
        if j != label:
            c = np.zeros(n_out, np.float32)
            c[label], c[j] = 1, -1
            rows.append((j, c))
    return rows


def property_text(n_in: int, n_out: int, label: int, thr, kind: str) -> str:
    """Counterexample: Y_label - Y_j <= t_j for one j (kind "or"), or for every
    j (kind "conj")."""
    lines = [f"; margins of output {label}, {kind}"]
    lines += [f"(declare-const X_{k} Real)" for k in range(n_in)]
    lines += [f"(declare-const Y_{k} Real)" for k in range(n_out)]
    cmps = [f"(<= (- Y_{label} Y_{j}) {float(t):.9g})" for (j, _), t in zip(margin_rows(n_out, label), thr)]
    if kind == "or":
        lines.append("(assert (or " + " ".join(f"(and {c})" for c in cmps) + "))")
    elif kind == "conj":
        lines += [f"(assert {c})" for c in cmps]
    return "\n".join(lines) + "\n"


def cases():
    """(name, generator, kwargs, n_boxes, method, options, kind, quantile)."""
    return [
        ("prop_mlp5_conj_alpha", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 0.1}, "conj", 0.6),
        ("prop_mlp5_or_alpha", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 0.1}, "or", 0.3),
        ("prop_mlp5_or_crown", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_CROWN, {}, "or", 0.3),
        ("prop_mlp5_nocrownstop_alpha", "mlp_5_50x6_5", {"n_boxes": 16}, 16, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 0.1, "stop_crown_on_verified": 0}, "conj", 0.6),
        ("prop_rand_or_alpha", "random_mlp_case", {"seed": 103, "n_boxes": 8, "depth": 3, "width": 16}, 8,
         abi.METHOD_ALPHA_CROWN, {"alpha_lr": 0.5, "alpha_iterations": 12}, "or", 0.4),
        ("prop_mlp784_conj_alpha", "mlp_784_256x4_10", {"n_boxes": 4}, 4, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 0.1}, "conj", 0.5),
        ("prop_mlp5_none_crown", "mlp_5_50x6_5", {"n_boxes": 4}, 4, abi.METHOD_CROWN, {}, "none", 0.0),
        # Conv paths: dense starts, a patches start, residual joins.
        ("prop_cnn_or_alpha", "small_cnn_case", {"seed": 3, "n_boxes": 6, "big_first": False}, 6,
         abi.METHOD_ALPHA_CROWN, {"alpha_lr": 0.1, "alpha_iterations": 8}, "or", 0.4),
        ("prop_cnnpatch_conj_alpha", "small_cnn_case", {"seed": 5, "n_boxes": 4, "big_first": True}, 4,
         abi.METHOD_ALPHA_CROWN, {"alpha_lr": 0.1, "alpha_iterations": 5}, "conj", 0.5),
        ("prop_resnet_or_alpha", "small_resnet_case", {"seed": 7, "n_boxes": 4}, 4, abi.METHOD_ALPHA_CROWN,
         {"alpha_lr": 0.1, "alpha_iterations": 6}, "or", 0.5),
    ]


def main(only=()):
    for name, gen, kw, nb, method, over, kind, q in cases():
        if only and name not in only:
            continue
        g, bx = getattr(W, gen)(**kw)
        bx = bx.slice(0, nb)
        n_in = bx.lower.shape[1]
        n_out = int(np.prod(g.nodes[g.output_index].out_shape))
        label = 0
        rows = margin_rows(n_out, label)
        Cm = np.stack([c for _, c in rows])[None]
        opt = abi.default_options(**over)
        # Each threshold halfway between two neighbouring alpha-CROWN margins
        # of the boxes, so no box's bound sits at a threshold (a verdict
        # there would turn on the last bits of the arithmetic).
        base = abi.default_options(**{k: v for k, v in over.items() if not k.startswith("stop_")})
        lA, _ = luna_ref.compute_bounds(g, Boxes(bx.lower, bx.upper, Cm), abi.METHOD_ALPHA_CROWN, base)
        srt = np.sort(lA, axis=0)
        k = min(max(int(q * (nb - 1)), 0), nb - 2)
        thr = (0.5 * (srt[k] + srt[k + 1])).astype(np.float32)
        text = property_text(n_in, n_out, label, thr, kind)
        spec = luna_ref.vnnlib_parse(text, n_in, n_out)
        lb, ub, st = luna_ref.compute_property(g, spec, bx.lower, bx.upper, method, opt)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), lower=bx.lower, upper=bx.upper, lb=lb, ub=ub,
                            status=st, text=np.str_(text), method=np.int32(method), generator=np.str_(gen),
                            kwargs=np.str_(repr(kw)), options=np.str_(repr(over)))
        print(name, "status", st.tolist())


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
