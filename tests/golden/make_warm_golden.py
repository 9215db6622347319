"""Generate the warm-start golden fixtures in tests/golden/warm/ by running Luna.

Branch-and-bound bounds a sub-domain after loading its parent's state: the
parent box is bounded with alpha-CROWN, TorchModel::getState() taken and
handed to TorchModel::loadState() with the child's box, and the child
bounded with alpha-CROWN (oracle/luna_ref_driver.cpp,
luna_ref_compute_bounds_warm).  Each parent here is split in half along one
input dimension (the lower half for even children, the upper half for odd
ones), as an input split of branch-and-bound does.  Luna's fresh bounds of
the same children are stored beside the warm ones, to show that the state
changes the result.

    make -C oracle && python tests/golden/make_warm_golden.py [case names | split3]

Cases on networks with convolutions go to tests/golden/warm_conv/.  It
also writes tests/golden/warm_chain/split3.npz: Luna's bounds down a
three-level split tree, each box bounded after the state of the one above
it (getState / loadState repeated, luna_ref_compute_bounds_chain).
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from luna_b200 import abi, workloads as W  # noqa: E402
from luna_b200.workloads import Boxes  # noqa: E402
from oracle import luna_ref  # noqa: E402
from make_golden import weights_digest  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "warm")


def cases():
    """(name, generator, generator kwargs, option overrides, input dimensions split over)."""
    return [
        ("mlp5_warm", "mlp_5_50x6_5", {"n_boxes": 12}, {"alpha_lr": 0.1, "alpha_iterations": 8}, 5),
        ("rand_warm", "random_mlp_case", {"seed": 42, "n_boxes": 12, "depth": 3, "width": 16, "n_in": 6},
         {"alpha_lr": 0.1, "alpha_iterations": 10}, 6),
        ("mlp784_warm", "mlp_784_256x4_10", {"n_boxes": 6}, {"alpha_lr": 0.1, "alpha_iterations": 20}, 784),
    ]


def conv_cases():
    """Warm-start cases on networks with convolutions (tests/golden/warm_conv/):
    dense conv starts, a patches start (a first conv of 4608 features), and
    a strided transposed conv."""
    a5 = {"alpha_lr": 0.1, "alpha_iterations": 5}
    return [
        ("cnn_warm", "small_cnn_case", {"seed": 3, "n_boxes": 3, "big_first": False}, a5, None),
        ("cnnpatch_warm", "small_cnn_case", {"seed": 5, "n_boxes": 2, "big_first": True}, a5, None),
        ("convt_warm", "convt_cnn_case", {"seed": 1, "n_boxes": 2}, a5, None),
    ]


def children_of(bx: Boxes, nd: int) -> Boxes:
    """Child b: box b halved along input dimension (7 b) mod nd, the lower
    half for even b and the upper half for odd b (midpoint in fp32)."""
    lo = bx.lower.copy()
    hi = bx.upper.copy()
    for b in range(bx.n):
        d = (7 * b) % nd
        mid = np.float32((np.float32(bx.lower[b, d]) + np.float32(bx.upper[b, d])) / np.float32(2))
        if b % 2 == 0:
            hi[b, d] = mid
        else:
            lo[b, d] = mid
    return Boxes(lo, hi, bx.C.copy())


def start_rows(graph, bx):
    """Rows of every intermediate start per box: the IBP-unstable count of
    each pre-activation after the first (numpy interval arithmetic)."""
    lin = [nd for nd in graph.nodes if nd.type == abi.NODE_LINEAR]
    l, u = bx.lower.astype(np.float64), bx.upper.astype(np.float64)
    rows = []
    for k, nd in enumerate(lin[:-1]):
        W = np.asarray(nd.weight, np.float64) * nd.scale
        b = np.asarray(nd.bias, np.float64) if nd.bias is not None else 0.0
        if k > 0:
            l, u = np.maximum(l, 0), np.maximum(u, 0)
        Wp, Wn = np.maximum(W, 0), np.minimum(W, 0)
        l, u = l @ Wp.T + u @ Wn.T + b, u @ Wp.T + l @ Wn.T + b
        if k > 0:
            rows.append(((l < 0) & (u > 0)).sum(1))
    return np.stack(rows, 1)


def make_chain():
    """Luna down the paths of golden_cases.split_chain()'s tree: for leaf k
    the path is (root p1[p2[k]], level-1 box p2[k], level-2 box k).  Only
    paths whose level-1 box reuses every seeded alpha (each start has as
    many rows as at the root) are kept: where Luna recreates one, its best
    map keeps the seeded alpha's unstableIndices beside the new alpha
    (AlphaCROWNAnalysis.cpp:601 replaces only `alpha`), so the state it hands
    to level 2 pairs new values with old indices (its next run then throws a
    scatter-shape error when there are fewer values than indices)."""
    import golden_cases as GC
    g, opt, (L0, L1, L2), (p1, p2) = GC.split_chain()
    r0 = start_rows(g, L0)[p1[p2]]
    r1 = start_rows(g, L1)[p2]
    keep = np.nonzero((r0 == r1).all(1))[0]
    lo = np.stack([L0.lower[p1[p2]], L1.lower[p2], L2.lower], axis=1)[keep]
    hi = np.stack([L0.upper[p1[p2]], L1.upper[p2], L2.upper], axis=1)[keep]
    lb, ub = luna_ref.compute_bounds_chain(g, lo, hi, L2.C[keep], opt)
    out = os.path.join(os.path.dirname(OUT), "warm_chain")
    os.makedirs(out, exist_ok=True)
    levels = {f"lower{k}": L.lower for k, L in enumerate((L0, L1, L2))}
    levels.update({f"upper{k}": L.upper for k, L in enumerate((L0, L1, L2))})
    np.savez_compressed(os.path.join(out, "split3.npz"), leaves=keep, lb1=lb[:, 1], ub1=ub[:, 1], lb2=lb[:, 2],
                        ub2=ub[:, 2], weights_sha256=np.str_(weights_digest(g)), **levels)
    print("split3: paths kept", keep.tolist(), "of", len(p2), flush=True)


def main(only=()):
    for name, gen, kw, over, nd in cases() + conv_cases():
        if only and name not in only:
            continue
        out_dir = OUT if nd is not None else os.path.join(os.path.dirname(OUT), "warm_conv")
        os.makedirs(out_dir, exist_ok=True)
        g, parents = getattr(W, gen)(**kw)
        kids = children_of(parents, nd if nd is not None else parents.lower.shape[1])
        opt = abi.default_options(**over)
        lb, ub = luna_ref.compute_bounds_warm(g, parents, kids, opt)
        flb, fub = luna_ref.compute_bounds(g, kids, abi.METHOD_ALPHA_CROWN, opt)
        moved = int(np.sum(np.any((lb != flb) | (ub != fub), axis=1)))
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), lb=lb, ub=ub, fresh_lb=flb, fresh_ub=fub,
                            parent_lower=parents.lower, parent_upper=parents.upper, lower=kids.lower,
                            upper=kids.upper, C=kids.C, generator=np.str_(gen), kwargs=np.str_(repr(kw)),
                            options=np.str_(repr(over)), weights_sha256=np.str_(weights_digest(g)))
        print(name, lb.shape, f"warm differs from fresh on {moved}/{lb.shape[0]} boxes", flush=True)


if __name__ == "__main__":
    args = tuple(sys.argv[1:])
    rest = tuple(a for a in args if a != "split3")
    if not args or "split3" in args:
        make_chain()
    if not args or rest:
        main(rest)
