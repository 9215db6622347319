"""Fixtures of the CPU oracle (oracle/lirpa_oracle.py) on networks at their
full workload size, where Luna itself cannot give a reference in bounded
time or at all:

* oracle_resnet_cifar_crown: the CIFAR ResNet of the ResNet workload
  (3x32x32, stem 16, residual blocks 16/16/32s2/32 with BatchNorm, Sigmoid
  head); Luna's alpha-CROWN throws on its Sigmoid node
  (AlphaCROWNAnalysis.cpp:264-272);
* oracle_convt_sweep_crown: the transposed-conv CIFAR CNN of the sub-domain
  sweep, on its first sub-domains.
At these sizes almost every pre-activation is IBP-unstable (16384 rows per
start on the ResNet, 32768 on the sweep network), and the oracle keeps dense
A matrices: CROWN fits in host memory, while alpha-CROWN, which keeps every
start's A for autograd, needs well over 60 GB; the alpha paths of both
networks are pinned on their smaller relatives (resnet_*, convt_* fixtures).

The oracle itself is pinned against Luna's outputs by
tests/test_oracle_golden.py.  Boxes and weights are regenerated from the
seeded generators and checked by checksum, as for Luna's large fixtures.

    python tests/golden/make_oracle_golden.py [case names]
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from luna_b200 import abi, workloads as W  # noqa: E402
from make_golden import boxes_digest, weights_digest  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle")


def cases():
    """(name, generator, kwargs, box count, method, option overrides)."""
    return [
        ("oracle_resnet_cifar_crown", "resnet_cifar", {"n_boxes": 128}, 2, abi.METHOD_CROWN, {}),
        ("oracle_convt_sweep_crown", "convt_sweep_boxes", {"n_boxes": 256}, 2, abi.METHOD_CROWN, {}),
    ]


def main(only=()):
    import torch
    from oracle.lirpa_oracle import LirpaOracle
    torch.set_num_threads(os.cpu_count() or 1)
    os.makedirs(OUT, exist_ok=True)
    for name, gen, kw, nb, method, over in cases():
        if only and name not in only:
            continue
        g, bx = getattr(W, gen)(**kw)
        bx = bx.slice(0, nb)
        opt = abi.default_options(**over)
        t0 = time.time()
        lb, ub = LirpaOracle(g, opt).compute_bounds(bx, method)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), lb=lb, ub=ub, method=np.int32(method),
                            generator=np.str_(gen), kwargs=np.str_(repr(kw)), options=np.str_(repr(over)),
                            weights_sha256=np.str_(weights_digest(g)), box_range=np.array([0, nb], np.int64),
                            boxes_sha256=np.str_(boxes_digest(bx)))
        print(name, lb.shape, float(lb.min()), float(ub.max()), f"{time.time() - t0:.0f} s", flush=True)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
