"""A resumable sweep on the GPU: the property workload's split bounded in
chunks, interrupted after two chunks and resumed, gives the bounds and
verdicts of one call over every sub-domain."""
import os

import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.engine import Model
from luna_b200.sweep import SweepDir, run_sweep
from luna_b200.vnnlib import Property

pytestmark = pytest.mark.gpu


def test_sweep_resumes_to_the_one_call_result(tmp_path):
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available()
    g, split, text = W.mlp_property_split()
    # The first 64 sub-domains, as a split of their own (6 of the 9 groups).
    sub = W.SubdomainSplit(split.lower, split.upper, split.centre, split.C, split.groups[:6])
    prop = Property(text, 784, 10)
    m = Model(g, options=abi.default_options(alpha_lr=0.1, alpha_iterations=20))
    sd = run_sweep(m, sub, abi.METHOD_ALPHA_CROWN, str(tmp_path), chunk=16, prop=prop, max_chunks=2)
    assert len(sd.pending()) == 2
    os.remove(os.path.join(str(tmp_path), "chunk_000001.npz"))   # lost with the interrupted process
    sd = run_sweep(m, sub, abi.METHOD_ALPHA_CROWN, str(tmp_path), chunk=16, prop=prop)
    lb, ub, st = sd.collect()
    bx = sub.boxes(0, 64)
    rlb, rub, rst = m.compute_property(prop, abi.METHOD_ALPHA_CROWN, bx.lower, bx.upper)
    assert G.excess(lb, rlb) <= 1.0 and G.excess(ub, rub) <= 1.0
    assert np.array_equal(st, rst)
    # Without a property: the split's own specification, no verdicts.
    sd2 = run_sweep(m, sub, abi.METHOD_CROWN, str(tmp_path / "crown"), chunk=32)
    lb2, ub2, st2 = sd2.collect()
    r2 = m.compute_bounds(bx, abi.METHOD_CROWN)
    assert st2 is None and G.excess(lb2, r2[0]) <= 1.0 and G.excess(ub2, r2[1]) <= 1.0
    assert isinstance(sd2, SweepDir)
