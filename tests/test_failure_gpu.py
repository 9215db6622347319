"""Failure detection on the GPU without a GPU fault: the tensor-core
kernels' bounded waits (tc_ptx.cuh: mbar_wait) are made to run out by a
test hook that has the TMA producers issue no loads -- a barrier nothing
completes.  The kernels must raise the device error flag and return, the
call must fail with an error, and the context must stay usable: the next
call on the same model gives the right bounds."""
import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.engine import EngineError, Model, set_contraction_fault

pytestmark = pytest.mark.gpu


def test_expired_waits_fail_the_call_and_leave_the_context_usable():
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available()
    g, bx = W.mlp_784_256x4_10(4)  # widths multiples of 16: tensor-core contractions
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=3)
    m = Model(g, options=opt)
    ref = m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    try:
        # ~0.5 ms per wait at 2 GHz, so the expired waits cost little.
        set_contraction_fault(0, True, 1_000_000)
        with pytest.raises(EngineError, match="bounded wait expired"):
            m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    finally:
        set_contraction_fault(0, False, 0)
    torch.cuda.synchronize()
    lb, ub = m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    assert np.array_equal(lb, ref[0]) and np.array_equal(ub, ref[1])
    G.parity("after expired waits", lb, ub, ref[0], ref[1])
