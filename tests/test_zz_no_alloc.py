"""lb200_ibp_bounds_noalloc, the entry point for callers that cannot
allocate device memory where they need bounds (a service that reserves its
GPU memory up front, or a host whose memory manager owns all allocations):
it must give the same IBP bounds as the allocating entry point, call after
call, from its fixed scratch array.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test; it also passes on its own."""
import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.engine import EngineError, Model

pytestmark = pytest.mark.gpu


def _device(bx):
    return (torch.from_numpy(bx.lower).cuda(), torch.from_numpy(bx.upper).cuda(),
            torch.from_numpy(bx.C).cuda())


def test_no_alloc_ibp_matches_allocating_entry_point():
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available()
    g, boxes = W.mlp_784_256x4_10(128)
    m = Model(g)
    s = torch.cuda.current_stream().cuda_stream
    for call, (a, b) in enumerate([(0, 64), (64, 128)]):  # two calls in a row, different boxes
        bx = boxes.slice(a, b)
        xl, xu, Cm = _device(bx)
        n, nspec = bx.n, bx.C.shape[1]
        ref_l = torch.empty((n, nspec), device="cuda")
        ref_u = torch.empty((n, nspec), device="cuda")
        m.compute_bounds_ptr(abi.METHOD_IBP, xl.data_ptr(), xu.data_ptr(), n, Cm.data_ptr(), Cm.shape[0],
                             nspec, ref_l.data_ptr(), ref_u.data_ptr(), s)
        out_l = torch.full((n, nspec), float("nan"), device="cuda")
        out_u = torch.full((n, nspec), float("nan"), device="cuda")
        m.ibp_bounds_noalloc_ptr(xl.data_ptr(), xu.data_ptr(), n, Cm.data_ptr(), Cm.shape[0], nspec,
                                 out_l.data_ptr(), out_u.data_ptr(), s)
        torch.cuda.synchronize()
        ol, ou = out_l.cpu().numpy(), out_u.cpu().numpy()
        rl, ru = ref_l.cpu().numpy(), ref_u.cpu().numpy()
        assert np.isfinite(ol).all() and np.isfinite(ou).all(), call
        assert G.excess(ol, rl) <= 1.0 and G.excess(ou, ru) <= 1.0, call


def test_no_alloc_rejects_batches_above_its_scratch():
    g, bx = W.mlp_784_256x4_10(4)
    m = Model(g)
    xl, xu, Cm = _device(bx)
    out = torch.empty((4, 9), device="cuda")
    too_many = 3000  # 3000 boxes x 2 x 1034 floats > 4 Mi floats
    with pytest.raises(EngineError, match="scratch"):
        m.ibp_bounds_noalloc_ptr(xl.data_ptr(), xu.data_ptr(), too_many, Cm.data_ptr(), 1, 9,
                                 out.data_ptr(), out.data_ptr())
    # Sizes whose products overflow 32 or 64 bits are refused before any launch.
    for n in (2 ** 31, (2 ** 63 - 1) // 2068 + 1, 2 ** 62):
        with pytest.raises(EngineError, match="2\\^31|scratch"):
            m.ibp_bounds_noalloc_ptr(xl.data_ptr(), xu.data_ptr(), n, Cm.data_ptr(), 1, 9,
                                     out.data_ptr(), out.data_ptr())
    with pytest.raises(EngineError, match="2\\^31"):
        m.ibp_bounds_noalloc_ptr(xl.data_ptr(), xu.data_ptr(), 4, Cm.data_ptr(), 1, 2 ** 30,
                                 out.data_ptr(), out.data_ptr())


def test_no_alloc_rejects_networks_other_than_linear_relu():
    """A conv network is refused with an error (nothing is launched)."""
    g, bx = W.small_cnn_case(1, n_boxes=2, big_first=False)
    m = Model(g)
    xl, xu, Cm = _device(bx)
    n, nspec = bx.n, bx.C.shape[1]
    out = torch.empty((n, nspec), device="cuda")
    with pytest.raises(EngineError, match="Linear/ReLU"):
        m.ibp_bounds_noalloc_ptr(xl.data_ptr(), xu.data_ptr(), n, Cm.data_ptr(), Cm.shape[0], nspec,
                                 out.data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
