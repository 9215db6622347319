"""luna_b200.lunapy: Luna's Python API (lunapy.TorchModel) over the engine."""
import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.lunapy import BoundedTensor, TorchModel


def test_model_interface_on_cpu():
    g, bx = W.mlp_5_50x6_5(3)
    m = TorchModel(g)
    assert (m.getInputSize(), m.getOutputSize(), m.getNumNodes()) == (5, 5, len(g.nodes))
    assert not m.hasInputBounds() and not m.hasSpecificationMatrix() and not m.hasFinalAnalysisBounds()
    with pytest.raises(ValueError):
        m.setInputBounds(np.zeros(4), np.ones(4))
    with pytest.raises(ValueError):
        m.setInputBounds(np.ones(5), np.zeros(5))
    m.setInputBounds(bx.lower[0], bx.upper[0])
    b = m.getInputBounds()
    assert isinstance(b, BoundedTensor) and np.array_equal(b.lower(), bx.lower[0])
    with pytest.raises(ValueError):
        m.setSpecificationMatrix(np.ones((2, 4)))
    m.setSpecificationMatrix(bx.C[0])
    assert m.hasSpecificationMatrix()
    y = m.forward(bx.lower[0])
    assert y.shape == (5,)
    assert np.allclose(y, W.graph_forward(g, torch.from_numpy(bx.lower[:1])).detach().numpy()[0])
    with pytest.raises(ValueError):
        m.compute_bounds(method="DeepPoly")
    with pytest.raises(NotImplementedError):
        TorchModel("model.onnx")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["mlp5_crown", "mlp5_alpha", "cnn_dense_crown", "resnet_crown"])
def test_compute_bounds_per_box_matches_luna(name):
    """Box by box, as a lunapy user calls it, against Luna's golden bounds."""
    from luna_b200.build import build
    build()
    c = G.load(name)
    m = TorchModel(c["graph"], options=c["options"])
    method = {abi.METHOD_CROWN: "CROWN", abi.METHOD_ALPHA_CROWN: "alpha-CROWN"}[c["method"]]
    bx = c["boxes"]
    lbs, ubs = [], []
    for b in range(min(bx.n, 4)):
        m.setInputBounds(bx.lower[b], bx.upper[b])
        res = m.compute_bounds(method=method, C=bx.C[0 if bx.C.shape[0] == 1 else b])
        assert res.lower().shape == (bx.C.shape[1],) and m.getFinalAnalysisBounds() is res
        lbs.append(res.lower())
        ubs.append(res.upper())
    n = len(lbs)
    lb, ub = np.stack(lbs), np.stack(ubs)
    scaled = max(G.excess_scaled(lb, c["lb"][:n], c["lb"][:n], c["ub"][:n]),
                 G.excess_scaled(ub, c["ub"][:n], c["lb"][:n], c["ub"][:n]))
    assert scaled <= 1.0, scaled


@pytest.mark.gpu
def test_identity_specification_and_batches():
    """Without C: bounds of every output; a batch gives the per-box results."""
    from luna_b200.build import build
    build()
    g, bx = W.mlp_5_50x6_5(4)
    m = TorchModel(g)
    m.setInputBounds(bx.lower, bx.upper)
    res = m.runCROWN()
    assert res.lower().shape == (4, 5) and (res.lower() <= res.upper()).all()
    for b in range(4):
        m.setInputBounds(bx.lower[b], bx.upper[b])
        one = m.compute_bounds()
        assert G.excess_scaled(one.lower(), res.lower()[b], res.lower()[b], res.upper()[b]) <= 1.0
        assert G.excess_scaled(one.upper(), res.upper()[b], res.lower()[b], res.upper()[b]) <= 1.0
        y = m.forward(0.5 * (bx.lower[b] + bx.upper[b]))
        assert (one.lower() <= y + 1e-5).all() and (y <= one.upper() + 1e-5).all()
