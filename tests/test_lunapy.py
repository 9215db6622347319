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
    G.parity("lunapy/" + name, lb, ub, c["lb"][:n], c["ub"][:n])


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
        G.parity(f"lunapy one box {b}", one.lower(), one.upper(), res.lower()[b], res.upper()[b])
        y = m.forward(0.5 * (bx.lower[b] + bx.upper[b]))
        assert (one.lower() <= y + 1e-5).all() and (y <= one.upper() + 1e-5).all()


def test_vnnlib_constructor_reads_box_and_spec(tmp_path):
    """TorchModel(graph, vnnlib_path): the box and the specification come
    from the property file (CPU: nothing is bounded)."""
    from luna_b200 import workloads as W
    g, _ = W.mlp_5_50x6_5(n_boxes=1)
    f = tmp_path / "p.vnnlib"
    f.write_text("(assert (<= X_0 0.5))\n(assert (>= X_0 -0.5))\n"
                 "(assert (or (and (>= Y_1 Y_0)) (and (>= Y_2 Y_0))))\n")
    m = TorchModel(g, str(f))
    b = m.getInputBounds()
    assert b.lower()[0] == -0.5 and b.upper()[0] == 0.5 and np.isinf(b.lower()[1])
    assert m.hasSpecificationMatrix()
    m.setSpecificationMatrix(np.eye(5, dtype=np.float32))
    assert m._property is None


@pytest.mark.gpu
def test_vnnlib_property_through_lunapy(tmp_path):
    import golden_cases as G
    c = G.load_prop("prop_mlp5_or_alpha")
    lo, hi = c["lower"][6], c["upper"][6]
    text = c["text"] + "".join(f"(assert (>= X_{k} {float(v):.9g}))\n(assert (<= X_{k} {float(w):.9g}))\n"
                               for k, (v, w) in enumerate(zip(lo, hi)))
    f = tmp_path / "p.vnnlib"
    f.write_text(text)
    m = TorchModel(c["graph"], str(f), options=c["options"])
    r = m.compute_bounds("alpha-CROWN")
    assert G.excess(r.lower(), c["lb"][6]) <= 1.0
    assert m.propertyStatus() == abi.STATUS_NAMES[int(c["status"][6])]
    # A batch of sub-boxes: one verdict per box.
    m.setInputBounds(c["lower"][:4], c["upper"][:4])
    m.compute_bounds("alpha-CROWN")
    assert m.propertyStatus() == [abi.STATUS_NAMES[int(v)] for v in c["status"][:4]]
