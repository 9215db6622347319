"""The CPU oracle (oracle/lirpa_oracle.py) against Luna's own outputs.

The golden fixtures were produced by Luna's CPU implementation compiled from
the reference sources (tests/golden/make_golden.py); the oracle is trusted as
the parity checker only because it reproduces them.
"""
import os

import numpy as np
import pytest
import torch

import golden_cases as G
from oracle.lirpa_oracle import LirpaOracle


@pytest.fixture(autouse=True, scope="module")
def _one_thread():
    n = torch.get_num_threads()
    torch.set_num_threads(1)
    yield
    torch.set_num_threads(n)


# Fixtures at a workload's own size: the CPU suite checks the oracle on the
# first boxes only (the GPU suite checks the engine on all of them).
ORACLE_BOXES = {"cfg2_alpha512": 48, "cfg3_alpha": 1}


@pytest.mark.parametrize("name", G.names())
def test_oracle_matches_luna(name):
    c = G.load(name)
    if c["boxes"].lower.shape[1] >= 1000:
        # Large conv maps: several cores keep the CPU suite within minutes.
        torch.set_num_threads(min(8, os.cpu_count() or 1))
    n = ORACLE_BOXES.get(name, c["boxes"].n)
    res = LirpaOracle(c["graph"], c["options"]).compute_bounds(c["boxes"].slice(0, n), c["method"],
                                                               intermediate="inter_lb" in c)
    G.parity("oracle/" + name, res[0], res[1], c["lb"][:n], c["ub"][:n])
    if "inter_lb" in c:
        e, states = G.check_intermediate(res[2], res[3], c["inter_lb"], c["inter_ub"])
        assert e <= 1.0 and states


def test_planted_error_is_caught():
    """A wrong relaxation planted in the oracle must break parity."""
    c = G.load("mlp5_crown")
    orc = LirpaOracle(c["graph"], c["options"])
    orig = LirpaOracle._upper
    try:
        LirpaOracle._upper = staticmethod(lambda l, u: tuple(v * 1.001 for v in orig(l, u)))
        lb, ub = orc.compute_bounds(c["boxes"], c["method"])
    finally:
        LirpaOracle._upper = staticmethod(orig)
    assert G.excess(lb, c["lb"]) > 1.0 or G.excess(ub, c["ub"]) > 1.0


@pytest.mark.parametrize("name", [n for n in G.prop_names() if "mlp5" in n or "rand" in n])
def test_oracle_property_matches_luna(name):
    """The oracle's early stops on verified boxes (thresholds from a VNN-LIB
    property) against Luna's CLI flow on the same boxes."""
    from luna_b200.vnnlib import Property
    from oracle.lirpa_oracle import LirpaOracle
    c = G.load_prop(name)
    g = c["graph"]
    n_out = int(np.prod(g.nodes[g.output_index].out_shape))
    p = Property(c["text"], c["lower"].shape[1], n_out)
    C = p.C if p.has_spec else np.eye(n_out, dtype=np.float32)
    lb, ub, st = LirpaOracle(g, c["options"]).compute_property(c["lower"], c["upper"], C, p.thresholds, p.branches,
                                                                p.n_branches, c["method"])
    G.parity("oracle/" + name, lb, ub, c["lb"], c["ub"])
    if p.has_spec:
        assert st.tolist() == c["status"].tolist()


def test_concat_alpha_rounding_sensitivity():
    """Summation order alone moves concat_alpha beyond the bar: the oracle on
    the graph as Luna builds it meets the bar, the oracle on the same graph
    with the Concat of Linear nodes merged into one Linear (the same products
    summed in another order) does not; the engine is held to the second."""
    c = G.load("concat_alpha")
    as_luna = LirpaOracle(c["graph"], c["options"]).compute_bounds(c["boxes"], c["method"])
    merged = LirpaOracle(G.merged_concat_graph(c["graph"]), c["options"]).compute_bounds(c["boxes"], c["method"])
    assert max(G.excess(as_luna[0], c["lb"]), G.excess(as_luna[1], c["ub"])) <= 1.0
    assert max(G.excess(merged[0], c["lb"]), G.excess(merged[1], c["ub"])) > 1.0
    # The CROWN bounds of the same graph are insensitive.
    cc = G.load("concat_crown")
    m = LirpaOracle(G.merged_concat_graph(cc["graph"]), cc["options"]).compute_bounds(cc["boxes"], cc["method"])
    assert max(G.excess(m[0], cc["lb"]), G.excess(m[1], cc["ub"])) <= 1.0


def test_luna_thread_count_spread_on_cfg2():
    """Luna's own alpha-CROWN result on some of the 512 MLP boxes moves by
    more than the strict bar between 1 and 4 ATen threads (the golden uses 1):
    20 Adam steps amplify a last-bit difference in a gradient sum.  This is
    the measured reason why cfg2_alpha512 cannot be held to the strict bar
    box by box."""
    from oracle import luna_ref
    if not luna_ref.available():
        pytest.skip("oracle/_ref is not built (make -C oracle)")
    c = G.load("cfg2_alpha512")
    spread = {}
    for b in (429, 251):
        sub = c["boxes"].slice(b, b + 1)
        one = luna_ref.compute_bounds(c["graph"], sub, c["method"], c["options"], num_threads=1)
        four = luna_ref.compute_bounds(c["graph"], sub, c["method"], c["options"], num_threads=4)
        assert np.array_equal(one[0], c["lb"][b:b + 1]) and np.array_equal(one[1], c["ub"][b:b + 1])
        spread[b] = max(G.excess(four[0], one[0]), G.excess(four[1], one[1]))
    assert spread[429] > 5.0, spread   # 9.1 measured
    assert spread[251] <= 1.0, spread  # most boxes do not move
