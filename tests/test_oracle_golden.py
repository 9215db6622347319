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
# first boxes only (the GPU suite checks the engine on all of them).  The
# CIFAR CNN's 30-iteration alpha-CROWN takes the oracle's autograd loop over
# dense A matrices about an hour per box, so that golden pins the engine
# alone (and Luna pins itself: it is Luna's output).
ORACLE_BOXES = {"cfg2_alpha512": 48, "cfg3_alpha": 0}


def _oracle_case(name):
    """The oracle's bounds for one golden case (run in a pool worker): one
    ATen thread, as the goldens were made, or several for large conv maps."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import golden_cases as GC
    from oracle.lirpa_oracle import LirpaOracle as Oracle
    c = GC.load(name)
    if ORACLE_BOXES.get(name, 1) == 0:
        return None
    torch.set_num_threads(min(4, os.cpu_count() or 1) if c["boxes"].lower.shape[1] >= 1000 else 1)
    n = ORACLE_BOXES.get(name, c["boxes"].n)
    res = Oracle(c["graph"], c["options"]).compute_bounds(c["boxes"].slice(0, n), c["method"],
                                                          intermediate="inter_lb" in c)
    return tuple(np.asarray(r) for r in res)


@pytest.fixture(scope="module")
def oracle_results():
    """Every golden case through the oracle, spread over the host's cores
    (spawned worker processes; each case's arithmetic is unchanged)."""
    import multiprocessing as mp
    names = G.names()
    procs = max(1, min(8, (os.cpu_count() or 1)))
    with mp.get_context("spawn").Pool(procs) as pool:
        res = pool.map(_oracle_case, names, chunksize=1)
    return dict(zip(names, res))


@pytest.mark.parametrize("name", G.names())
def test_oracle_matches_luna(name, oracle_results):
    c = G.load(name)
    n = ORACLE_BOXES.get(name, c["boxes"].n)
    if n == 0:
        pytest.skip("no oracle run at this size (the engine is checked against this golden on the GPU)")
    res = oracle_results[name]
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


@pytest.mark.parametrize("sub,name", [("warm", n) for n in G.warm_names()] +
                         [("warm_conv", n) for n in G.warm_names("warm_conv")])
def test_oracle_warm_start_matches_luna(sub, name):
    """The oracle's warm start (a child bounded from its parent's alphas,
    TorchModel::getState / loadState) against Luna's own on the same parent
    and child boxes, on MLPs and on networks with convolutions (dense and
    patches starts, a transposed conv).  Luna's warm bounds differ from its
    fresh ones on these cases, so a warm start that ignored the state would
    fail here."""
    c = G.load_warm(name, sub)
    lb, ub = LirpaOracle(c["graph"], c["options"]).compute_bounds_warm(c["parents"], c["children"])
    G.parity("oracle/warm/" + name, lb, ub, c["lb"], c["ub"])
    assert not (np.array_equal(c["lb"], c["fresh_lb"]) and np.array_equal(c["ub"], c["fresh_ub"]))


def test_oracle_warm_chain_matches_luna():
    """Two warm starts in a row (root, level-1 box, level-2 box), as Luna's
    repeated getState / loadState / compute_bounds: the oracle's chain of
    seeded runs against Luna's on the paths whose level-1 run reuses every
    seeded alpha (tests/golden/warm_chain/split3.npz)."""
    c = G.load_chain()
    L0, L1, L2 = c["levels"]
    p1, p2 = c["parents"]
    o = LirpaOracle(c["graph"], c["options"])

    def run(bx, b, seed=None):
        C = torch.from_numpy(bx.C[0 if bx.C.shape[0] == 1 else b].copy())
        lo, hi, _ = o.alpha_crown(torch.from_numpy(bx.lower[b].copy()), torch.from_numpy(bx.upper[b].copy()), C,
                                  seed=seed)
        return lo.numpy(), hi.numpy(), o.last_alphas

    out = []
    for k in c["leaves"]:
        s0 = run(L0, p1[p2[k]])[2]
        r1 = run(L1, p2[k], s0)
        r2 = run(L2, k, r1[2])
        out.append((r1[0], r1[1], r2[0], r2[1]))
    lb1, ub1, lb2, ub2 = (np.stack([r[i] for r in out]) for i in range(4))
    G.parity("oracle/warm chain/level 1", lb1, ub1, c["lb1"], c["ub1"])
    G.parity("oracle/warm chain/level 2", lb2, ub2, c["lb2"], c["ub2"])


@pytest.mark.parametrize("name", G.nostab_names())
def test_oracle_matches_luna_without_stabilised_bounds(name):
    """STABILIZE_INTERMEDIATE_BOUNDS off: no straight-through clamp of the
    intermediate bounds, so a layer stable when its alphas were created can
    turn unstable during the optimisation (box 2 here); the oracle follows
    Luna through it."""
    c = G.load(name, "nostab")
    lb, ub = LirpaOracle(c["graph"], c["options"]).compute_bounds(c["boxes"], c["method"])
    G.parity("oracle/nostab/" + name, lb, ub, c["lb"], c["ub"])


@pytest.mark.parametrize("name", G.option_names())
def test_oracle_matches_luna_at_non_default_options(name):
    """Early-stop patience that ends runs early, the best-alpha save window
    moved both ways, a faster learning-rate decay, CROWN with the first
    Linear layer back-substituted, and a large first conv concretised
    densely (tests/golden/options/)."""
    c = G.load(name, "options")
    lb, ub = LirpaOracle(c["graph"], c["options"]).compute_bounds(c["boxes"], c["method"])
    G.parity("oracle/options/" + name, lb, ub, c["lb"], c["ub"])
