"""Bounding boxes against VNN-LIB properties on the GPU, against Luna.

Luna's CLI flow (the property read by Luna's parser, its thresholds kept on
the model so STOP_CROWN_ON_VERIFIED / STOP_ALPHA_ON_VERIFIED apply, then the
verdict) produced the golden fixtures tests/golden/prop_*.npz
(make_property_golden.py).  Their thresholds put some boxes past the
threshold after the initial CROWN pass, some part-way through the alpha
optimisation and some never, so the bounds below check where each box
stopped.  Every call goes through the C ABI (lb200_compute_property and
lb200_property_status_device)."""
import ctypes as C

import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi
from luna_b200.engine import Model, _check, load_library
from luna_b200.vnnlib import Property

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


@pytest.mark.parametrize("name", G.prop_names())
def test_property_matches_luna(name):
    c = G.load_prop(name)
    g = c["graph"]
    n_out = int(np.prod(g.nodes[g.output_index].out_shape))
    prop = Property(c["text"], c["lower"].shape[1], n_out)
    m = Model(g, options=c["options"])
    lb, ub, status = m.compute_property(prop, c["method"], c["lower"], c["upper"])
    assert m.last_stats.kernel_launches > 0
    print(f"{name}: alpha iterations run {m.last_stats.alpha_iterations_run}")
    G.parity(name, lb, ub, c["lb"], c["ub"])
    assert status.tolist() == c["status"].tolist()
    assert (prop.status(lb, ub) == status).all()


def test_property_own_box():
    """With no boxes given, the property's own input box is bounded."""
    c = G.load_prop("prop_mlp5_or_crown")
    g = c["graph"]
    lo, hi = c["lower"][3], c["upper"][3]
    text = c["text"] + "".join(f"(assert (>= X_{k} {float(v):.9g}))\n(assert (<= X_{k} {float(w):.9g}))\n"
                               for k, (v, w) in enumerate(zip(lo, hi)))
    prop = Property(text, len(lo), 5)
    assert (prop.lower == lo).all() and (prop.upper == hi).all()
    m = Model(g, options=c["options"])
    lb, ub, status = m.compute_property(prop, c["method"])
    assert G.excess(lb[0], c["lb"][3]) <= 1.0 and G.excess(ub[0], c["ub"][3]) <= 1.0
    assert status[0] == c["status"][3]


def test_thresholds_through_compute_bounds():
    """lb200_compute_bounds with thresholds (a conjunction) stops boxes as
    lb200_compute_property does for the same property."""
    c = G.load_prop("prop_mlp5_conj_alpha")
    prop = Property(c["text"], c["lower"].shape[1], 5)
    from luna_b200.workloads import Boxes
    m = Model(c["graph"], options=c["options"])
    lb, ub = m.compute_bounds(Boxes(c["lower"], c["upper"], prop.C[None]), c["method"], thresholds=prop.thresholds)
    G.parity("thresholds via compute_bounds", lb, ub, c["lb"], c["ub"])


def test_status_device_matches_host():
    rng = np.random.default_rng(3)
    lib = load_library()
    seen = set()
    for nspec, nb in ((4, 0), (6, 3), (1, 0), (9, 9), (2, 1)):
        B = 5000
        thr = rng.normal(size=nspec).astype(np.float32)
        lb = (thr + rng.normal(size=(B, nspec)) - 1.0).astype(np.float32)
        ub = (lb + 2 * np.abs(rng.normal(size=(B, nspec)))).astype(np.float32)
        lb[rng.random(lb.shape) < 0.02] = np.nan
        ub[rng.random(ub.shape) < 0.02] = np.nan
        br = rng.integers(0, max(nb, 1), nspec).astype(np.int32)
        host = np.zeros(B, np.int32)
        ip = C.POINTER(C.c_int32)
        fp = C.POINTER(C.c_float)
        _check(lib.lb200_property_status(lb.ctypes.data_as(fp), ub.ctypes.data_as(fp), B, nspec,
                                         thr.ctypes.data_as(fp), br.ctypes.data_as(ip), nb, host.ctypes.data_as(ip)),
               "status")
        t = {k: torch.from_numpy(v).cuda() for k, v in dict(lb=lb, ub=ub, thr=thr, br=br).items()}
        dev = torch.zeros(B, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        _check(lib.lb200_property_status_device(t["lb"].data_ptr(), t["ub"].data_ptr(), B, nspec, t["thr"].data_ptr(),
                                                t["br"].data_ptr(), nb, dev.data_ptr(), stream), "status_device")
        torch.cuda.synchronize()
        assert (dev.cpu().numpy() == host).all()
        seen |= set(host.tolist())
    assert seen == {abi.STATUS_UNKNOWN, abi.STATUS_UNSAT, abi.STATUS_SAT}


def test_verdicts_sound_by_sampling():
    """Verdicts hold on sampled points: in a box called UNSAT no point is a
    counterexample, in a box called SAT every point is one, and every sampled
    margin lies within the box's bounds."""
    from luna_b200 import workloads as W
    g, split, text = W.mlp_property_split()
    bx = split.boxes(0, 64)
    t = int(np.argmax(split.C[0].sum(0)))  # the label: its column is +1 in every row
    # The same box with the label's worst rival as the label: SAT.
    y0 = W.graph_forward(g, torch.from_numpy(split.centre[None])).detach().numpy()[0]
    worst = int(np.argmin(y0))
    text_sat = W.robustness_property(split.lower, split.upper, worst, 10)
    m = Model(g, options=abi.default_options(alpha_lr=0.1, alpha_iterations=20))
    rng = np.random.default_rng(0)
    seen = set()
    for txt, label in ((text, t), (text_sat, worst)):
        prop = Property(txt, 784, 10)
        lb, ub, status = m.compute_property(prop, abi.METHOD_ALPHA_CROWN, bx.lower, bx.upper)
        for b in range(0, 64, 4):
            u = rng.random((4000, 784), dtype=np.float32)
            x = bx.lower[b] + u * (bx.upper[b] - bx.lower[b])
            y = W.graph_forward(g, torch.from_numpy(x)).detach().numpy()
            margins = (y @ prop.C.T).astype(np.float64)   # rows Y_label - Y_j
            assert (margins >= lb[b] - 1e-4).all() and (margins <= ub[b] + 1e-4).all()
            counterexample = (margins <= prop.thresholds).any(axis=1)   # OR of single-row branches
            if status[b] == abi.STATUS_UNSAT:
                assert not counterexample.any()
            elif status[b] == abi.STATUS_SAT:
                assert counterexample.all()
            seen.add(int(status[b]))
    assert {abi.STATUS_UNSAT, abi.STATUS_SAT} <= seen


def test_property_device_entry_matches_host_entry():
    """lb200_compute_property_device on device buffers gives the host entry's
    bounds and verdicts bit for bit."""
    c = G.load_prop("prop_mlp5_or_alpha")
    prop = Property(c["text"], c["lower"].shape[1], 5)
    m = Model(c["graph"], options=c["options"])
    lb, ub, status = m.compute_property(prop, c["method"], c["lower"], c["upper"])
    B = lb.shape[0]
    xl = torch.from_numpy(c["lower"]).cuda()
    xu = torch.from_numpy(c["upper"]).cuda()
    dlb = torch.empty((B, prop.nspec), device="cuda")
    dub = torch.empty_like(dlb)
    dst = torch.empty(B, dtype=torch.int32, device="cuda")
    m.compute_property_ptr(prop, c["method"], xl.data_ptr(), xu.data_ptr(), B, dlb.data_ptr(), dub.data_ptr(),
                           dst.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dlb.cpu().numpy(), lb) and np.array_equal(dub.cpu().numpy(), ub)
    assert np.array_equal(dst.cpu().numpy(), status)


@pytest.mark.parametrize("seed", range(4))
def test_property_matches_oracle_random(seed):
    """Random MLPs and boxes, a margin property per seed (a conjunction for
    even seeds, an OR for odd ones) with thresholds halfway between
    neighbouring boxes' alpha-CROWN margins: the engine's early-stopped
    bounds and verdicts against the CPU oracle's."""
    from luna_b200 import workloads as W
    from luna_b200.workloads import Boxes
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.random_mlp_case(700 + seed, n_boxes=8, depth=2 + seed % 3, width=16)
    n_in, n_out = bx.lower.shape[1], 4
    rows = [j for j in range(1, n_out)]
    C = np.zeros((len(rows), n_out), np.float32)
    for r, j in enumerate(rows):
        C[r, 0], C[r, j] = 1, -1
    opt = abi.default_options(alpha_lr=0.3, alpha_iterations=10)
    ora = LirpaOracle(g, opt)
    lA, _ = ora.compute_bounds(Boxes(bx.lower, bx.upper, C[None]), abi.METHOD_ALPHA_CROWN)
    srt = np.sort(lA, axis=0)
    thr = (0.5 * (srt[3] + srt[4])).astype(np.float32)
    cmps = [f"(<= (- Y_0 Y_{j}) {float(t):.9g})" for j, t in zip(rows, thr)]
    text = "\n".join(f"(assert {c})" for c in cmps) if seed % 2 == 0 else \
        "(assert (or " + " ".join(f"(and {c})" for c in cmps) + "))"
    prop = Property(text, n_in, n_out)
    assert prop.nspec == len(rows) and (prop.n_branches > 0) == (seed % 2 == 1)
    olb, oub, ost = ora.compute_property(bx.lower, bx.upper, prop.C, prop.thresholds, prop.branches,
                                         prop.n_branches, abi.METHOD_ALPHA_CROWN)
    lb, ub, st = Model(g, options=opt).compute_property(prop, abi.METHOD_ALPHA_CROWN, bx.lower, bx.upper)
    G.parity(f"random property {seed}", lb, ub, olb, oub)
    assert st.tolist() == ost.tolist()
