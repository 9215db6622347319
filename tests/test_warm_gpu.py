"""Warm start (lb200_set_warm_start / lb200_set_warm_parents / lb200_warm_alpha)
against Luna's own: a parent box bounded with alpha-CROWN, TorchModel::getState
taken and loaded into the model with a child box (TorchModel::loadState), and
the child bounded with alpha-CROWN (tests/golden/make_warm_golden.py).  Every
call goes through the C ABI."""
import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi
from luna_b200.engine import Model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def _warm(c, parents, path=0):
    """The children of case c bounded after their parents, box b seeded from
    parent parents[b]; returns (lb, ub) and the model."""
    m = Model(c["graph"], options=c["options"])
    m.set_contraction_path(path)
    m.set_warm_start(True)
    m.compute_bounds(c["parents"], abi.METHOD_ALPHA_CROWN)
    m.set_warm_parents(parents)
    lb, ub = m.compute_bounds(c["children"], abi.METHOD_ALPHA_CROWN)
    return lb, ub, m


@pytest.mark.parametrize("path", [0, 1])
@pytest.mark.parametrize("name", G.warm_names())
def test_warm_start_matches_luna(name, path):
    c = G.load_warm(name)
    B = c["children"].n
    lb, ub, _ = _warm(c, np.arange(B), path)
    G.parity("warm/" + name + ("/simt" if path == 1 else ""), lb, ub, c["lb"], c["ub"])
    # The state matters: Luna's warm bounds are not its fresh ones.
    assert not (np.array_equal(c["lb"], c["fresh_lb"]) and np.array_equal(c["ub"], c["fresh_ub"]))


@pytest.mark.parametrize("path", [0, 1])
@pytest.mark.parametrize("name", G.warm_names("warm_conv"))
def test_warm_start_with_convolutions_matches_luna(name, path):
    """Warm start on networks with convolutions: dense conv starts, a patches
    start (window rows), a strided transposed conv."""
    c = G.load_warm(name, "warm_conv")
    lb, ub, _ = _warm(c, np.arange(c["children"].n), path)
    G.parity("warm/" + name + ("/simt" if path == 1 else ""), lb, ub, c["lb"], c["ub"])


def _oracle_seed(oracle, graph, model, box):
    """The engine's retained alphas of one box (lb200_warm_alpha) as the
    oracle's seed: keyed by (ReLU node, start node), compacted to the
    creation set as Luna stores them."""
    from oracle.lirpa_oracle import _Alpha
    pre = oracle.preact_ids
    K = len(pre) + 1
    relus = [i for i, nd in enumerate(graph.nodes) if nd.type == abi.NODE_RELU]
    seed = {}
    for st in range(2, K + 1):
        start_node = pre[st - 1] if st < K else graph.output_index
        for m in range(1, st):
            a, aset = model.warm_alpha(m, st, box)
            idx = np.nonzero(aset)[0]
            seed[(relus[m - 1], start_node)] = _Alpha(torch.from_numpy(np.ascontiguousarray(a[:, :, idx])),
                                                      torch.from_numpy(idx.astype(np.int64)))
    return seed


@pytest.mark.parametrize("path,child_iters", [(0, None), (1, None), (0, 3)])
@pytest.mark.parametrize("name", G.warm_names())
def test_warm_start_pinned_by_oracle_from_engine_state(name, path, child_iters):
    """The warm start itself, free of the parent's rounding: the oracle's
    child run started from the engine's own retained alphas (the state
    lb200_warm_alpha reads back) must give the engine's child bounds.  With
    child_iters the children take that many Adam steps instead (the parents
    keep the case's count), which bounds how far the tensor-core rounding of
    the child's own steps can grow."""
    from oracle.lirpa_oracle import LirpaOracle
    c = G.load_warm(name)
    B = c["children"].n
    m = Model(c["graph"], options=c["options"])
    m.set_contraction_path(path)
    m.set_warm_start(True)
    m.compute_bounds(c["parents"], abi.METHOD_ALPHA_CROWN)
    o = LirpaOracle(c["graph"], c["options"])
    seeds = [_oracle_seed(o, c["graph"], m, b) for b in range(B)]
    child_opt = c["options"]
    if child_iters is not None:
        child_opt = abi.default_options(**{**{f: getattr(c["options"], f) for f, _ in c["options"]._fields_},
                                           "alpha_iterations": child_iters})
        m.set_options(child_opt)
    m.set_warm_parents(np.arange(B))
    lb, ub = m.compute_bounds(c["children"], abi.METHOD_ALPHA_CROWN)
    ch = c["children"]
    olb = np.zeros_like(lb)
    oub = np.zeros_like(ub)
    n = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        for b in range(B):
            C = torch.from_numpy(ch.C[0 if ch.C.shape[0] == 1 else b].copy())
            lo, hi, _ = LirpaOracle(c["graph"], child_opt).alpha_crown(
                torch.from_numpy(ch.lower[b].copy()), torch.from_numpy(ch.upper[b].copy()), C, seed=seeds[b])
            olb[b], oub[b] = lo.numpy(), hi.numpy()
    finally:
        torch.set_num_threads(n)
    tag = "warm-pinned/" + name + ("/simt" if path == 1 else "") + (f"/{child_iters}it" if child_iters else "")
    G.parity(tag, lb, ub, olb, oub)


def test_unseeded_boxes_are_bounded_afresh():
    """parent -1 bounds a box as a call without warm start does, bit for bit;
    the seeded boxes of the same call still take their parents' state."""
    c = G.load_warm("mlp5_warm")
    B = c["children"].n
    parents = np.where(np.arange(B) % 2 == 0, -1, np.arange(B))
    lb, ub, _ = _warm(c, parents)
    m = Model(c["graph"], options=c["options"])
    flb, fub = m.compute_bounds(c["children"], abi.METHOD_ALPHA_CROWN)
    even = np.arange(B) % 2 == 0
    assert np.array_equal(lb[even], flb[even]) and np.array_equal(ub[even], fub[even])
    G.parity("warm/mlp5_warm/odd", lb[~even], ub[~even], c["lb"][~even], c["ub"][~even])


def test_warm_start_rejections():
    c = G.load_warm("mlp5_warm")
    B = c["children"].n
    m = Model(c["graph"], options=c["options"])
    with pytest.raises(RuntimeError, match="no retained state"):
        m.set_warm_parents(np.arange(B))
    m.set_warm_start(True)
    m.compute_bounds(c["parents"], abi.METHOD_ALPHA_CROWN)
    with pytest.raises(RuntimeError, match="out of range"):
        m.set_warm_parents(np.full(B, B))
    with pytest.raises(RuntimeError, match="bad level or start"):
        m.warm_alpha(2, 2, 0)
    m.set_warm_parents(np.arange(B - 1))
    with pytest.raises(RuntimeError, match="one parent index per box"):
        m.compute_bounds(c["children"], abi.METHOD_ALPHA_CROWN)
    m.set_warm_parents(np.arange(B))
    with pytest.raises(RuntimeError, match="alpha-CROWN calls only"):
        m.compute_bounds(c["children"], abi.METHOD_CROWN)
    # The parents applied to one call only: the next call is a fresh one.
    lb, ub = m.compute_bounds(c["children"], abi.METHOD_ALPHA_CROWN)
    G.parity("warm/mlp5_warm/fresh", lb, ub, c["fresh_lb"], c["fresh_ub"])
    m.set_warm_start(False)
    with pytest.raises(RuntimeError, match="no retained state"):
        m.set_warm_parents(np.arange(B))



def test_warm_start_chain_matches_oracle_and_is_sound():
    """Three levels of a split tree (as Luna's own repeated loadState / run /
    getState test does, tests/unit/analysis/test_bab_state.cpp): 6 boxes,
    then both halves of each (12 children, shuffled, so parent indices are
    not the identity and every parent has two children), then one half of
    each child (parents in reverse order).  Each level is seeded from the
    one before; its bounds match the oracle's chain of seeded runs and hold
    at sampled points."""
    from luna_b200 import workloads as W
    from oracle.lirpa_oracle import LirpaOracle
    g, opt, (L0, L1, L2), (p1, p2) = G.split_chain()
    m = Model(g, options=opt)
    m.set_contraction_path(1)
    m.set_warm_start(True)
    m.compute_bounds(L0, abi.METHOD_ALPHA_CROWN)
    m.set_warm_parents(p1)
    lb1, ub1 = m.compute_bounds(L1, abi.METHOD_ALPHA_CROWN)
    m.set_warm_parents(p2)
    lb2, ub2 = m.compute_bounds(L2, abi.METHOD_ALPHA_CROWN)

    def run(o, bx, b, seed=None):
        C = torch.from_numpy(bx.C[0 if bx.C.shape[0] == 1 else b].copy())
        lo, hi, _ = o.alpha_crown(torch.from_numpy(bx.lower[b].copy()), torch.from_numpy(bx.upper[b].copy()), C,
                                  seed=seed)
        return lo.numpy(), hi.numpy(), o.last_alphas

    n = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        o = LirpaOracle(g, opt)
        s0 = [run(o, L0, b)[2] for b in range(6)]
        r1 = [run(o, L1, j, s0[p1[j]]) for j in range(12)]
        r2 = [run(o, L2, k, r1[p2[k]][2]) for k in range(12)]
    finally:
        torch.set_num_threads(n)
    G.parity("warm chain/level 1", lb1, ub1, np.stack([r[0] for r in r1]), np.stack([r[1] for r in r1]))
    G.parity("warm chain/level 2", lb2, ub2, np.stack([r[0] for r in r2]), np.stack([r[1] for r in r2]))
    for bx, lb, ub in ((L1, lb1, ub1), (L2, lb2, ub2)):
        t = np.random.default_rng(5).random((bx.n, 2000, bx.lower.shape[1]), dtype=np.float32)
        x = bx.lower[:, None] + t * (bx.upper - bx.lower)[:, None]
        y = W.graph_forward(g, torch.from_numpy(x.reshape(-1, x.shape[-1]))).numpy().reshape(bx.n, 2000, -1)
        C = np.broadcast_to(bx.C, (bx.n,) + bx.C.shape[1:])
        cy = np.einsum("bsn,bpn->bps", C, y)
        tol = 1e-4 * (1 + np.abs(lb).max())
        assert (cy >= lb[:, None] - tol).all() and (cy <= ub[:, None] + tol).all()
