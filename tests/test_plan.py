"""The engine's host-side plan (lb200_describe_plan, no GPU): graph analysis,
concretisation forms against the oracle's reading of Luna's rules, row
windows against the support of the oracle's dense rows, and rejections."""
import copy

import numpy as np
import pytest
import torch

from luna_b200 import abi, workloads as W
from luna_b200.abi import Graph, Node
from luna_b200.engine import EngineError, describe_plan
from oracle.lirpa_oracle import LirpaOracle, _BoxState

CASES = {
    "cnn_dense": lambda: W.small_cnn_case(3, n_boxes=1, big_first=False),
    "cnn_patch": lambda: W.small_cnn_case(5, n_boxes=1, big_first=True),
    "cnnbn_patch": lambda: W.small_cnn_bn_case(6, n_boxes=1, big_first=True),
    "convt": lambda: W.convt_cnn_case(1, n_boxes=1, conv_after=True),
    "resnet": lambda: W.small_resnet_case(7, n_boxes=1),
    "resnet_big": lambda: W.small_resnet_case(8, n_boxes=1, big=True),
    "sigmoid": lambda: W.sigmoid_mlp_case(0, n_boxes=1),
    "cnn_cifar": lambda: W.cnn_cifar(1),
    "resnet_cifar": lambda: W.resnet_cifar(1),
}


def _oracle_state(g, bx):
    o = LirpaOracle(g, abi.default_options())
    st = _BoxState()
    x = (torch.from_numpy(bx.lower[0]), torch.from_numpy(bx.upper[0]))
    with torch.no_grad():
        o._compute_ibp(st, x)
    return o, st, x


@pytest.mark.parametrize("name", sorted(CASES))
def test_forms_match_the_oracle(name):
    """Per backward start, the engine concretises in the form (patches or
    dense) that Luna's CPU path ends with at the input."""
    g, bx = CASES[name]()
    plan = describe_plan(g)
    o, st, x = _oracle_state(g, bx)
    nodes = {lv["level"]: lv["node"] for lv in plan["levels"]}
    for s in plan["starts"]:
        node = nodes[s["level"]]
        if node < 0:  # the output start: the specification matrix, a dense start
            assert s["form"] == "dense"
            continue
        with torch.no_grad():
            patches = o._backward_from(st, node, x, rows=[0])[4]
        assert s["form"] == ("patches" if patches else "dense"), (name, s["level"])


@pytest.mark.parametrize("name", ["cnn_patch", "cnnbn_patch", "resnet", "resnet_big"])
def test_windows_cover_the_dense_rows(name):
    """For window starts, every nonzero of the oracle's dense row at the input
    lies inside the engine's input window of that row."""
    g, bx = CASES[name]()
    plan = describe_plan(g)
    o, st, x = _oracle_state(g, bx)
    levels = {lv["level"]: lv for lv in plan["levels"]}
    C0, H0, W0 = levels[0]["map"]
    rng = np.random.default_rng(0)
    checked = 0
    for s in plan["starts"]:
        lv = levels[s["level"]]
        wh, ww, mul, off, full = s["windows"][0]
        if full or lv["node"] < 0:
            continue
        C, H, Wd = lv["map"]
        for neuron in rng.choice(C * H * Wd, 4, replace=False):
            y, xx = (neuron % (H * Wd)) // Wd, neuron % Wd
            with torch.no_grad():
                A = o._backward_from(st, lv["node"], x, rows=[int(neuron)])[0].reshape(C0, H0, W0)
            ys, xs = np.nonzero(A.abs().sum(0).numpy())
            oy, ox = mul * y + off, mul * xx + off
            assert ((ys >= oy) & (ys < oy + wh) & (xs >= ox) & (xs < ox + ww)).all(), (name, s["level"], neuron)
            checked += 1
    assert checked > 0


def _mlp_graph():
    g, _ = W.sigmoid_mlp_case(0, n_boxes=1)
    return g


def _expect_rejected(g, text):
    with pytest.raises(EngineError, match=text):
        describe_plan(g)


def test_rejections():
    g, _ = W.small_resnet_case(0, n_boxes=1)
    # An Add with one (constant) operand.
    bad = copy.deepcopy(g)
    add = next(i for i, n in enumerate(bad.nodes) if n.type == abi.NODE_ADD)
    bad.nodes[add].inputs = bad.nodes[add].inputs[:1]
    _expect_rejected(bad, "constant operand")
    # A skip edge from the level just below the Add.
    bad = copy.deepcopy(g)
    conv2 = bad.nodes[bad.nodes[add].inputs[0]].inputs[0]  # the Add's main operand is BatchNorm(conv2)
    relu_h = bad.nodes[conv2].inputs[0]  # conv2's input: the block's inner ReLU
    assert bad.nodes[relu_h].type == abi.NODE_RELU
    bad.nodes[add].inputs[1] = relu_h
    _expect_rejected(bad, "skip edge")
    # A Sigmoid on a conv map.
    bad = copy.deepcopy(g)
    first_relu = next(i for i, n in enumerate(bad.nodes) if n.type == abi.NODE_RELU)
    bad.nodes[first_relu].type = abi.NODE_SIGMOID
    _expect_rejected(bad, "Sigmoid")
    # The output must be a Linear.
    nodes = [Node(abi.NODE_INPUT, [], (4, 1, 1)),
             Node(abi.NODE_LINEAR, [0], (3, 1, 1), weight=np.ones((3, 4), np.float32),
                  bias=np.zeros(3, np.float32)),
             Node(abi.NODE_RELU, [1], (3, 1, 1))]
    _expect_rejected(Graph(nodes, 0, 2), "output node")
    # A node kind the engine does not take.
    bad = copy.deepcopy(_mlp_graph())
    bad.nodes[2].type = abi.NODE_CONSTANT
    _expect_rejected(bad, "not supported")


def test_rejections_of_sub_slice_concat_reshape():
    """Placements of the rewritten node kinds with no exact rewrite are
    refused with a message naming the node."""
    g, _ = W.sub_mlp_case(1)
    bad = copy.deepcopy(g)
    bad.nodes[1].inputs = [0, 0]  # Sub of two tensors
    _expect_rejected(bad, "two tensors")
    bad = copy.deepcopy(g)
    bad.nodes[1].constant = None
    _expect_rejected(bad, "without a constant")
    g, _ = W.sub_cnn_case(9)
    bad = copy.deepcopy(g)
    conv = 2
    relu = 3
    # A Sub after a conv whose constant varies inside a channel.
    bad.nodes.append(Node(abi.NODE_SUB, [conv], bad.nodes[conv].out_shape,
                          constant=np.arange(bad.nodes[conv].size, dtype=np.float32)))
    bad.nodes[relu].inputs = [len(bad.nodes) - 1]
    _expect_rejected(bad, "producers must precede|uniform")
    g, _ = W.slice_mlp_case(5)
    bad = copy.deepcopy(g)
    bad.nodes[2].step = 2
    _expect_rejected(bad, "steps")
    bad = copy.deepcopy(g)
    bad.nodes[2].axis = 2
    _expect_rejected(bad, "features of a flat vector")
    g, _ = W.concat_mlp_case(7)
    bad = copy.deepcopy(g)
    bad.nodes[2].inputs = [1]  # operands of different producers
    _expect_rejected(bad, "one producer")
    g, _ = W.concat_cnn_case(8)
    bad = copy.deepcopy(g)
    reshape = next(i for i, n in enumerate(bad.nodes) if n.type == abi.NODE_RESHAPE)
    bad.nodes[reshape].out_shape = (6, 4, 4)
    _expect_rejected(bad, "Reshape")


@pytest.mark.parametrize("gen,kw,pre", [
    ("sub_mlp_case", {"seed": 1}, [2, 4]),
    ("sub_mlp_case", {"seed": 3, "where": "linear"}, [2, 4]),
    ("slice_mlp_case", {"seed": 5}, [2, 4]),
    ("concat_mlp_case", {"seed": 7}, [3, 5]),
    ("concat_cnn_case", {"seed": 8}, [3, 5, 8]),
    ("sub_cnn_case", {"seed": 9}, [2, 4, 7]),
])
def test_rewritten_kinds_keep_luna_node_ids(gen, kw, pre):
    """Sub / Slice / Concat / Reshape graphs are taken, and the pre-activation
    of every level keeps the id of the node that feeds its ReLU in Luna's
    graph (the key of intermediate bounds)."""
    g, _ = getattr(W, gen)(**kw)
    plan = describe_plan(g)
    nodes = [lv["node"] for lv in plan["levels"]][1:-1]
    assert nodes == pre == g.activation_inputs()


def test_plan_levels_of_the_cifar_resnet():
    plan = describe_plan(W.resnet_cifar(1)[0])
    acts = [lv["act"] for lv in plan["levels"]]
    assert acts == ["", "relu"] + ["relu"] * 8 + ["sigmoid", ""]
    skips = {lv["level"]: lv["skips"] for lv in plan["levels"] if lv.get("skips")}
    assert skips == {3: [{"src": 1, "conv": False}], 5: [{"src": 3, "conv": False}],
                     7: [{"src": 5, "conv": True}], 9: [{"src": 7, "conv": False}]}
