"""Parity of the CUDA engine with Luna (golden fixtures) and with the CPU
oracle, plus soundness by sampling.  Every call goes through the C ABI."""
import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.engine import Model

pytestmark = pytest.mark.gpu

# The sampled network outputs the bounds are checked against are computed
# with torch on the GPU: in full fp32, not with TF32 convolutions / matmuls.
torch.backends.cudnn.allow_tf32 = False
torch.backends.cuda.matmul.allow_tf32 = False


@pytest.fixture(scope="module", autouse=True)
def _built():
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


@pytest.mark.parametrize("name", G.names())
def test_engine_matches_luna(name):
    c = G.load(name)
    m = Model(c["graph"], options=c["options"])
    lb, ub = m.compute_bounds(c["boxes"], c["method"])
    assert m.last_stats.kernel_launches > 0
    if name in G.ROUNDING_SENSITIVE:
        from oracle.lirpa_oracle import LirpaOracle
        olb, oub = LirpaOracle(G.merged_concat_graph(c["graph"]), c["options"]).compute_bounds(c["boxes"],
                                                                                               c["method"])
        _assert_parity(name + " (vs oracle on the merged graph)", lb, ub, olb, oub)
        return
    _assert_parity(name, lb, ub, c["lb"], c["ub"])
    if "inter_lb" in c:
        lo, hi = m.intermediate_bounds()
        B = c["boxes"].n
        e, states = G.check_intermediate(lo.reshape(B, -1), hi.reshape(B, -1), c["inter_lb"], c["inter_ub"])
        assert e <= 1.0 and states, e


def test_cfg2_simt_path_matches_luna_as_luna_matches_itself():
    """The 512-box MLP alpha-CROWN golden through the SIMT fp32 contractions:
    as many boxes beyond the strict bar as Luna's own result shows between
    1 and 4 ATen threads (the tensor-core path's larger count comes from its
    accumulation, not from the algorithm)."""
    c = G.load("cfg2_alpha512")
    m = Model(c["graph"], options=c["options"])
    m.set_contraction_path(1)
    lb, ub = m.compute_bounds(c["boxes"], c["method"])
    G.parity("cfg2_alpha512/simt", lb, ub, c["lb"], c["ub"])


@pytest.mark.parametrize("name", G.oracle_names())
def test_engine_matches_oracle_full_size(name):
    """Full-size networks of the ResNet and sweep workloads against the CPU
    oracle's committed results (tests/golden/make_oracle_golden.py)."""
    c = G.load(name)
    lb, ub = Model(c["graph"], options=c["options"]).compute_bounds(c["boxes"], c["method"])
    # The oracle, not Luna, is the reference here: both it and the engine are
    # held to the bar against Luna on these networks' smaller relatives, so
    # the two may differ by the sum of their allowances (twice the bar).
    e = max(G.excess(lb, c["lb"], 2 * G.RTOL, 2 * G.ATOL), G.excess(ub, c["ub"], 2 * G.RTOL, 2 * G.ATOL))
    es = max(G.excess_scaled(lb, c["lb"], c["lb"], c["ub"], 2 * G.RTOL, 2 * G.ATOL),
             G.excess_scaled(ub, c["ub"], c["lb"], c["ub"], 2 * G.RTOL, 2 * G.ATOL))
    print(f"PARITY {name} vs oracle (2x bar) {e:.4f}, strict {max(G.excess(lb, c['lb']), G.excess(ub, c['ub'])):.4f}"
          f", scaled (2x bar) {es:.4f}")
    if name in G.LOOSE:
        assert es <= 1.0, (e, es)
    else:
        assert e <= 1.0, e


def _assert_parity(name, lb, ub, ref_lb, ref_ub):
    """The strict bar (1e-5 rel / 1e-6 abs), except for the cases that
    golden_cases.LOOSE names with their reason."""
    G.parity(name, lb, ub, ref_lb, ref_ub)


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_engine_matches_oracle_random(seed, method):
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.random_mlp_case(500 + seed, n_boxes=6, depth=2 + seed % 3, width=16)
    opt = abi.default_options(alpha_lr=0.3, alpha_iterations=6)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"mlp{seed}/{method}", lb, ub, olb, oub)


@pytest.mark.parametrize("bn", [False, True])
@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_cnn_matches_oracle_random(seed, method, bn):
    """Random conv geometries (kernel 2-5, stride 1-2, padding 0-2), with and
    without BatchNorm after each conv, against the oracle."""
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.random_cnn_case(seed, bn=bn)
    opt = abi.default_options(alpha_lr=0.3, alpha_iterations=6)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"cnn{seed}/{method}/bn{int(bn)}", lb, ub, olb, oub)


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_tc_conv_matches_simt_and_oracle(method):
    """Strided 32/64-channel convs (tcgen05 implicit-GEMM steps, windows and
    whole maps) agree with the SIMT conv kernels and with the oracle."""
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.cnn_wide_case(21)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=6)
    m = Model(g, options=opt)
    tlb, tub = m.compute_bounds(bx, method)
    m.set_contraction_path(1)
    slb, sub = m.compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"simt vs oracle/{method}", slb, sub, olb, oub)
    # The tensor-core path is held to the bar against Luna itself on this
    # network (the cnnwide_* goldens).  Against the oracle, which is itself
    # within the bar of Luna, and against the SIMT path, the allowance is the
    # sum of the two: twice the bar.
    for what, rl, ru in (("oracle", olb, oub), ("simt", slb, sub)):
        e = max(G.excess(tlb, rl, 2 * G.RTOL, 2 * G.ATOL), G.excess(tub, ru, 2 * G.RTOL, 2 * G.ATOL))
        print(f"PARITY tc vs {what}/{method} (2x bar) {e:.4f}")
        assert e <= 1.0, (what, e)


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_tc_convt_matches_simt(method):
    """A 32 -> 32-channel transposed conv takes its back-substitution (a
    strided correlation read by element-strided TMA boxes) and its adjoint (a
    transposed conv, phases stacked in M) on tensor cores; against the SIMT
    kernels at twice the bar (each is held to the bar against Luna by the
    convttc_* goldens)."""
    g, bx = W.convt_cnn_case(11, n_boxes=3, tc=True)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=5)
    m = Model(g, options=opt)
    tlb, tub = m.compute_bounds(bx, method)
    m.set_contraction_path(1)
    slb, sub = m.compute_bounds(bx, method)
    e = max(G.excess(tlb, slb, 2 * G.RTOL, 2 * G.ATOL), G.excess(tub, sub, 2 * G.RTOL, 2 * G.ATOL))
    print(f"PARITY tc convT vs simt/{method} (2x bar) {e:.4f}")
    assert e <= 1.0, e


def _forward(graph, x):
    """Forward of a graph (any DAG of the supported nodes) on a batch of flat
    inputs in CHW order."""
    import torch.nn.functional as F
    from oracle.lirpa_oracle import topo_order
    f = lambda a: torch.from_numpy(a).cuda()
    val = {}
    for i in topo_order(graph)[0]:
        n = graph.nodes[i]
        ins = [val[p] for p in n.inputs]
        if n.type == abi.NODE_INPUT:
            y = x.reshape(x.shape[0], *n.out_shape)
        elif n.type == abi.NODE_LINEAR:
            y = ins[0].reshape(x.shape[0], -1) @ f(n.weight).T + f(n.bias)
        elif n.type == abi.NODE_CONV:
            y = F.conv2d(ins[0], f(n.weight), f(n.bias), stride=n.stride, padding=n.padding)
        elif n.type == abi.NODE_CONVTRANSPOSE:
            y = F.conv_transpose2d(ins[0], f(n.weight), f(n.bias), stride=n.stride, padding=n.padding)
        elif n.type == abi.NODE_BATCHNORM:
            w = f(n.weight) / torch.sqrt(f(n.running_var) + n.eps)
            b = f(n.bias) - f(n.running_mean) * w
            y = ins[0] * w.view(1, -1, 1, 1) + b.view(1, -1, 1, 1)
        elif n.type == abi.NODE_RELU:
            y = torch.relu(ins[0])
        elif n.type == abi.NODE_SIGMOID:
            y = torch.sigmoid(ins[0])
        elif n.type == abi.NODE_ADD:
            y = ins[0] + ins[1]
        elif n.type in (abi.NODE_FLATTEN, abi.NODE_IDENTITY):
            y = ins[0].reshape(x.shape[0], -1) if n.type == abi.NODE_FLATTEN else ins[0]
        else:
            raise NotImplementedError(n.type)
        val[i] = y
    return val[graph.output_index].reshape(x.shape[0], -1)


def _sample_outputs(graph, boxes, n_pts, seed=0, batch=20_000):
    """C . f(x) at n_pts uniform points (and the corners' mix) per box, on the GPU."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    lo = torch.from_numpy(boxes.lower).cuda()
    hi = torch.from_numpy(boxes.upper).cuda()
    Cm = torch.from_numpy(boxes.C).cuda()
    B = lo.shape[0]
    out = []
    for b in range(B):
        ys = []
        for i0 in range(0, n_pts, batch):
            k = min(batch, n_pts - i0)
            t = torch.rand((k, lo.shape[1]), generator=gen, device="cuda")
            if i0 == 0:
                t[: k // 10] = (t[: k // 10] > 0.5).float()  # vertices
            x = lo[b] + t * (hi[b] - lo[b])
            c = Cm[0 if Cm.shape[0] == 1 else b]
            ys.append(_forward(graph, x) @ c.T)
        out.append(torch.cat(ys))
    return out


@pytest.mark.parametrize("method", [abi.METHOD_IBP, abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_sound_by_sampling(method):
    g, bx = W.mlp_784_256x4_10(8)
    opt = abi.default_options(alpha_lr=0.1)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    ys = _sample_outputs(g, bx, 100_000)
    for b, y in enumerate(ys):
        tol = 1e-4 * (1 + np.abs(lb[b]).max())
        assert (y.min(0).values.cpu().numpy() >= lb[b] - tol).all()
        assert (y.max(0).values.cpu().numpy() <= ub[b] + tol).all()


def test_full_size_properties():
    """512 boxes of the 784-256x4-10 MLP: alpha-CROWN is sound, at least as
    tight as CROWN, and CROWN is at least as tight as IBP."""
    g, bx = W.mlp_784_256x4_10(512)
    opt = abi.default_options(alpha_lr=0.1)
    m = Model(g, options=opt)
    ilb, iub = m.compute_bounds(bx, abi.METHOD_IBP)
    clb, cub = m.compute_bounds(bx, abi.METHOD_CROWN)
    alb, aub = m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    assert np.isfinite(alb).all() and np.isfinite(aub).all()
    tol = 1e-4 * (1 + np.abs(clb))
    assert (clb >= ilb - tol).all() and (cub <= iub + tol).all()
    assert (alb >= clb - tol).all()
    assert (alb <= aub).all()
    sub = bx.slice(0, 16)
    for b, y in enumerate(_sample_outputs(g, sub, 20_000, seed=1)):
        assert (y.min(0).values.cpu().numpy() >= alb[b] - tol[b]).all()
        assert (y.max(0).values.cpu().numpy() <= aub[b] + tol[b]).all()
    # Per-box independence: a box bounded alone gets the same result.
    one = Model(g, options=opt).compute_bounds(bx.slice(5, 6), abi.METHOD_ALPHA_CROWN)
    assert G.excess(one[0], alb[5:6]) <= 1.0 and G.excess(one[1], aub[5:6]) <= 1.0


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_tensor_core_path_matches_simt_path(method):
    """The tcgen05 3xTF32 contractions agree with the SIMT fp32 ones within
    the parity bar (both are fp32-accurate; summation orders differ)."""
    g, bx = W.mlp_784_256x4_10(24)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=8)
    m = Model(g, options=opt)
    tlb, tub = m.compute_bounds(bx, method)
    m.set_contraction_path(1)
    slb, sub = m.compute_bounds(bx, method)
    print(f"tc vs simt: lb {G.excess(tlb, slb):.3f} ub {G.excess(tub, sub):.3f}")
    assert G.excess(tlb, slb) <= 1.0 and G.excess(tub, sub) <= 1.0
    # Tensor-core forward contractions with SIMT adjoint ones (path 3).
    m.set_contraction_path(3)
    mlb, mub = m.compute_bounds(bx, method)
    G.parity(f"tc forward + simt adjoint vs simt/{method}", mlb, mub, slb, sub)


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_cta_pair_contractions_match_single_cta(method):
    """Contractions on CTA pairs (tcgen05 cta_group::2, 256-row tiles) against
    single-CTA tiles.  A network of 256-wide layers never takes pairs
    (bit-identical by construction, a check of the path switch); the MLP's
    784-wide input concretisation takes 224-column pair tiles instead of
    112-column ones (its per-tile partial sums are added in another order),
    so that MLP is held to the parity bar.  600 boxes: M = 2 R rows spans
    several 256-row tiles with a ragged last one."""
    rng = np.random.default_rng(7)
    g = W.mlp([256, 256, 256, 256, 10], 11, bias_std=0.1)
    c = rng.uniform(-1.0, 1.0, (40, 256)).astype(np.float32)
    bx = W.Boxes((c - 0.05).astype(np.float32), (c + 0.05).astype(np.float32),
                 W.margin_spec(rng.integers(0, 10, 40), 10))
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=4)
    m = Model(g, options=opt)
    plb, pub = m.compute_bounds(bx, method)
    m.set_contraction_path(2)
    slb, sub = m.compute_bounds(bx, method)
    assert np.array_equal(plb, slb) and np.array_equal(pub, sub)
    g, bx = W.mlp_784_256x4_10(600)
    m = Model(g, options=opt)
    plb, pub = m.compute_bounds(bx, method)
    m.set_contraction_path(2)
    slb, sub = m.compute_bounds(bx, method)
    G.parity(f"cta pairs vs single ctas/{method}", plb, pub, slb, sub)


def test_device_pointer_entry_point_matches_host_entry_point():
    g, bx = W.mlp_5_50x6_5(64)
    m = Model(g, options=abi.default_options(alpha_lr=0.1))
    lb, ub = m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    xl = torch.from_numpy(bx.lower).cuda()
    xu = torch.from_numpy(bx.upper).cuda()
    Cm = torch.from_numpy(bx.C).cuda()
    dl = torch.empty((64, 4), device="cuda")
    du = torch.empty((64, 4), device="cuda")
    s = torch.cuda.current_stream()
    m.compute_bounds_ptr(abi.METHOD_ALPHA_CROWN, xl.data_ptr(), xu.data_ptr(), 64, Cm.data_ptr(), 1, 4,
                         dl.data_ptr(), du.data_ptr(), s.cuda_stream)
    # Same computation through both entry points: bit-identical results.
    assert np.array_equal(dl.cpu().numpy(), lb) and np.array_equal(du.cpu().numpy(), ub)


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_cnn_cifar_sound_and_ordered(method):
    """CIFAR-shaped CNN: bounds are sound at 10^5 sampled points per box and
    CROWN / alpha-CROWN are at least as tight as IBP / CROWN."""
    g, bx = W.cnn_cifar(6)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=8)
    m = Model(g, options=opt)
    ilb, iub = m.compute_bounds(bx, abi.METHOD_IBP)
    clb, cub = m.compute_bounds(bx, abi.METHOD_CROWN)
    lb, ub = m.compute_bounds(bx, method) if method != abi.METHOD_CROWN else (clb, cub)
    assert np.isfinite(lb).all() and np.isfinite(ub).all()
    tol = 1e-4 * (1 + np.abs(clb))
    assert (clb >= ilb - tol).all() and (cub <= iub + tol).all()
    assert (lb >= clb - tol).all() and (lb <= ub).all()
    for b, y in enumerate(_sample_outputs(g, bx.slice(0, 3), 100_000)):
        assert (y.min(0).values.cpu().numpy() >= lb[b] - tol[b]).all()
        assert (y.max(0).values.cpu().numpy() <= ub[b] + tol[b]).all()


@pytest.mark.parametrize("conv_after,wide", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_convt_matches_oracle(method, conv_after, wide):
    """Strided transposed conv below a linear head / below another conv; wide
    takes the register-blocked transposed-conv kernels."""
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.convt_cnn_case(31, n_boxes=3, conv_after=conv_after, wide=wide)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=6)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"convT/{method}/{int(conv_after)}/{int(wide)}", lb, ub, olb, oub)


def test_cnn_convt_cifar_sound():
    """The transposed-conv variant of the CIFAR CNN: CROWN bounds are sound at
    10^5 sampled points per box and at least as tight as IBP."""
    g, bx = W.cnn_convt_cifar(2, eps=2.0 / 255.0)
    m = Model(g, options=abi.default_options())
    ilb, iub = m.compute_bounds(bx, abi.METHOD_IBP)
    lb, ub = m.compute_bounds(bx, abi.METHOD_CROWN)
    tol = 1e-4 * (1 + np.abs(lb))
    assert np.isfinite(lb).all() and (lb >= ilb - tol).all() and (ub <= iub + tol).all()
    for b, y in enumerate(_sample_outputs(g, bx, 100_000)):
        assert (y.min(0).values.cpu().numpy() >= lb[b] - tol[b]).all()
        assert (y.max(0).values.cpu().numpy() <= ub[b] + tol[b]).all()


@pytest.mark.parametrize("seed,big", [(0, False), (1, False), (2, False), (3, True)])
@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_resnet_matches_oracle(method, seed, big):
    """Residual blocks (identity and 1x1 projection skips joined by Add), with
    dense starts and, with big, patches starts at the block convs."""
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.small_resnet_case(40 + seed, n_boxes=1 if big else 3, big=big)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=3 if big else 5)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"resnet{seed}/{method}/{int(big)}", lb, ub, olb, oub)


@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_resnet_cifar_sound_and_ordered(method):
    """The CIFAR ResNet (Sigmoid head): bounds are sound at 10^5 sampled
    points per box, CROWN at least as tight as IBP, alpha-CROWN's lower
    bound at least CROWN's."""
    g, bx = W.resnet_cifar(2)
    m = Model(g, options=abi.default_options(alpha_lr=0.1, alpha_iterations=5))
    ilb, iub = m.compute_bounds(bx, abi.METHOD_IBP)
    clb, cub = m.compute_bounds(bx, abi.METHOD_CROWN)
    lb, ub = m.compute_bounds(bx, method) if method != abi.METHOD_CROWN else (clb, cub)
    tol = 1e-4 * (1 + np.abs(clb))
    assert np.isfinite(lb).all() and (clb >= ilb - tol).all() and (cub <= iub + tol).all()
    assert (lb >= clb - tol).all() and (lb <= ub).all()
    for b, y in enumerate(_sample_outputs(g, bx, 100_000)):
        assert (y.min(0).values.cpu().numpy() >= lb[b] - tol[b]).all()
        assert (y.max(0).values.cpu().numpy() <= ub[b] + tol[b]).all()


@pytest.mark.parametrize("case", ["sig", "sigmix", "relusig", "resnetsig"])
@pytest.mark.parametrize("method", [abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_sigmoid_matches_oracle(method, case):
    """Sigmoid relaxations (secant, midpoint and table tangents), alone and
    mixed with ReLU; under alpha-CROWN the gradient runs through the Sigmoid
    relaxation's dependence on its input bounds."""
    from oracle.lirpa_oracle import LirpaOracle
    if case == "resnetsig":
        g, bx = W.small_resnet_case(60, n_boxes=3, head_act=abi.NODE_SIGMOID)
    else:
        acts = {"sig": (abi.NODE_SIGMOID, abi.NODE_SIGMOID), "sigmix": (abi.NODE_SIGMOID, abi.NODE_RELU),
                "relusig": (abi.NODE_RELU, abi.NODE_SIGMOID)}[case]
        g, bx = W.sigmoid_mlp_case(70, n_boxes=6, widths=(8, 24, 20, 5), acts=acts, eps=1.0)
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=6)
    lb, ub = Model(g, options=opt).compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"{case}/{method}", lb, ub, olb, oub)


@pytest.mark.parametrize("method", [abi.METHOD_IBP, abi.METHOD_CROWN, abi.METHOD_ALPHA_CROWN])
def test_batch_edge_cases(method):
    """Empty batch; a batch of one; zero-width boxes (points) and boxes with
    some zero-width pixels in a CNN; one shared specification matrix against
    one per box; splitting a batch does not change a box's bounds beyond the
    parity bar."""
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.small_cnn_case(11, n_boxes=5, big_first=False)
    bx.upper[0] = bx.lower[0]                  # a point
    bx.upper[1, ::3] = bx.lower[1, ::3]        # some pixels fixed
    opt = abi.default_options(alpha_lr=0.1, alpha_iterations=4)
    m = Model(g, options=opt)
    lb0, ub0 = m.compute_bounds(bx.slice(0, 0), method)
    assert lb0.shape == (0, bx.C.shape[1]) and ub0.shape == (0, bx.C.shape[1])
    lb, ub = m.compute_bounds(bx, method)
    olb, oub = LirpaOracle(g, opt).compute_bounds(bx, method)
    _assert_parity(f"edge/{method}", lb, ub, olb, oub)
    # A point box: lower and upper bounds meet at the network's value.
    y = W.graph_forward(g, torch.from_numpy(bx.lower[:1])).detach().numpy()[0] @ bx.C[0].T
    assert np.allclose(lb[0], y, atol=1e-4, rtol=1e-4) and np.allclose(ub[0], y, atol=1e-4, rtol=1e-4)
    # Batch of one, and the same boxes with a per-box copy of C.
    l1, u1 = m.compute_bounds(bx.slice(2, 3), method)
    _assert_parity(f"edge1/{method}", l1, u1, lb[2:3], ub[2:3])
    shared = W.Boxes(bx.lower, bx.upper, np.ascontiguousarray(bx.C[:1]))
    per_box = W.Boxes(bx.lower, bx.upper, np.repeat(bx.C[:1], bx.n, 0))
    ls, us = m.compute_bounds(shared, method)
    lp, up = m.compute_bounds(per_box, method)
    _assert_parity(f"edgeC/{method}", ls, us, lp, up)


@pytest.mark.parametrize("path", [0, 1])
@pytest.mark.parametrize("name", G.nostab_names())
def test_engine_matches_luna_without_stabilised_bounds(name, path):
    """STABILIZE_INTERMEDIATE_BOUNDS off, on a case where a layer stable at
    alpha creation turns unstable during the optimisation."""
    c = G.load(name, "nostab")
    m = Model(c["graph"], options=c["options"])
    m.set_contraction_path(path)
    lb, ub = m.compute_bounds(c["boxes"], c["method"])
    G.parity("nostab/" + name + ("/simt" if path == 1 else ""), lb, ub, c["lb"], c["ub"])
