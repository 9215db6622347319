"""CPU restatement of Luna's IBP / CROWN / alpha-CROWN -- test infrastructure.

This module is the oracle: a plain PyTorch (fp32, CPU, autograd) restatement
of the algorithm Luna runs for one input box, written from the reference's
behaviour and checked against Luna itself (oracle/_ref, built by
oracle/Makefile) in tests/test_oracle_golden.py, over the fixtures that
tests/golden/make_golden.py writes from Luna's outputs.  Only tests, smoke() and the
bench's CPU-baseline leg import it; the product never does.

Each function cites the Luna source (path within the Luna project) whose
behaviour it restates.  Per-box state follows Luna's: IBP bounds, "node
bounds" set by concretisation (BoundedTorchNode::setBounds), alpha
parameters keyed by (activation node, start node), and STE reference bounds.

Supported node kinds: Input, Linear, Conv2d, ConvTranspose2d, BatchNorm, ReLU, Sigmoid,
Add (of two tensors), Flatten, Identity, Reshape (flattening), Sub with a
constant, Slice of a flat vector (steps 1 / -1), Concat of flat vectors or
of maps along the channels.  A
matrices are kept dense over the flattened (C, H, W) features; Luna's
patches mode (CROWNAnalysis.cpp:255-405, BoundedConvNode.cpp:556-709) is the
same arithmetic on a window of those features, and it is tracked only to
pick the concretisation form Luna uses at the end of a start.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

import torch.nn.functional as F

from luna_b200.abi import (METHOD_ALPHA_CROWN, METHOD_CROWN, METHOD_IBP, NODE_ADD, NODE_BATCHNORM,
                           NODE_CONCAT, NODE_CONV, NODE_CONVTRANSPOSE, NODE_FLATTEN, NODE_IDENTITY, NODE_INPUT,
                           NODE_LINEAR, NODE_RELU, NODE_RESHAPE, NODE_SIGMOID, NODE_SLICE, NODE_SUB, Options,
                           default_options)

# Dense identity starts above this many conv output features switch to
# patches on Luna's CPU path (CROWNAnalysis.cpp:257,269).
PATCHES_SIZE_THRESHOLD = 4096


def slice_indices(nd, n_in: int):
    """Input feature of each output feature of a flat Slice, after
    BoundedSliceNode::_fixup_params (BoundedSliceNode.cpp:28-52): negative
    start / end count from the end, step -1 swaps them and reverses."""
    start, end = nd.start, nd.end
    if start < 0:
        start += n_in
    if end < 0:
        end = 0 if end == -9223372036854775807 else end + n_in
    if nd.step == -1:
        start, end = end, start
        end += 1
    end = min(end, n_in)
    start = max(start, 0)
    idx = list(range(start, end))
    return idx[::-1] if nd.step == -1 else idx


def topo_order(graph):
    """Kahn order seeded with in-degree-0 nodes by id (TorchModel::topologicalSort,
    src/engine/TorchModel.cpp:146-184)."""
    n = len(graph.nodes)
    deg = [len(graph.nodes[i].inputs) for i in range(n)]
    dependents = [[] for _ in range(n)]
    for i, nd in enumerate(graph.nodes):
        for p in nd.inputs:
            dependents[p].append(i)
    q = [i for i in range(n) if deg[i] == 0]
    out = []
    while q:
        c = q.pop(0)
        out.append(c)
        for d in dependents[c]:
            deg[d] -= 1
            if deg[d] == 0:
                q.append(d)
    return out, dependents


# ---------------------------------------------------------------- Sigmoid
# BoundedSigmoidNode's tangent-point tables (BoundedSigmoidNode.cpp:75-151):
# entry i of d_lower is the point whose tangent passes through
# (0.01 i, sigmoid(0.01 i)) from below, found by doubling then 100 bisection
# steps in fp32; d_upper mirrors it for (-0.01 i).  Every entry is computed
# independently of the table length, so one cache grown on demand serves
# every node (Luna grows its tables to the observed bound + 1, at least 20).
SIG_STEP = 0.01
SIG_CUTOFF = 20.0  # LunaConfiguration::SIGMOID_CUTOFF_CONSTANT


def _sig(x):
    return torch.sigmoid(x)


def _dsig(x):
    s = torch.sigmoid(x)
    return s * (1 - s)


class _SigmoidTables:
    def __init__(self):
        self.n = -1
        self.d_lower = None
        self.d_upper = None

    def ensure(self, limit):
        n = int(max(SIG_CUTOFF, limit) / SIG_STEP)
        if n <= self.n:
            return
        def check_lower(upper, d):
            return (_dsig(d) * (upper - d) + _sig(d)) <= _sig(upper)

        def check_upper(lower, d):
            return (_dsig(d) * (lower - d) + _sig(d)) >= _sig(lower)

        upper = SIG_STEP * torch.arange(0, n + 5, dtype=torch.float32)
        r = torch.zeros_like(upper)
        l = -torch.ones_like(upper)
        while True:
            c = check_lower(upper, l).to(torch.int64)
            l = c * l + (1 - c) * (l * 2)
            if int(c.sum()) == l.numel():
                break
        for _ in range(100):
            m = (l + r) / 2
            c = check_lower(upper, m).to(torch.int64)
            l = c * m + (1 - c) * l
            r = c * r + (1 - c) * m
        d_lower = l.clone()
        lower = -SIG_STEP * torch.arange(0, n + 5, dtype=torch.float32)
        l = torch.zeros_like(upper)
        r = torch.ones_like(upper)
        while True:
            c = check_upper(lower, r).to(torch.int64)
            r = c * r + (1 - c) * (r * 2)
            if int(c.sum()) == l.numel():
                break
        for _ in range(100):
            m = (l + r) / 2
            c = check_upper(lower, m).to(torch.int64)
            l = (1 - c) * m + c * l
            r = (1 - c) * r + c * m
        self.n, self.d_lower, self.d_upper = n, d_lower, r.clone()

    @staticmethod
    def retrieve(table, bound, default):
        """retrieveFromPrecompute (:162-186): entry max(0, int(bound / 0.01)) + 1."""
        idx = torch.clamp_min((bound.detach() / SIG_STEP).to(torch.int64).reshape(-1), 0) + 1
        if int(idx.max()) >= table.numel():
            ok = (idx < table.numel()).view(bound.shape)
            sel = table.index_select(0, torch.clamp(idx, 0, table.numel() - 1)).view(bound.shape)
            return torch.where(ok, sel, default)
        return table.index_select(0, idx).view(bound.shape)


_SIG_TABLES = _SigmoidTables()


def sigmoid_relaxation(l, u):
    """BoundedSigmoidNode::boundRelaxImpl (:282-338) with generateDLowerUpper
    (:188-209): (lw, lb, uw, ub) with lw x + lb <= sigmoid(x) <= uw x + ub on
    [l, u].  Secants where they are valid, the midpoint tangent on the
    convex / concave side, table tangents across 0."""
    needed = max(abs(float(l.detach().min())), abs(float(u.detach().max()))) + 1.0
    _SIG_TABLES.ensure(needed)
    mask_pos = l >= 0
    mask_neg = u <= 0
    mask_both = ~(mask_pos | mask_neg)
    zero = torch.zeros_like(l)
    lw, lb, uw, ub = zero, zero, zero, zero
    y_l, y_u = _sig(l), _sig(u)
    k_direct = (y_u - y_l) / (u - l).clamp_min(1e-8)
    same = (u - l).abs() < 1e-4
    k_direct = torch.where(same, _dsig(l), k_direct)
    uw = torch.where(mask_neg, k_direct, uw)
    ub = torch.where(mask_neg, y_l - k_direct * l, ub)
    lw = torch.where(mask_pos, k_direct, lw)
    lb = torch.where(mask_pos, y_l - k_direct * l, lb)
    d_lo = _SigmoidTables.retrieve(_SIG_TABLES.d_lower, u, l.detach())
    d_up = _SigmoidTables.retrieve(_SIG_TABLES.d_upper, -l, u.detach())
    mdl = mask_both & (k_direct < _dsig(l))
    mdu = mask_both & (k_direct < _dsig(u))
    lw = torch.where(mdl, k_direct, lw)
    lb = torch.where(mdl, y_l - k_direct * l, lb)
    uw = torch.where(mdu, k_direct, uw)
    ub = torch.where(mdu, y_l - k_direct * l, ub)
    mbl = mask_both & ~mdl
    mbu = mask_both & ~mdu
    k_t, y_t = _dsig(d_lo), _sig(d_lo)
    lw = torch.where(mbl, k_t, lw)
    lb = torch.where(mbl, y_t - k_t * d_lo, lb)
    k_t, y_t = _dsig(d_up), _sig(d_up)
    uw = torch.where(mbu, k_t, uw)
    ub = torch.where(mbu, y_t - k_t * d_up, ub)
    m = (l + u) / 2
    y_m, k_m = _sig(m), _dsig(m)
    lw = torch.where(mask_neg, k_m, lw)
    lb = torch.where(mask_neg, y_m - k_m * m, lb)
    uw = torch.where(mask_pos, k_m, uw)
    ub = torch.where(mask_pos, y_m - k_m * m, ub)
    return lw, lb, uw, ub


@dataclass
class _Alpha:
    alpha: torch.Tensor          # [2, spec, nU] leaf, requires grad
    idx: torch.Tensor            # [nU] int64 neuron ids unstable at creation


@dataclass
class _BoxState:
    node_bounds: dict = field(default_factory=dict)   # id -> (l, u): BoundedTorchNode::setBounds
    ibp: dict = field(default_factory=dict)           # CROWNAnalysis::_ibpBounds
    concrete: dict = field(default_factory=dict)      # CROWNAnalysis::_concreteBounds
    alphas: dict = field(default_factory=dict)        # (relu id, start id) -> _Alpha
    reference: dict = field(default_factory=dict)     # STE reference bounds id -> (l, u)
    alpha_mode: bool = False                          # ReLU stage "opt"
    method_alpha: bool = False                        # ANALYSIS_METHOD == AlphaCROWN
    first_linear_ibp: bool = True                     # ENABLE_FIRST_LINEAR_IBP


class _Adam:
    """torch::optim::Adam (betas 0.9/0.999, eps 1e-8, no weight decay) as
    AlphaCROWNAnalysis configures it (src/engine/AlphaCROWNAnalysis.cpp:366-368):
    m = m*b1 + (1-b1)*g;  v = v*b2 + (1-b2)*g*g;
    p += (-lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps), bias corrections in double."""

    def __init__(self, params):
        self.params = params
        self.m = [torch.zeros_like(p) for p in params]
        self.v = [torch.zeros_like(p) for p in params]
        self.t = 0

    @torch.no_grad()
    def step(self, lr):
        self.t += 1
        bc1 = 1.0 - 0.9 ** self.t
        bc2 = 1.0 - 0.999 ** self.t
        for p, m, v in zip(self.params, self.m, self.v):
            g = p.grad if p.grad is not None else torch.zeros_like(p)
            m.mul_(0.9).add_(g, alpha=1.0 - 0.9)
            v.mul_(0.999).addcmul_(g, g, value=1.0 - 0.999)
            denom = (v.sqrt() / np.sqrt(bc2)).add_(1e-8)
            p.addcdiv_(m, denom, value=-(lr / bc1))


class LirpaOracle:
    def __init__(self, graph, options: Options | None = None):
        self.g = graph
        self.opt = options if options is not None else default_options()
        self.order, self.dependents = topo_order(graph)
        self.W = {}
        self.b = {}
        for i, nd in enumerate(graph.nodes):
            if nd.type == NODE_LINEAR:
                # BoundedLinearNode bakes alpha (Gemm scale) into the weight (:91-93).
                self.W[i] = torch.from_numpy(np.asarray(nd.weight, np.float32)) * nd.scale
                self.b[i] = (torch.from_numpy(np.asarray(nd.bias, np.float32))
                             if nd.bias is not None else torch.zeros(nd.weight.shape[0]))
            elif nd.type in (NODE_CONV, NODE_CONVTRANSPOSE):
                self.W[i] = torch.from_numpy(np.asarray(nd.weight, np.float32))
                self.b[i] = (torch.from_numpy(np.asarray(nd.bias, np.float32))
                             if nd.bias is not None else torch.zeros(nd.weight.shape[0]))
            elif nd.type == NODE_BATCHNORM:
                # BoundedBatchNormNode::ensureCachedParams (BoundedBatchNormNode.cpp:68-80):
                # w = scale / sqrt(var + eps), b = B - mean * w, per channel,
                # repeated over the spatial positions of a flat CHW input (:94-116).
                f = lambda a: torch.from_numpy(np.asarray(a, np.float32))
                w = f(nd.weight) / torch.sqrt(f(nd.running_var) + np.float32(nd.eps))
                b = f(nd.bias) - f(nd.running_mean) * w
                spatial = nd.size // w.numel()
                self.W[i] = w.repeat_interleave(spatial)
                self.b[i] = b.repeat_interleave(spatial)
            elif nd.type == NODE_ADD:
                if len(nd.inputs) != 2:
                    raise NotImplementedError("oracle: Add of a constant")
            elif nd.type == NODE_SUB:
                if len(nd.inputs) != 1 or nd.constant is None:
                    raise NotImplementedError("oracle: Sub of two tensors")
                self.W[i] = torch.from_numpy(np.asarray(nd.constant, np.float32)).flatten()
            elif nd.type == NODE_SLICE:
                self.W[i] = torch.as_tensor(slice_indices(nd, graph.nodes[nd.inputs[0]].size), dtype=torch.long)
            elif nd.type not in (NODE_INPUT, NODE_RELU, NODE_SIGMOID, NODE_FLATTEN, NODE_IDENTITY, NODE_RESHAPE,
                                 NODE_CONCAT):
                raise NotImplementedError(f"oracle: node type {nd.type}")
        self.act_ids = [i for i, nd in enumerate(graph.nodes) if nd.type in (NODE_RELU, NODE_SIGMOID)]
        self.preact_ids = sorted({graph.nodes[i].inputs[0] for i in self.act_ids})

    # ------------------------------------------------------------------ IBP
    def _ibp_node(self, i, ins):
        """Interval forward of one node: Linear W+/W- matmuls
        (BoundedLinearNode.cpp:197-228,266-292), ReLU clamp (BoundedReLUNode.cpp:399-422)."""
        nd = self.g.nodes[i]
        if nd.type == NODE_LINEAR:
            l, u = ins[0]
            W = self.W[i]
            Wp, Wn = torch.clamp(W, min=0), torch.clamp(W, max=0)
            lo = torch.matmul(l, Wp.t()) + torch.matmul(u, Wn.t())
            hi = torch.matmul(u, Wp.t()) + torch.matmul(l, Wn.t())
            return lo + self.b[i], hi + self.b[i]
        if nd.type == NODE_CONV:
            # W+/W- convolutions (BoundedConvNode.cpp:864-943).
            l, u = ins[0]
            ci, h, w = self.g.nodes[nd.inputs[0]].out_shape
            W = self.W[i]
            Wp, Wn = torch.clamp_min(W, 0), torch.clamp_max(W, 0)
            conv = lambda t, k: F.conv2d(t.reshape(1, ci, h, w), k, stride=nd.stride, padding=nd.padding)
            b = self.b[i].view(1, -1, 1, 1)
            lo = (conv(l, Wp) + conv(u, Wn)) + b
            hi = (conv(u, Wp) + conv(l, Wn)) + b
            return lo.flatten(), hi.flatten()
        if nd.type == NODE_CONVTRANSPOSE:
            # Centre / radius (BoundedConvTransposeNode.cpp:466-488):
            # c = convT(mid, W) + b, d = convT(diff, |W|), [c - d, c + d].
            l, u = ins[0]
            ci, h, w = self.g.nodes[nd.inputs[0]].out_shape
            mid = ((u + l) / 2.0).reshape(1, ci, h, w)
            diff = ((u - l) / 2.0).reshape(1, ci, h, w)
            dev = F.conv_transpose2d(diff, self.W[i].abs(), stride=nd.stride, padding=nd.padding)
            cen = F.conv_transpose2d(mid, self.W[i], self.b[i], stride=nd.stride, padding=nd.padding)
            return (cen - dev).flatten(), (cen + dev).flatten()
        if nd.type == NODE_BATCHNORM:
            # BoundedBatchNormNode::computeIntervalBoundPropagation (:151-178).
            l, u = ins[0]
            w, b = self.W[i], self.b[i]
            wp, wn = torch.clamp_min(w, 0), torch.clamp_max(w, 0)
            return wp * l + wn * u + b, wp * u + wn * l + b
        if nd.type == NODE_RELU:
            l, u = ins[0]
            return torch.clamp_min(l, 0), torch.clamp_min(u, 0)
        if nd.type == NODE_SIGMOID:
            # Monotone (BoundedSigmoidNode.cpp:248-272).
            l, u = ins[0]
            return _sig(l), _sig(u)
        if nd.type == NODE_ADD:
            # BoundedAddNode::computeIntervalBoundPropagation (:281-304).
            (l1, u1), (l2, u2) = ins
            return l1 + l2, u1 + u2
        if nd.type in (NODE_FLATTEN, NODE_IDENTITY, NODE_RESHAPE):
            return ins[0]
        if nd.type == NODE_SUB:
            # BoundedSubNode::computeIntervalBoundPropagation (:205-233):
            # [l - c, u - c], or [c - u, c - l] for a constant first operand.
            l, u = ins[0]
            c = self.W[i]
            if nd.constant_second:
                return l - c, u - c
            return c - u, c - l
        if nd.type == NODE_SLICE:
            # BoundedSliceNode::forward on both bounds (narrow, flipped for step -1).
            l, u = ins[0]
            return l[self.W[i]], u[self.W[i]]
        if nd.type == NODE_CONCAT:
            # BoundedConcatNode::computeIntervalBoundPropagation: cat of the
            # flat bounds (channel order for maps).
            return torch.cat([x[0] for x in ins]), torch.cat([x[1] for x in ins])
        raise NotImplementedError

    def _input_bounds_of(self, st, i, x):
        """CROWNAnalysis::getInputBoundsForNode (src/engine/CROWNAnalysis.cpp:1043-1101):
        input box for the Input node, else node bounds > concrete > IBP."""
        out = []
        for p in self.g.nodes[i].inputs:
            if self.g.nodes[p].type == NODE_INPUT:
                out.append(x)
            elif p in st.node_bounds:
                out.append(st.node_bounds[p])
            elif p in st.concrete:
                out.append(st.concrete[p])
            else:
                out.append(st.ibp[p])
        return out

    def _compute_ibp(self, st, x):
        """CROWNAnalysis::computeIBPBounds (src/engine/CROWNAnalysis.cpp:180-214)."""
        st.ibp = {}
        for i in self.order:
            if self.g.nodes[i].type == NODE_INPUT:
                st.ibp[i] = x
                continue
            lo, hi = self._ibp_node(i, self._input_bounds_of(st, i, x))
            st.ibp[i] = (lo.detach(), hi.detach())

    # ------------------------------------------------------------ ReLU relax
    @staticmethod
    def _upper(l, u):
        """BoundedReLUNode::_reluUpperBound (BoundedReLUNode.cpp:469-479)."""
        lb_r = torch.clamp_max(l, 0)
        ub_r = torch.clamp_min(u, 0)
        ub_r = torch.max(ub_r, lb_r + 1e-8)
        d = ub_r / (ub_r - lb_r)
        return d, -lb_r * d

    @staticmethod
    def _crown_lower(l, u):
        """BoundedReLUNode::_computeStandardCROWNLowerBound (BoundedReLUNode.cpp:481-504)."""
        s = torch.zeros_like(l)
        s = torch.where(l >= 0, torch.ones_like(s), s)
        unc = (l < 0) & (u > 0)
        lb_r = torch.clamp_max(l, 0)
        ub_r = torch.clamp_min(u, 0)
        ub_r = torch.max(ub_r, lb_r + 1e-8)
        up = ub_r / (ub_r - lb_r)
        ad = torch.where(up > 0.5, torch.ones_like(l), torch.zeros_like(l))
        return torch.where(unc, ad, s)

    def _relu_backward(self, st, relu_id, start_id, lA, uA, l, u):
        """BoundedReLUNode::boundBackward (BoundedReLUNode.cpp:54-362) for dense A
        [spec, n], with _backwardRelaxation (:446-467) and, in the
        optimisation stage, _maskAlpha (:507-612).  Returns new A and bias
        terms (bias [spec])."""
        d_up, b_up = self._upper(l, u)
        d_lo = self._crown_lower(l, u)
        spec = lA.shape[0]
        if st.alpha_mode:
            key = (relu_id, start_id)
            ap = st.alphas.get(key)
            if ap is None or ap.alpha.shape[1] != spec:
                ap = self._ensure_alpha(st, key, spec, l, u, d_lo)
            active = l >= 0
            inactive = u <= 0
            if ap.idx.numel() > 0:
                n = l.numel()
                idx = ap.idx.unsqueeze(0).expand(spec, ap.idx.numel())
                a_lo = torch.zeros(spec, n).scatter(1, idx, ap.alpha[0])
                a_up = torch.zeros(spec, n).scatter(1, idx, ap.alpha[1])
                one = torch.ones(spec, n)
                a_lo = torch.where(active.unsqueeze(0).expand(spec, n), one, a_lo)
                a_up = torch.where(active.unsqueeze(0).expand(spec, n), one, a_up)
                k_up = torch.where(active, torch.ones_like(d_up), d_up)
                k_up = torch.where(inactive, torch.zeros_like(k_up), k_up)
                bu = -l * d_up
                bu = torch.where(active | inactive, torch.zeros_like(bu), bu)
                Lpos, Lneg = torch.clamp_min(lA, 0), torch.clamp_max(lA, 0)
                Upos, Uneg = torch.clamp_min(uA, 0), torch.clamp_max(uA, 0)
                k = k_up.unsqueeze(0)
                new_l = Lpos * a_lo + Lneg * k
                new_u = Upos * k + Uneg * a_up
                bl = (Lpos * torch.zeros_like(bu) + Lneg * bu).sum(-1)
                bu_ = (Upos * bu + Uneg * torch.zeros_like(bu)).sum(-1)
                return new_l, new_u, bl, bu_
        # Standard CROWN relaxation.
        Lpos, Lneg = torch.clamp_min(lA, 0), torch.clamp_max(lA, 0)
        Upos, Uneg = torch.clamp_min(uA, 0), torch.clamp_max(uA, 0)
        zero = torch.zeros_like(l)
        new_l = Lpos * d_lo + Lneg * d_up
        new_u = Upos * d_up + Uneg * d_lo
        bl = (Lpos * zero + Lneg * b_up).sum(-1)
        bu_ = (Upos * b_up + Uneg * zero).sum(-1)
        return new_l, new_u, bl, bu_

    def _ensure_alpha(self, st, key, spec, l, u, d_lo):
        """AlphaCROWNAnalysis::ensureAlphaFor (src/engine/AlphaCROWNAnalysis.cpp:132-304):
        alpha [2, spec, nU] at the neurons unstable now, initialised with the
        CROWN lower slope, clamped to [0, 1]."""
        mask = (l.detach() < 0) & (u.detach() > 0)
        idx = torch.nonzero(mask).flatten()
        init = d_lo.detach().flatten().index_select(0, idx)
        a = init.view(1, 1, -1).expand(2, spec, idx.numel()).contiguous().clone()
        # With no unstable neuron Luna stores an empty alpha that does not
        # require grad (AlphaCROWNAnalysis.cpp:179-188).
        a = torch.clamp(a, 0.0, 1.0).detach().requires_grad_(idx.numel() > 0)
        ap = _Alpha(a, idx)
        st.alphas[key] = ap
        return ap

    # -------------------------------------------------------- backward pass
    def _conv_backward(self, c, A):
        """BoundedConvNode::boundOneSide, tensor mode (BoundedConvNode.cpp:448-556):
        A [spec, Co*Ho*Wo] -> conv_transpose2d with the output padding that
        restores the input size; bias term sum_{c,h,w} A b_c."""
        nd = self.g.nodes[c]
        ci, hi, wi = self.g.nodes[nd.inputs[0]].out_shape
        co, ho, wo = nd.out_shape
        kh, kw = nd.kernel
        (sh, sw), (ph, pw) = nd.stride, nd.padding
        op = (hi - ((ho - 1) * sh - 2 * ph + kh), wi - ((wo - 1) * sw - 2 * pw + kw))
        spec = A.shape[0]
        A4 = A.reshape(spec, co, ho, wo)
        out = F.conv_transpose2d(A4, self.W[c], stride=nd.stride, padding=nd.padding, output_padding=op)
        bias = (A4 * self.b[c].view(1, -1, 1, 1)).sum((1, 2, 3))
        return out.reshape(spec, -1), bias

    def _starts_in_patches(self, start, is_output):
        """usePatchesInit on the CPU path (CROWNAnalysis.cpp:255-298): a conv
        start, or a BatchNorm start whose producer is a conv, with more than
        4096 output features."""
        nd = self.g.nodes[start]
        if not self.opt.use_patches_mode or is_output or nd.size <= PATCHES_SIZE_THRESHOLD:
            return False
        if nd.type == NODE_CONV:
            return True
        return nd.type == NODE_BATCHNORM and self.g.nodes[nd.inputs[0]].type == NODE_CONV

    def _backward_from(self, st, start, x, rows=None, C=None):
        """CROWNAnalysis::backwardFrom (src/engine/CROWNAnalysis.cpp:231-706) for
        dense A: start A is the spec C (output) or one-hot rows at `rows`;
        Kahn-style reverse schedule; bias attached to the first dependency.
        Returns (lA, uA, lbias, ubias, patches) at the input node; `patches`
        tells whether Luna would still hold the start's A as patches there
        (it converts to a matrix once a patch is wider than the conv input,
        BoundedConvNode.cpp:671-694, and at a join of patches with a matrix,
        CROWNAnalysis::addA :1307-1354; patches meeting patches are padded to
        the wider one, Patches::add, Patches.cpp:86-129)."""
        n = self.g.nodes[start].size
        # (patches?, patch width) of the A accumulated at each node; width
        # None = the identity patches of the start.
        form = {start: (self._starts_in_patches(start, C is not None), None)}
        # Luna keeps a tensor A flat ([spec, 1, n]) between nodes: a conv node
        # reshapes its [spec, 1, C, H, W] result back when the input bounds
        # are flat (BoundedConvNode.cpp:430-445).  ConvTranspose adds its
        # bias term only for a 4-D / 5-D A or patches, so in tensor mode its
        # bias never enters the back-substitution (BoundedConvTransposeNode.cpp:289-311).
        if C is not None:
            A0 = C
        else:
            A0 = torch.zeros(len(rows), n)
            A0[torch.arange(len(rows)), torch.as_tensor(rows, dtype=torch.long)] = 1.0
        spec = A0.shape[0]
        lA = {start: A0}
        uA = {start: A0}
        lb = {start: torch.zeros(spec)}
        ub = {start: torch.zeros(spec)}
        reach = {start}
        work = [start]
        while work:
            c = work.pop(0)
            for p in self.g.nodes[c].inputs:
                if p not in reach:
                    reach.add(p)
                    work.append(p)
        pending = {v: sum(1 for d in self.dependents[v] if d in reach) for v in reach}
        queue = [start]
        done = set()
        inp = self.g.input_index
        while queue:
            c = queue.pop(0)
            if c in done:
                continue
            done.add(c)
            nd = self.g.nodes[c]
            if c in lA:
                a_l, a_u = lA[c], uA[c]
                patches, pwidth = form[c]
                if nd.type == NODE_LINEAR:
                    W, bb = self.W[c], self.b[c]
                    out = [(torch.matmul(a_l, W), torch.matmul(a_u, W))]
                    nb_l = (a_l * bb).sum(-1)
                    nb_u = (a_u * bb).sum(-1)
                elif nd.type == NODE_BATCHNORM:
                    # BoundedBatchNormNode::boundOneSideTensor (:180-361): A w, bias A b.
                    w, bb = self.W[c], self.b[c]
                    out = [(a_l * w, a_u * w)]
                    nb_l = (a_l * bb).sum(-1)
                    nb_u = (a_u * bb).sum(-1)
                    if patches and pwidth is None:
                        pwidth = 1  # identity patches become 1x1 channel-diagonal patches (:389-420)
                elif nd.type == NODE_CONVTRANSPOSE:
                    # BoundedConvTransposeNode::boundOneSide, tensor mode (:250-311):
                    # conv2d(A, W, stride, padding); bias sum_{c,h,w} A b_c.
                    ci, hi, wi = self.g.nodes[nd.inputs[0]].out_shape
                    co, ho, wo = nd.out_shape
                    outs = []
                    for a in (a_l, a_u):
                        a4 = a.reshape(a.shape[0], co, ho, wo)
                        bias = ((a4.sum((2, 3)) * self.b[c].view(1, -1)).sum(-1) if patches
                                else torch.zeros(a.shape[0]))
                        outs.append((F.conv2d(a4, self.W[c], stride=nd.stride, padding=nd.padding)
                                     .reshape(a.shape[0], -1), bias))
                    out = [(outs[0][0], outs[1][0])]
                    nb_l, nb_u = outs[0][1], outs[1][1]
                    patches = False
                elif nd.type == NODE_CONV:
                    nl, nb_l = self._conv_backward(c, a_l)
                    nu, nb_u = self._conv_backward(c, a_u)
                    out = [(nl, nu)]
                    if patches:
                        kw = nd.kernel[1]
                        pwidth = kw if pwidth is None else (pwidth - 1) * nd.stride[1] + kw
                        if pwidth > self.g.nodes[nd.inputs[0]].out_shape[2]:
                            patches = False
                elif nd.type == NODE_RELU:
                    l, u = self._input_bounds_of(st, c, x)[0]
                    nl, nu, nb_l, nb_u = self._relu_backward(st, c, start, a_l, a_u, l, u)
                    out = [(nl, nu)]
                elif nd.type == NODE_SIGMOID:
                    # BoundedSigmoidNode::boundBackward, tensor A (:639-832):
                    # lower A+ lw + A- uw, bias A+ lb + A- ub; upper mirrored.
                    # No alpha for Sigmoid: Luna's alpha-CROWN cannot create it
                    # (ensureAlphaFor writes its 8 tangent slots along the
                    # neuron axis and throws, AlphaCROWNAnalysis.cpp:264-272),
                    # so the CROWN relaxation stays, differentiable in (l, u).
                    l, u = self._input_bounds_of(st, c, x)[0]
                    lw, lbs, uw, ubs = sigmoid_relaxation(l, u)
                    Lp, Ln = torch.clamp_min(a_l, 0), torch.clamp_max(a_l, 0)
                    Up, Un = torch.clamp_min(a_u, 0), torch.clamp_max(a_u, 0)
                    out = [(Lp * lw + Ln * uw, Up * uw + Un * lw)]
                    nb_l = (Lp * lbs + Ln * ubs).sum(-1)
                    nb_u = (Up * ubs + Un * lbs).sum(-1)
                elif nd.type == NODE_ADD:
                    # BoundedAddNode::boundBackward (:167-279): the same A to both
                    # operands (equal shapes), no bias of its own.
                    out = [(a_l, a_u), (a_l, a_u)]
                    nb_l = nb_u = None
                elif nd.type in (NODE_FLATTEN, NODE_IDENTITY, NODE_INPUT, NODE_RESHAPE):
                    out = [(a_l, a_u)]
                    nb_l = nb_u = None
                elif nd.type == NODE_SUB:
                    # BoundedSubNode::boundBackward with a constant (:61-165):
                    # x - c passes A and adds -A c; c - x passes -A and adds A c.
                    c_ = self.W[c]
                    if nd.constant_second:
                        out = [(a_l, a_u)]
                        nb_l, nb_u = -torch.matmul(a_l, c_), -torch.matmul(a_u, c_)
                    else:
                        out = [(-a_l, -a_u)]
                        nb_l, nb_u = torch.matmul(a_l, c_), torch.matmul(a_u, c_)
                elif nd.type == NODE_SLICE:
                    # BoundedSliceNode::boundBackward (:113-201): A scattered
                    # into zeros of the input size at the sliced features.
                    n_in = self.g.nodes[nd.inputs[0]].size
                    idx = self.W[c]
                    outs = []
                    for a in (a_l, a_u):
                        z = torch.zeros(a.shape[0], n_in)
                        z[:, idx] = a
                        outs.append(z)
                    out = [tuple(outs)]
                    nb_l = nb_u = None
                elif nd.type == NODE_CONCAT:
                    # BoundedConcatNode::boundBackward (:56-178): A split along
                    # the features into the operands' sizes, no bias.
                    sizes = [self.g.nodes[p].size for p in nd.inputs]
                    out = list(zip(torch.split(a_l, sizes, dim=1), torch.split(a_u, sizes, dim=1)))
                    nb_l = nb_u = None
                else:
                    raise NotImplementedError
                for k, p in enumerate(nd.inputs):
                    if k >= len(out):
                        break
                    pl, pu = out[k]
                    lA[p] = lA[p] + pl if p in lA else pl
                    uA[p] = uA[p] + pu if p in uA else pu
                    if p in form:
                        fp, wp = form[p]
                        form[p] = (fp and patches, max(wp or 1, pwidth or 1))
                    else:
                        form[p] = (patches, pwidth)
                    if k == 0:
                        # propagated = node bias + accumulated bias (:629-657)
                        # A node reached only through a second operand has no
                        # accumulated bias of its own.
                        zero = torch.zeros(a_l.shape[0])
                        acc_l, acc_u = lb.get(c, zero), ub.get(c, zero)
                        tl = acc_l if nb_l is None else nb_l + acc_l
                        tu = acc_u if nb_u is None else nb_u + acc_u
                        lb[p] = lb[p] + tl if p in lb else tl
                        ub[p] = ub[p] + tu if p in ub else tu
                if c != inp:
                    del lA[c], uA[c]
                    lb.pop(c, None)
                    ub.pop(c, None)
            for p in nd.inputs:
                if p in pending and pending[p] > 0:
                    pending[p] -= 1
                    if pending[p] == 0:
                        queue.append(p)
        return lA[inp], uA[inp], lb[inp], ub[inp], form[inp][0]

    @staticmethod
    def _concretize(lA, uA, lb, ub, x, patches=False):
        """computeConcreteLowerBound/UpperBound (src/engine/CROWNAnalysis.cpp:1164-1224):
        lb = A+ xL + A- xU + bias, ub = A+ xU + A- xL + bias; for patches
        (concretizeNode, :791-848 with Patches::matmul) lb = A c - |A| d + bias,
        ub = A c + |A| d + bias with c = (xU + xL)/2, d = (xU - xL)/2."""
        xl, xu = x
        if patches:
            c = (xu + xl) / 2.0
            d = (xu - xl) / 2.0
            lo = (torch.matmul(lA, c) - torch.matmul(lA.abs(), d)) + lb
            hi = (torch.matmul(uA, c) + torch.matmul(uA.abs(), d)) + ub
            return lo, hi
        lo = (torch.matmul(torch.clamp_min(lA, 0), xl) + torch.matmul(torch.clamp_max(lA, 0), xu)) + lb
        hi = (torch.matmul(torch.clamp_min(uA, 0), xu) + torch.matmul(torch.clamp_max(uA, 0), xl)) + ub
        return lo, hi

    def _is_first_linear(self, i):
        """CROWNAnalysis::isFirstLinearLayer (:1672-1701)."""
        nd = self.g.nodes[i]
        return (nd.type == NODE_LINEAR and len(nd.inputs) == 1
                and self.g.nodes[nd.inputs[0]].type == NODE_INPUT)

    def _lazy_intermediate(self, st, i, x):
        """CROWNAnalysis::computeIntermediateBoundsLazy (:1744-1795) and
        concretizeNode's scatter + STE clamp (:877-938)."""
        if i in st.node_bounds or i in st.concrete:
            return
        if st.first_linear_ibp and self._is_first_linear(i):
            lo, hi = self._ibp_node(i, self._input_bounds_of(st, i, x))
            st.node_bounds[i] = (lo, hi)
            st.ibp[i] = (lo, hi)
            st.concrete[i] = (lo, hi)
            return
        il, iu = st.ibp[i]
        rows = torch.nonzero((il < 0) & (iu > 0)).flatten().tolist()
        if not rows:
            st.concrete[i] = st.ibp[i]
            st.node_bounds[i] = st.ibp[i]
            return
        lA, uA, lb, ub, patches = self._backward_from(st, i, x, rows=rows)
        lo, hi = self._concretize(lA, uA, lb, ub, x, patches)
        idx = torch.as_tensor(rows, dtype=torch.long)
        if not st.method_alpha:
            lo, hi = lo.detach(), hi.detach()
        full_l = il.detach().clone().index_put((idx,), lo)
        full_u = iu.detach().clone().index_put((idx,), hi)
        if st.method_alpha and i in st.reference:
            rl, ru = st.reference[i]
            full_l = torch.max(rl, full_l).detach() - full_l.detach() + full_l
            full_u = full_u - (full_u.detach() - torch.min(ru, full_u).detach())
        st.concrete[i] = (full_l, full_u)
        st.node_bounds[i] = (full_l, full_u)

    def _check_prior(self, st, i, x):
        """CROWNAnalysis::checkPriorBounds (:1797-1818)."""
        nd = self.g.nodes[i]
        for p in nd.inputs:
            self._check_prior(st, p, x)
        if nd.type in (NODE_RELU, NODE_SIGMOID):
            self._lazy_intermediate(st, nd.inputs[0], x)

    def _run(self, st, x, C):
        """CROWNAnalysis::run with USE_STANDARD_CROWN (:93-142).  Returns the
        output (lb, ub) [nspec]."""
        self._compute_ibp(st, x)
        out = self.g.output_index
        self._check_prior(st, out, x)
        lA, uA, lb, ub, patches = self._backward_from(st, out, x, C=C)
        lo, hi = self._concretize(lA, uA, lb, ub, x, patches)
        st.node_bounds[out] = (lo, hi)
        st.concrete[out] = (lo, hi)
        return lo, hi

    # ---------------------------------------------------------- public API
    def ibp(self, xl, xu, C):
        st = _BoxState()
        x = (torch.as_tensor(xl), torch.as_tensor(xu))
        self._compute_ibp(st, x)
        lo, hi = st.ibp[self.g.output_index]
        Cp, Cn = torch.clamp_min(C, 0), torch.clamp_max(C, 0)
        return Cp @ lo + Cn @ hi, Cp @ hi + Cn @ lo

    def crown(self, xl, xu, C, st=None):
        """TorchModel::runCROWN (src/engine/TorchModel.cpp:710-740) on a fresh model."""
        st = st or _BoxState(first_linear_ibp=bool(self.opt.enable_first_linear_ibp))
        x = (torch.as_tensor(xl), torch.as_tensor(xu))
        with torch.no_grad():
            lo, hi = self._run(st, x, C)
        return lo, hi, st

    @staticmethod
    def verified(lb, spec) -> bool:
        """TorchModel::isSpecVerified (src/engine/TorchModel.cpp:616-651) from
        the lower bounds: spec = (thresholds, branch of each row, n_branches);
        a conjunction (n_branches 0) is broken by one row with lb - thr > 0,
        a disjunction needs such a row in every branch
        (OutputConstraintSet::evaluateORBranches, OutputConstraint.cpp:187-278)."""
        thr, branch, nb = spec
        d = (lb.reshape(-1) - thr.reshape(-1)) > 0
        if nb <= 0:
            return bool(d.any())
        return all(bool(d[torch.as_tensor(branch) == b].any()) for b in range(nb))

    def alpha_crown(self, xl, xu, C, trace=None, spec=None, seed=None):
        """TorchModel::runAlphaCROWN (src/engine/TorchModel.cpp:798-893) with
        AlphaCROWNAnalysis::computeOptimizedBounds(Lower)
        (src/engine/AlphaCROWNAnalysis.cpp:306-511) for the lower side and
        runCROWN on the same nodes for the upper side.  With `spec`
        (thresholds, branches, n_branches; see verified()) the early stops
        apply: STOP_CROWN_ON_VERIFIED returns the CROWN initialisation pass's
        bounds when they verify (TorchModel.cpp:816-834), and
        STOP_ALPHA_ON_VERIFIED ends the optimisation at the first iteration
        whose bounds verify, after taking them into the best bound
        (AlphaCROWNAnalysis.cpp:394-407).

        `seed` ({(relu id, start id): _Alpha}, another box's last_alphas) is
        TorchModel::loadState's warm start (TorchModel.cpp:975-983, :813-814;
        AlphaCROWNAnalysis::seedAlphas, AlphaCROWNAnalysis.cpp:971-997): the
        analysis starts from copies of those alphas, all requiring grad,
        marked initialised (no CROWN initialisation pass), with the
        best-alpha map aliasing the seeded tensors; ensureAlphaFor reuses a
        seeded alpha only when its specification count matches and
        recreates it otherwise (_relu_backward).  After the call,
        last_alphas holds this box's alphas as TorchModel::getState returns
        them."""
        o = self.opt
        x = (torch.as_tensor(xl), torch.as_tensor(xu))
        if seed is None and spec is not None and o.stop_crown_on_verified:
            # performCROWNInitializationPass (AlphaCROWNAnalysis.cpp:118-129):
            # plain CROWN with the first-linear-IBP shortcut off.
            lo0, hi0, st0 = self.crown(xl, xu, C, _BoxState(first_linear_ibp=False))
            if self.verified(lo0, spec):
                inter = {i: st0.node_bounds[i] for i in self.preact_ids if i in st0.node_bounds}
                return lo0.detach(), hi0.detach(), inter
        st = _BoxState(method_alpha=True, first_linear_ibp=False)
        st.alpha_mode = True
        st.seeded = {}
        for k, ap in (seed or {}).items():
            a = ap.alpha.detach().clone().requires_grad_(True)
            st.alphas[k] = _Alpha(a, ap.idx.clone())
            st.seeded[k] = a
        # TorchModel::runAlphaCROWN (:838-862): the upper side first when it is
        # optimised, then the lower side, in one AlphaCROWNAnalysis (the alphas
        # carry over); a side that is not optimised comes from the runCROWN
        # that follows; with neither side optimised it is runCROWN alone.
        sides = ([True] if o.optimize_upper else []) + ([False] if o.optimize_lower else [])
        if not sides:
            lo, hi, st0 = self.crown(xl, xu, C)
            inter = {i: st0.node_bounds[i] for i in self.preact_ids if i in st0.node_bounds}
            return lo.detach(), hi.detach(), inter
        res = {}
        for up in sides:
            res[up] = self._optimize_side(st, x, C, up, trace, spec)
        self.last_alphas = {k: _Alpha(ap.alpha.detach().clone(), ap.idx.clone()) for k, ap in st.alphas.items()}
        lb = res[False][0] if False in res else res[True][1]
        ub = res[True][0] if True in res else res[False][1]
        return lb, ub, res[sides[-1]][2]

    def _optimize_side(self, st, x, C, upper, trace, spec):
        """AlphaCROWNAnalysis::computeOptimizedBounds(side)
        (src/engine/AlphaCROWNAnalysis.cpp:306-511) on the state `st` (alphas
        kept across calls).  Upper: loss = sum ub, best = min, improvement =
        decrease; STOP_ALPHA_ON_VERIFIED checks the lower bounds on either
        side.  Returns (the optimised side's bound, the other side from the
        runCROWN that follows over the same nodes, best intermediate bounds)."""
        o = self.opt
        st.node_bounds, st.concrete, st.reference = {}, {}, {}
        self._run(st, x, C)
        best_int = {i: (st.node_bounds[i][0].detach().clone(), st.node_bounds[i][1].detach().clone())
                    for i in self.preact_ids if i in st.node_bounds}
        if o.stabilize_intermediate_bounds:
            st.reference = {k: (v[0].clone(), v[1].clone()) for k, v in best_int.items()}

        def other_side():
            st2 = _BoxState(node_bounds={k: v for k, v in st.node_bounds.items() if k in best_int},
                            alphas=st.alphas, alpha_mode=True, method_alpha=True, first_linear_ibp=False)
            lo2, hi2 = self._run(st2, x, C)
            return (lo2 if upper else hi2).detach()

        params = [ap.alpha for ap in st.alphas.values() if ap.alpha.requires_grad]
        if not params:
            # collectAlphaParameters() found nothing to optimise: one more
            # run(false) over the bounds still on the nodes (:360-364).
            with torch.no_grad():
                lo, hi = self._run(st, x, C)
                return (hi if upper else lo).detach(), other_side(), best_int
        adam = _Adam(params)
        iters = int(o.alpha_iterations)
        best = None
        lr = float(o.alpha_lr)
        patience = 0
        best_loss = None
        # Seeded alphas: the best-alpha map starts as the alpha map itself
        # (the same tensors), so saving and restoring them are no-ops.
        best_alpha = {k: a.detach() for k, a in getattr(st, "seeded", {}).items()}
        for it in range(iters):
            last = it == iters - 1
            st.node_bounds, st.concrete = {}, {}
            with torch.set_grad_enabled(not last):
                cur_l, cur_u = self._run(st, x, C)
            cur = (cur_u if upper else cur_l).detach()
            if trace is not None:
                trace.append(cur.clone())
            if spec is not None and o.stop_alpha_on_verified and self.verified(cur_l.detach(), spec):
                best = cur.clone() if best is None else (torch.min(best, cur) if upper else torch.max(best, cur))
                break
            loss = None if last else (cur_u.sum() if upper else -cur_l.sum())
            if best is None:
                best = cur.clone()
                improved_idx = list(range(cur.numel()))
            else:
                improved_idx = torch.nonzero(cur < best if upper else cur > best).flatten().tolist()
                if improved_idx:
                    best = torch.min(best, cur) if upper else torch.max(best, cur)
            improved = len(improved_idx) > 0
            save = it < 1 or it > int(iters * o.start_save_best) or patience >= o.early_stop_patience
            if improved and save:
                self._update_best_alphas(st, best_alpha, improved_idx)
                for i in self.preact_ids:
                    if i in st.node_bounds:
                        cl, cu = st.node_bounds[i]
                        if i in best_int:
                            best_int[i] = (torch.max(best_int[i][0], cl.detach()).clone(),
                                           torch.min(best_int[i][1], cu.detach()).clone())
                        else:
                            best_int[i] = (cl.detach().clone(), cu.detach().clone())
                if o.stabilize_intermediate_bounds:
                    st.reference = {k: (v[0].clone(), v[1].clone()) for k, v in best_int.items()}
            if improved:
                if loss is not None:
                    best_loss = loss.detach().abs()
                patience = 0
            elif loss is not None:
                cl = loss.detach().abs()
                if best_loss is None or bool(cl < best_loss):
                    best_loss = cl
                    patience = 0
                else:
                    patience += 1
            if patience >= o.early_stop_patience:
                break
            if not last and loss is not None and loss.requires_grad:
                for p in params:
                    p.grad = None
                loss.backward()
                adam.step(lr)
                with torch.no_grad():
                    for p in params:
                        p.clamp_(0.0, 1.0)
                lr = float(np.float32(lr) * np.float32(o.alpha_lr_decay))
        # restoreBestAlphas / restoreBestIntermediateBounds / final run(false)
        with torch.no_grad():
            for key, ap in st.alphas.items():
                if key in best_alpha and best_alpha[key].shape == ap.alpha.shape:
                    ap.alpha.copy_(best_alpha[key])
            st.reference = {}
            st.concrete = {}
            st.node_bounds = {k: (v[0].clone(), v[1].clone()) for k, v in best_int.items()}
            fin_l, fin_u = self._run(st, x, C)
            if upper:
                final = torch.min(fin_u, best) if best is not None else fin_u
            else:
                final = torch.max(fin_l, best) if best is not None else fin_l
            # runCROWN for the non-optimised side: a new analysis over the same
            # nodes, whose pre-activation bounds are still the best ones and
            # whose ReLUs still read the optimised alphas (stage "opt").
            other = other_side()
        inter = {k: (v[0].clone(), v[1].clone()) for k, v in best_int.items()}
        return final.detach(), other, inter

    @staticmethod
    def _update_best_alphas(st, best_alpha, improved_idx):
        """AlphaCROWNAnalysis::updateBestAlphas (src/engine/AlphaCROWNAnalysis.cpp:567-622):
        first call copies every alpha; later calls copy the rows whose index
        along the spec dimension is an improved output spec index (also for
        intermediate starts, where that dimension counts unstable neurons)."""
        with torch.no_grad():
            for key, ap in st.alphas.items():
                if ap.alpha.numel() == 0:
                    continue
                cur = ap.alpha.detach()
                if key not in best_alpha or best_alpha[key].shape != cur.shape:
                    best_alpha[key] = cur.clone()
                    continue
                idx = torch.as_tensor([i for i in improved_idx if i < cur.shape[1]], dtype=torch.long)
                if idx.numel():
                    best_alpha[key][:, idx] = cur[:, idx]

    def compute_property(self, lower, upper, C, thresholds, branches, n_branches, method):
        """Luna's CLI flow for each box [B, n_in] against one specification
        (C [nspec, n_out] with thresholds and OR branches): bounds with the
        early stops, and the CLI's verdict (LunaMain.cpp:60-135).  Returns
        lb, ub [B, nspec] and status [B] (0 unknown, 1 unsat, 2 sat)."""
        has_spec = np.size(thresholds) > 0  # without one: raw output bounds, verdict unknown
        spec = (torch.as_tensor(np.asarray(thresholds, np.float32)), np.asarray(branches), int(n_branches)) \
            if has_spec else None
        Ct = torch.from_numpy(np.ascontiguousarray(C, np.float32))
        B = lower.shape[0]
        lb = np.zeros((B, Ct.shape[0]), np.float32)
        ub = np.zeros((B, Ct.shape[0]), np.float32)
        status = np.zeros(B, np.int32)
        thr = np.asarray(thresholds, np.float32)
        for b in range(B):
            xl = torch.from_numpy(np.ascontiguousarray(lower[b]))
            xu = torch.from_numpy(np.ascontiguousarray(upper[b]))
            if method == METHOD_ALPHA_CROWN:
                lo, hi, _ = self.alpha_crown(xl, xu, Ct, spec=spec)
            else:
                lo, hi, _ = self.crown(xl, xu, Ct)
            lb[b], ub[b] = lo.numpy(), hi.numpy()
            if not has_spec:
                continue
            dl, du = lb[b] - thr > 0, ub[b] - thr <= 0
            if n_branches <= 0:
                status[b] = 1 if dl.any() else (2 if du.all() else 0)
            else:
                br = np.asarray(branches)
                rows = [br == k for k in range(n_branches)]
                if all(dl[r].any() for r in rows):
                    status[b] = 1
                elif any(r.any() and not (ub[b][r] - thr[r] > 0).any() for r in rows):
                    status[b] = 2
        return lb, ub, status

    def compute_bounds_warm(self, parents, children):
        """Branch-and-bound's warm start: for each i, alpha-CROWN on parent box
        i, then alpha-CROWN on child box i seeded with the parent's alphas
        (TorchModel::getState / loadState).  Intermediate bounds are not
        seeded: RECOMPUTE_INTERMEDIATE_BOUNDS (default true) recomputes them.
        C is taken from `children`.  Returns the children's lb, ub [B, nspec]."""
        B = children.n
        nspec = children.C.shape[1]
        lb = np.zeros((B, nspec), np.float32)
        ub = np.zeros((B, nspec), np.float32)
        for b in range(B):
            C = torch.from_numpy(children.C[0 if children.C.shape[0] == 1 else b].copy())
            self.alpha_crown(torch.from_numpy(parents.lower[b].copy()), torch.from_numpy(parents.upper[b].copy()), C)
            lo, hi, _ = self.alpha_crown(torch.from_numpy(children.lower[b].copy()),
                                         torch.from_numpy(children.upper[b].copy()), C, seed=self.last_alphas)
            lb[b] = lo.numpy()
            ub[b] = hi.numpy()
        return lb, ub

    def compute_bounds(self, boxes, method, intermediate=False):
        """Bound every box with a fresh state.  Returns lb, ub [B, nspec] (and
        the pre-activation bounds concatenated in node-id order)."""
        B = boxes.n
        nspec = boxes.C.shape[1]
        lb = np.zeros((B, nspec), np.float32)
        ub = np.zeros((B, nspec), np.float32)
        inter_l, inter_u = [], []
        for b in range(B):
            C = torch.from_numpy(boxes.C[0 if boxes.C.shape[0] == 1 else b].copy())
            xl = torch.from_numpy(boxes.lower[b].copy())
            xu = torch.from_numpy(boxes.upper[b].copy())
            if method == METHOD_IBP:
                lo, hi = self.ibp(xl, xu, C)
                inter = {}
            elif method == METHOD_CROWN:
                lo, hi, st = self.crown(xl, xu, C)
                inter = {i: st.node_bounds[i] for i in self.preact_ids if i in st.node_bounds}
            elif method == METHOD_ALPHA_CROWN:
                lo, hi, inter = self.alpha_crown(xl, xu, C)
            else:
                raise ValueError(method)
            lb[b] = lo.numpy()
            ub[b] = hi.numpy()
            if intermediate:
                inter_l.append(np.concatenate([inter[i][0].numpy() for i in self.preact_ids]))
                inter_u.append(np.concatenate([inter[i][1].numpy() for i in self.preact_ids]))
        if intermediate:
            return lb, ub, np.stack(inter_l), np.stack(inter_u)
        return lb, ub
