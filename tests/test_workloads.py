"""Seeded workload generators (CPU): the sub-domain split of a box."""
import numpy as np

from luna_b200 import workloads as W


def test_subdomains_tile_the_box():
    g, _ = W.small_cnn_case(3, n_boxes=1, big_first=False)
    sp = W.subdomain_split(g, 11, 0.05, n_groups=3, group_size=2, n_in_shape=(3, 10, 10))
    assert sp.count == 8 and sp.groups.shape == (3, 2)
    assert len(np.unique(sp.groups)) == 6
    bx = sp.boxes(0, sp.count)
    # Every sub-domain lies in the box and differs from it only on grouped pixels.
    assert (bx.lower >= sp.lower).all() and (bx.upper <= sp.upper).all()
    other = np.setdiff1d(np.arange(sp.lower.size), sp.groups.ravel())
    assert (bx.lower[:, other] == sp.lower[other]).all() and (bx.upper[:, other] == sp.upper[other]).all()
    # All sub-domains differ; bit g of the id picks the half of group g.
    mid = (sp.lower + sp.upper) / np.float32(2)
    assert len({(tuple(l), tuple(u)) for l, u in zip(bx.lower, bx.upper)}) == sp.count
    for sid in range(sp.count):
        for grp in range(3):
            idx = sp.groups[grp]
            upper_half = (sid >> grp) & 1
            assert (bx.lower[sid, idx] == (mid[idx] if upper_half else sp.lower[idx])).all()


def test_widest_gradient_pixels_rank_first():
    g, _ = W.small_cnn_case(4, n_boxes=1, big_first=False)
    sp = W.subdomain_split(g, 12, 0.05, n_groups=2, group_size=3, n_in_shape=(3, 10, 10))
    import torch
    x = torch.from_numpy(sp.centre[None]).requires_grad_(True)
    # The chosen pixels carry the largest |gradient| * width at the centre.
    assert sp.groups.size == 6
    y = W.graph_forward(g, x)
    (y @ torch.from_numpy(sp.C[0]).T).sum().backward()
    score = np.abs(x.grad.numpy()[0]) * (sp.upper - sp.lower)
    chosen = score[sp.groups.ravel()]
    rest = np.delete(score, sp.groups.ravel())
    assert chosen.min() >= rest.max() - 1e-6


def test_property_workload_split():
    """The property workload: 512 sub-domains inside the property's box, the
    property's label the network's prediction at the centre, and the text
    reads back as that box with 9 OR branches."""
    import torch

    from luna_b200.vnnlib import Property
    g, split, text = W.mlp_property_split()
    bx = split.boxes(0, 512)
    assert bx.n == 512
    assert (bx.lower >= split.lower).all() and (bx.upper <= split.upper).all()
    assert (bx.lower <= bx.upper).all()
    t = int(W.graph_forward(g, torch.from_numpy(split.centre[None])).argmax())
    assert (split.C[0][:, t] == 1).all()
    p = Property(text, 784, 10)
    assert p.n_branches == 9 and p.nspec == 9
    assert (p.lower == split.lower).all() and (p.upper == split.upper).all()
    assert (p.C == split.C[0]).all() and (p.thresholds == 0).all()
