"""The Luna-side shim (oracle/luna_b200_shim.h): graphs built twice from the
same torch modules -- as Luna's own nodes (NLR::TorchModel, its CPU path) and
as the shim's (lb200_luna::TorchModel, the engine behind the C ABI) -- must
give the same bounds through TorchModel::compute_bounds
(src/engine/TorchModel.cpp:653-698), box by box, at the parity bar."""
import ctypes as C
import os

import numpy as np
import pytest

import golden_cases as G
from luna_b200 import abi, workloads as W
from luna_b200.abi import GraphDesc, Options, fptr

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "libluna_shim_check.so")


@pytest.fixture(scope="module")
def shim():
    import torch  # noqa: F401  (loads LibTorch before Luna's library)
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available()
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is missing: build it with `make -C oracle`")
    lib = C.CDLL(LIB)
    fp = C.POINTER(C.c_float)
    lib.luna_shim_check.argtypes = [C.POINTER(GraphDesc), C.POINTER(Options), C.c_int, fp, fp, C.c_int64, fp,
                                    C.c_int64, C.c_int64, C.c_int, fp, fp, fp, fp, C.c_char_p, C.c_size_t]
    lib.luna_shim_check.restype = C.c_int
    return lib


def _run(lib, g, bx, b, method, opt):
    desc = g.desc()
    n_in = bx.lower.shape[1]
    Cm = np.ascontiguousarray(bx.C[0 if bx.C.shape[0] == 1 else b], np.float32)
    nspec, n_out = Cm.shape
    out = [np.zeros(nspec, np.float32) for _ in range(4)]
    err = C.create_string_buffer(4096)
    xl = np.ascontiguousarray(bx.lower[b])
    xu = np.ascontiguousarray(bx.upper[b])
    rc = lib.luna_shim_check(C.byref(desc), C.byref(opt), method, fptr(xl), fptr(xu), n_in, fptr(Cm), nspec, n_out,
                             0, *[fptr(o) for o in out], err, len(err))
    assert rc == 0, err.value.decode()
    return out


CASES = [
    ("mlp5", lambda: W.mlp_5_50x6_5(2), 0.1, 5),
    ("mlp784", lambda: W.mlp_784_256x4_10(1), 0.1, 5),
    ("cnn_dense", lambda: W.small_cnn_case(3, n_boxes=1, big_first=False), 0.1, 4),
    ("cnn_patch", lambda: W.small_cnn_case(5, n_boxes=1, big_first=True), 0.1, 3),
    ("cnnbn", lambda: W.small_cnn_bn_case(4, n_boxes=1, big_first=False), 0.1, 3),
    ("convt", lambda: W.convt_cnn_case(1, n_boxes=1), 0.1, 3),
    ("resnet", lambda: W.small_resnet_case(7, n_boxes=1), 0.1, 3),
    ("resnet_sigmoid", lambda: W.small_resnet_case(9, n_boxes=1, head_act=abi.NODE_SIGMOID), 0.1, 0),
    ("sub_input", lambda: W.sub_mlp_case(1, n_boxes=2), 0.1, 4),
    ("slice", lambda: W.slice_mlp_case(6, n_boxes=2, reverse=True), 0.1, 4),
    ("concat_cnn", lambda: W.concat_cnn_case(8, n_boxes=1), 0.1, 3),
    ("sub_cnn", lambda: W.sub_cnn_case(10, n_boxes=1, constant_second=0), 0.1, 3),
]


@pytest.mark.parametrize("name,make,lr,iters", CASES, ids=[c[0] for c in CASES])
def test_shim_matches_luna(shim, name, make, lr, iters):
    g, bx = make()
    methods = [abi.METHOD_CROWN] + ([abi.METHOD_ALPHA_CROWN] if iters else [])
    for method in methods:
        opt = abi.default_options(alpha_lr=lr, alpha_iterations=max(iters, 1))
        for b in range(bx.n):
            llb, lub, slb, sub = _run(shim, g, bx, b, method, opt)
            G.parity(f"shim/{name}/{method}/box{b}", slb, sub, llb, lub)
