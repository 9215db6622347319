"""The Luna-side shim (oracle/luna_b200_shim.h): graphs built from the same
torch modules as Luna's own nodes (NLR::TorchModel, its CPU path) and as the
shim's (lb200_luna::TorchModel, the engine behind the C ABI) must give the
same bounds through TorchModel::compute_bounds (src/engine/TorchModel.cpp:653-698),
box by box, at the parity bar.

Luna's CPU path chooses the patches form for every conv start when CUDA is
available to its process (CROWNAnalysis.cpp:261-271), so its side runs in a
child process with CUDA hidden, as Luna's CPU baseline does; the shim's side
runs in this process on the GPU."""
import ctypes as C
import multiprocessing as mp
import os

import numpy as np
import pytest

import golden_cases as G
from luna_b200 import abi, workloads as W

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libluna_shim_check.so")

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


def _load(lib_path):
    from luna_b200.abi import GraphDesc, Options
    lib = C.CDLL(lib_path)
    fp = C.POINTER(C.c_float)
    lib.luna_shim_check.argtypes = [C.POINTER(GraphDesc), C.POINTER(Options), C.c_int, fp, fp, C.c_int64, fp,
                                    C.c_int64, C.c_int64, C.c_int, C.c_int, fp, fp, fp, fp, C.c_char_p, C.c_size_t]
    lib.luna_shim_check.restype = C.c_int
    return lib


def _jobs():
    """(case, method, box, lr, iters) for every bound the test compares."""
    out = []
    for name, make, lr, iters in CASES:
        g, bx = make()
        for method in [abi.METHOD_CROWN] + ([abi.METHOD_ALPHA_CROWN] if iters else []):
            for b in range(bx.n):
                out.append((name, method, b, lr, max(iters, 1)))
    return out


def _run(lib, which, name, method, b, lr, iters):
    from luna_b200.abi import fptr
    make = dict((c[0], c[1]) for c in CASES)[name]
    g, bx = make()
    desc = g.desc()
    opt = abi.default_options(alpha_lr=lr, alpha_iterations=iters)
    Cm = np.ascontiguousarray(bx.C[0 if bx.C.shape[0] == 1 else b], np.float32)
    nspec, n_out = Cm.shape
    out = [np.zeros(nspec, np.float32) for _ in range(4)]
    err = C.create_string_buffer(4096)
    xl = np.ascontiguousarray(bx.lower[b])
    xu = np.ascontiguousarray(bx.upper[b])
    rc = lib.luna_shim_check(C.byref(desc), C.byref(opt), method, fptr(xl), fptr(xu), xl.size, fptr(Cm), nspec,
                             n_out, 0, which, *[fptr(o) for o in out], err, len(err))
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return out[:2] if which == 1 else out[2:]


def _luna_child(q):
    """Luna's side of every job, in a process where CUDA is hidden."""
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    import torch  # noqa: F401  (LibTorch before Luna's library)
    lib = _load(LIB)
    q.put([_run(lib, 1, *job) for job in _jobs()])


@pytest.fixture(scope="module")
def luna_results():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is missing: build it with `make -C oracle`")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_luna_child, args=(q,))
    p.start()
    res = q.get(timeout=900)
    p.join(timeout=60)
    return dict(zip(_jobs(), res))


@pytest.fixture(scope="module")
def shim():
    import torch
    from luna_b200.build import build
    build()
    assert torch.cuda.is_available()
    return _load(LIB)


@pytest.mark.parametrize("case", [c[0] for c in CASES])
def test_shim_matches_luna(shim, luna_results, case):
    for job in _jobs():
        if job[0] != case:
            continue
        slb, sub = _run(shim, 2, *job)
        llb, lub = luna_results[job]
        G.parity(f"shim/{case}/{job[1]}/box{job[2]}", slb, sub, llb, lub)
