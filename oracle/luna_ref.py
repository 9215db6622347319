"""ctypes wrapper of oracle/_ref/libluna_ref.so -- test infrastructure.

The library is Luna's own CPU implementation compiled from the reference
sources by oracle/Makefile, plus oracle/luna_ref_driver.cpp.  It is the
ground truth for parity and the CPU baseline; only tests, smoke() and the
bench's CPU-baseline leg use it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from luna_b200.abi import GraphDesc, Options, default_options, fptr

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libluna_ref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def _load():
    global _lib
    if _lib is None:
        # libluna_ref.so links the venv's libtorch; loading it through torch's
        # own import initialises libtorch the way the reference expects (a
        # bare dlopen crashed inside exception handling of the reference's
        # best-effort centre forward pass).
        import torch  # noqa: F401
        if not available():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C oracle`")
        lib = C.CDLL(LIB_PATH)
        lib.luna_ref_intermediate_size.argtypes = [C.POINTER(GraphDesc)]
        lib.luna_ref_intermediate_size.restype = C.c_int64
        fp = C.POINTER(C.c_float)
        lib.luna_ref_compute_bounds.argtypes = [
            C.POINTER(GraphDesc), C.POINTER(Options), C.c_int, fp, fp, C.c_int64, C.c_int64,
            fp, C.c_int64, C.c_int64, C.c_int64, fp, fp, fp, fp, C.c_int, C.c_char_p, C.c_size_t]
        lib.luna_ref_compute_bounds.restype = C.c_int
        lib.luna_ref_compute_bounds_warm.argtypes = [
            C.POINTER(GraphDesc), C.POINTER(Options), fp, fp, fp, fp, C.c_int64, C.c_int64, fp, C.c_int64,
            C.c_int64, C.c_int64, fp, fp, C.c_int, C.c_char_p, C.c_size_t]
        lib.luna_ref_compute_bounds_warm.restype = C.c_int
        lib.luna_ref_compute_bounds_chain.argtypes = [
            C.POINTER(GraphDesc), C.POINTER(Options), fp, fp, C.c_int64, C.c_int64, C.c_int64, fp, C.c_int64,
            C.c_int64, C.c_int64, fp, fp, C.c_int, C.c_char_p, C.c_size_t]
        lib.luna_ref_compute_bounds_chain.restype = C.c_int
        ip = C.POINTER(C.c_int32)
        lib.luna_ref_property_status.argtypes = [fp, fp, C.c_int64, C.c_int64, fp, ip, C.c_int32, ip, C.c_char_p,
                                                 C.c_size_t]
        lib.luna_ref_compute_property.argtypes = [
            C.POINTER(GraphDesc), C.POINTER(Options), C.c_int, fp, fp, ip, C.c_int64, C.c_int32, fp, fp, C.c_int64,
            C.c_int64, C.c_int64, fp, fp, ip, C.c_int, C.c_char_p, C.c_size_t]
        _lib = lib
    return _lib


def compute_bounds(graph, boxes, method: int, options: Options | None = None,
                   intermediate: bool = False, num_threads: int = 1):
    """Run Luna on every box (fresh model per box).  Returns (lb, ub) of shape
    [B, nspec], plus (inter_lb, inter_ub) [B, n_inter] when `intermediate`."""
    lib = _load()
    opt = options if options is not None else default_options()
    desc = graph.desc()
    B, n_in = boxes.lower.shape
    Cm = np.ascontiguousarray(boxes.C, np.float32)
    nspec, n_out = Cm.shape[1], Cm.shape[2]
    lb = np.zeros((B, nspec), np.float32)
    ub = np.zeros((B, nspec), np.float32)
    n_int = lib.luna_ref_intermediate_size(C.byref(desc))
    il = np.zeros((B, max(n_int, 1)), np.float32) if intermediate else None
    iu = np.zeros((B, max(n_int, 1)), np.float32) if intermediate else None
    err = C.create_string_buffer(4096)
    xl = np.ascontiguousarray(boxes.lower, np.float32)
    xu = np.ascontiguousarray(boxes.upper, np.float32)
    rc = lib.luna_ref_compute_bounds(C.byref(desc), C.byref(opt), method, fptr(xl), fptr(xu), B,
                                     n_in, fptr(Cm), Cm.shape[0], nspec, n_out, fptr(lb), fptr(ub),
                                     fptr(il), fptr(iu), num_threads, err, len(err))
    if rc != 0:
        raise RuntimeError("luna reference failed: " + err.value.decode(errors="replace"))
    if intermediate:
        return lb, ub, il[:, :n_int], iu[:, :n_int]
    return lb, ub


def compute_bounds_warm(graph, parents, children, options: Options | None = None, num_threads: int = 1):
    """Luna's warm start: child i bounded with alpha-CROWN after loading the
    state (TorchModel::getState / loadState) its parent box parents[i] left.
    C is taken from `children`.  Returns the children's (lb, ub) [B, nspec]."""
    lib = _load()
    opt = options if options is not None else default_options()
    desc = graph.desc()
    B, n_in = children.lower.shape
    if parents.lower.shape != (B, n_in):
        raise ValueError("one parent box per child")
    Cm = np.ascontiguousarray(children.C, np.float32)
    nspec, n_out = Cm.shape[1], Cm.shape[2]
    lb = np.zeros((B, nspec), np.float32)
    ub = np.zeros((B, nspec), np.float32)
    arrs = [np.ascontiguousarray(a, np.float32)
            for a in (parents.lower, parents.upper, children.lower, children.upper)]
    err = C.create_string_buffer(4096)
    rc = lib.luna_ref_compute_bounds_warm(C.byref(desc), C.byref(opt), *(fptr(a) for a in arrs), B, n_in,
                                          fptr(Cm), Cm.shape[0], nspec, n_out, fptr(lb), fptr(ub), num_threads,
                                          err, len(err))
    if rc != 0:
        raise RuntimeError("luna reference failed: " + err.value.decode(errors="replace"))
    return lb, ub


def compute_bounds_chain(graph, lower, upper, spec, options: Options | None = None, num_threads: int = 1):
    """Luna down split-tree paths: lower / upper [n_paths, depth, n_in] (root
    first), spec [1 or n_paths, nspec, n_out]; the root of each path is bounded
    fresh with alpha-CROWN and every later box after getState / loadState of
    the box above.  Returns (lb, ub) [n_paths, depth, nspec]."""
    lib = _load()
    opt = options if options is not None else default_options()
    desc = graph.desc()
    P, D, n_in = lower.shape
    Cm = np.ascontiguousarray(spec, np.float32)
    nspec, n_out = Cm.shape[1], Cm.shape[2]
    lb = np.zeros((P, D, nspec), np.float32)
    ub = np.zeros((P, D, nspec), np.float32)
    lo = np.ascontiguousarray(lower, np.float32)
    hi = np.ascontiguousarray(upper, np.float32)
    err = C.create_string_buffer(4096)
    rc = lib.luna_ref_compute_bounds_chain(C.byref(desc), C.byref(opt), fptr(lo), fptr(hi), P, D, n_in, fptr(Cm),
                                           Cm.shape[0], nspec, n_out, fptr(lb), fptr(ub), num_threads, err, len(err))
    if rc != 0:
        raise RuntimeError("luna reference failed: " + err.value.decode(errors="replace"))
    return lb, ub


def _ip(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


PARSE_BIN = os.path.join(_HERE, "_ref", "luna_ref_vnnlib")


def _parsed(r: dict, n_out: int):
    if r["rc"] == 2:
        return ValueError(r["error"])
    if r["rc"] != 0:
        raise RuntimeError("luna reference failed: " + r["error"])
    f32 = lambda xs: np.array([float.fromhex(x) for x in xs], np.float32)
    k = r["nspec"]
    return {"lower": f32(r["lower"]), "upper": f32(r["upper"]), "C": f32(r["C"]).reshape(k, n_out),
            "thresholds": f32(r["thresholds"]), "branches": np.array(r["branches"], np.int32).reshape(k),
            "n_branches": r["n_branches"], "spec_dropped": bool(r["spec_dropped"]),
            "error": r["error"] if r["spec_dropped"] else ""}


def vnnlib_parse_many(cases) -> list:
    """Luna's reading of each (text, n_in, n_out), run as its own process
    (oracle/luna_ref_vnnlib.cpp): per case a dict with lower, upper, C,
    thresholds, branches, n_branches, spec_dropped, error -- or a ValueError
    instance when the input bounds fail to parse."""
    import json
    import shutil
    import subprocess
    import tempfile
    if not os.path.exists(PARSE_BIN):
        raise RuntimeError(f"{PARSE_BIN} is missing: build it with `make -C oracle`")
    tmp = tempfile.mkdtemp(prefix="luna_vnnlib_")
    try:
        args = [PARSE_BIN]
        for k, (text, n_in, n_out) in enumerate(cases):
            path = os.path.join(tmp, f"p{k}.vnnlib")
            with open(path, "wb") as f:
                f.write(text.encode() if isinstance(text, str) else bytes(text))
            args += [path, str(n_in), str(n_out)]
        out = subprocess.run(args, capture_output=True, check=True, timeout=600)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    lines = out.stdout.decode().splitlines()
    if len(lines) != len(cases):
        raise RuntimeError(f"luna_ref_vnnlib printed {len(lines)} results for {len(cases)} properties")
    return [_parsed(json.loads(l), n_out) for l, (_, _, n_out) in zip(lines, cases)]


def vnnlib_parse(text, n_in: int, n_out: int) -> dict:
    """Luna's reading of one property; raises ValueError when the input
    bounds fail to parse."""
    r = vnnlib_parse_many([(text, n_in, n_out)])[0]
    if isinstance(r, ValueError):
        raise r
    return r


def property_status(lb, ub, thresholds, branches, n_branches: int) -> np.ndarray:
    """Luna's verdict per box for bounds [B, nspec]."""
    lib = _load()
    lb = np.ascontiguousarray(lb, np.float32)
    ub = np.ascontiguousarray(ub, np.float32)
    thr = np.ascontiguousarray(thresholds, np.float32)
    br = np.ascontiguousarray(branches, np.int32)
    out = np.zeros(lb.shape[0], np.int32)
    err = C.create_string_buffer(4096)
    rc = lib.luna_ref_property_status(fptr(lb), fptr(ub), lb.shape[0], lb.shape[1], fptr(thr), _ip(br), n_branches,
                                      _ip(out), err, len(err))
    if rc != 0:
        raise RuntimeError("luna reference failed: " + err.value.decode(errors="replace"))
    return out


def compute_property(graph, spec: dict, lower, upper, method: int, options: Options | None = None,
                     num_threads: int = 1):
    """Luna's CLI flow for each box [B, n_in] against a property read by
    `vnnlib_parse` (its C, thresholds and branches): returns (lb, ub, status)."""
    lib = _load()
    opt = options if options is not None else default_options()
    desc = graph.desc()
    xl = np.ascontiguousarray(lower, np.float32)
    xu = np.ascontiguousarray(upper, np.float32)
    B, n_in = xl.shape
    n_out = int(np.prod(graph.nodes[graph.output_index].out_shape))
    Cm = np.ascontiguousarray(spec["C"], np.float32).reshape(-1, n_out)
    thr = np.ascontiguousarray(spec["thresholds"], np.float32)
    br = np.ascontiguousarray(spec["branches"], np.int32)
    nspec = Cm.shape[0]
    rows = nspec or n_out
    lb = np.zeros((B, rows), np.float32)
    ub = np.zeros((B, rows), np.float32)
    st = np.zeros(B, np.int32)
    err = C.create_string_buffer(4096)
    rc = lib.luna_ref_compute_property(C.byref(desc), C.byref(opt), method, fptr(Cm), fptr(thr), _ip(br), nspec,
                                       int(spec["n_branches"]), fptr(xl), fptr(xu), B, n_in, n_out, fptr(lb),
                                       fptr(ub), _ip(st), num_threads, err, len(err))
    if rc != 0:
        raise RuntimeError("luna reference failed: " + err.value.decode(errors="replace"))
    return lb, ub, st
