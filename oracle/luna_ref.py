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
