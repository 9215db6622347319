"""VNN-LIB properties over the engine's C ABI.

`Property(text, n_in, n_out)` reads a property the way Luna's
`TorchModel(onnxPath, vnnlibPath)` does
(src/engine/TorchModelOnnxFactory.cpp:89-192, with
src/input_parsers/VnnLibInputParser.cpp and OutputConstraint.cpp): the input
box over X_i, and the output constraints over Y_j as a specification matrix
C [nspec, n_out] with thresholds [nspec] (each row reads C.y <= threshold)
and, for a disjunction, the OR branch of each row.  `status(lb, ub)` is the
verdict Luna's CLI prints (src/engine/LunaMain.cpp:60-135).  Parsing and the
verdict are host logic in the C++ library; bounding is
`engine.Model.compute_property`.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import abi
from .abi import PropertyInfo, fptr
from .engine import _check, load_library


class Property:
    """A parsed VNN-LIB property for a network with n_in inputs and n_out outputs."""

    def __init__(self, text: str | bytes, n_in: int, n_out: int):
        lib = load_library()
        data = text.encode() if isinstance(text, str) else bytes(text)
        h = C.c_void_p()
        _check(lib.lb200_property_parse(data, len(data), int(n_in), int(n_out), C.byref(h)), "lb200_property_parse")
        self._h = h
        info = PropertyInfo()
        _check(lib.lb200_property_get_info(h, C.byref(info)), "lb200_property_get_info")
        self.n_in, self.n_out = int(info.n_in), int(info.n_out)
        self.nspec = int(info.nspec)
        self.n_branches = int(info.n_branches)
        self.spec_dropped = bool(info.spec_dropped)
        self.spec_error = info.spec_error.decode(errors="replace")
        self.lower = np.empty(self.n_in, np.float32)
        self.upper = np.empty(self.n_in, np.float32)
        _check(lib.lb200_property_input_box(h, fptr(self.lower), fptr(self.upper)), "lb200_property_input_box")
        self.C = np.zeros((self.nspec, self.n_out), np.float32)
        self.thresholds = np.zeros(self.nspec, np.float32)
        self.branches = np.zeros(self.nspec, np.int32)
        _check(lib.lb200_property_spec(h, fptr(self.C), fptr(self.thresholds),
                                       self.branches.ctypes.data_as(C.POINTER(C.c_int32))), "lb200_property_spec")

    @classmethod
    def from_file(cls, path: str | os.PathLike, n_in: int, n_out: int) -> "Property":
        with open(path, "rb") as f:
            return cls(f.read(), n_in, n_out)

    @property
    def handle(self):
        return self._h

    @property
    def has_spec(self) -> bool:
        return self.nspec > 0

    @property
    def has_or(self) -> bool:
        return self.n_branches > 0

    def status(self, lb, ub) -> np.ndarray:
        """Verdict per box from bounds [B, nspec] (or [nspec] for one box):
        abi.STATUS_UNSAT, STATUS_SAT or STATUS_UNKNOWN."""
        lb = np.ascontiguousarray(lb, np.float32)
        ub = np.ascontiguousarray(ub, np.float32)
        single = lb.ndim == 1
        lb2 = lb.reshape(-1, self.nspec) if self.nspec else lb.reshape(-1, max(lb.shape[-1], 1))
        ub2 = ub.reshape(lb2.shape)
        out = np.empty(lb2.shape[0], np.int32)
        if not self.has_spec:
            out[:] = abi.STATUS_UNKNOWN
        else:
            _check(load_library().lb200_property_status(
                fptr(lb2), fptr(ub2), lb2.shape[0], self.nspec, fptr(self.thresholds),
                self.branches.ctypes.data_as(C.POINTER(C.c_int32)), self.n_branches,
                out.ctypes.data_as(C.POINTER(C.c_int32))), "lb200_property_status")
        return out[0] if single else out

    def close(self):
        if getattr(self, "_h", None):
            load_library().lb200_property_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __repr__(self):
        kind = f"{self.n_branches} OR branches" if self.has_or else "a conjunction"
        return f"<Property n_in={self.n_in} n_out={self.n_out} nspec={self.nspec} ({kind})>"
