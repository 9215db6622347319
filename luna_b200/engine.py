"""Python binding of the engine's C ABI (include/luna_b200.h) via ctypes.

This mirrors Luna's TorchModel entry point for the bound-propagation path:
`Model(graph)` replaces `TorchModel(nodes, inputIndices, outputIndex,
dependencies)` (src/engine/TorchModel.h:47-50) and `Model.compute_bounds`
replaces `TorchModel::compute_bounds` (src/engine/TorchModel.cpp:653-698),
bounding a whole batch of boxes per call.  Errors raise `EngineError` with the
engine's message, as Luna raises exceptions.  There is no CPU fallback: the
CUDA library must be present and a GPU visible.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .abi import GraphDesc, Options, PropertyInfo, Stats, default_options, fptr

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libluna_b200.so")

EXPORTS = ("lb200_options_default", "lb200_model_create", "lb200_set_options",
           "lb200_compute_bounds", "lb200_compute_bounds_device",
           "lb200_get_intermediate_bounds", "lb200_last_error", "lb200_model_destroy",
           "lb200_set_profiling", "lb200_set_contraction_path", "lb200_ibp_bounds_noalloc",
           "lb200_shard_range", "lb200_nccl_unique_id", "lb200_nccl_comm_create", "lb200_nccl_comm_destroy",
           "lb200_shard_run", "lb200_describe_plan", "lb200_property_parse", "lb200_property_get_info",
           "lb200_property_input_box", "lb200_property_spec", "lb200_property_free", "lb200_property_status",
           "lb200_property_status_device", "lb200_compute_property", "lb200_compute_property_device",
           "lb200_test_set_contraction_fault", "lb200_set_warm_start", "lb200_set_warm_parents",
           "lb200_warm_alpha")


class EngineError(RuntimeError):
    pass


_lib = None


def load_library():
    """Load libluna_b200.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise EngineError(f"{LIB_PATH} not built (python -m luna_b200.build)")
    lib = C.CDLL(LIB_PATH)
    fp = C.POINTER(C.c_float)
    vp = C.c_void_p
    lib.lb200_options_default.argtypes = [C.POINTER(Options)]
    lib.lb200_model_create.argtypes = [C.POINTER(GraphDesc), C.c_int, C.POINTER(vp)]
    lib.lb200_set_options.argtypes = [vp, C.POINTER(Options)]
    lib.lb200_compute_bounds.argtypes = [vp, C.c_int, fp, fp, C.c_int64, fp, C.c_int64, C.c_int64,
                                         fp, C.c_int, C.c_int, fp, fp, C.POINTER(Stats)]
    lib.lb200_compute_bounds_device.argtypes = [vp, C.c_int, vp, vp, C.c_int64, vp, C.c_int64,
                                                C.c_int64, vp, C.c_int, C.c_int, vp, vp, vp,
                                                C.POINTER(Stats)]
    lib.lb200_get_intermediate_bounds.argtypes = [vp, fp, fp, C.POINTER(C.c_int64)]
    lib.lb200_last_error.argtypes = [C.c_char_p, C.c_size_t]
    lib.lb200_set_profiling.argtypes = [vp, C.c_int]
    lib.lb200_set_contraction_path.argtypes = [vp, C.c_int]
    lib.lb200_set_warm_start.argtypes = [vp, C.c_int]
    lib.lb200_set_warm_parents.argtypes = [vp, C.POINTER(C.c_int64), C.c_int64]
    lib.lb200_warm_alpha.argtypes = [vp, C.c_int, C.c_int, C.c_int64, fp, C.c_int64, C.POINTER(C.c_int64),
                                     C.POINTER(C.c_int64), C.POINTER(C.c_uint8)]
    lib.lb200_ibp_bounds_noalloc.argtypes = [vp, vp, vp, C.c_int64, vp, C.c_int64, C.c_int64, vp, vp, vp]
    lib.lb200_model_destroy.argtypes = [vp]
    lib.lb200_model_destroy.restype = None
    u8p = C.POINTER(C.c_uint8)
    lib.lb200_shard_range.argtypes = [C.c_int, C.c_int, C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]
    lib.lb200_nccl_unique_id.argtypes = [u8p]
    lib.lb200_nccl_comm_create.argtypes = [u8p, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    lib.lb200_nccl_comm_destroy.argtypes = [vp]
    lib.lb200_shard_run.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, fp, fp, C.c_int64, fp, C.c_int64,
                                    C.c_int64, fp, fp, C.c_int, C.POINTER(Stats)]
    lib.lb200_test_set_contraction_fault.argtypes = [C.c_int, C.c_int, C.c_int64]
    lib.lb200_describe_plan.argtypes = [C.POINTER(GraphDesc), C.POINTER(Options), C.c_char_p, C.c_size_t,
                                        C.POINTER(C.c_size_t)]
    ip = C.POINTER(C.c_int32)
    lib.lb200_property_parse.argtypes = [C.c_char_p, C.c_int64, C.c_int64, C.c_int64, C.POINTER(vp)]
    lib.lb200_property_get_info.argtypes = [vp, C.POINTER(PropertyInfo)]
    lib.lb200_property_input_box.argtypes = [vp, fp, fp]
    lib.lb200_property_spec.argtypes = [vp, fp, fp, ip]
    lib.lb200_property_free.argtypes = [vp]
    lib.lb200_property_free.restype = None
    lib.lb200_property_status.argtypes = [fp, fp, C.c_int64, C.c_int64, fp, ip, C.c_int32, ip]
    lib.lb200_property_status_device.argtypes = [vp, vp, C.c_int64, C.c_int64, vp, vp, C.c_int32, vp, vp]
    lib.lb200_compute_property.argtypes = [vp, C.c_int, vp, fp, fp, C.c_int64, fp, fp, ip, C.POINTER(Stats)]
    lib.lb200_compute_property_device.argtypes = [vp, C.c_int, vp, vp, vp, C.c_int64, vp, vp, vp, vp,
                                                  C.POINTER(Stats)]
    _lib = lib
    return lib


def set_contraction_fault(device: int, starve: bool, wait_cycles: int = 0) -> None:
    """Failure-detection test hook (lb200_test_set_contraction_fault): with
    starve the tensor-core kernels' bounded waits run out on `device`."""
    load_library()
    _check(_lib.lb200_test_set_contraction_fault(device, 1 if starve else 0, wait_cycles),
           "lb200_test_set_contraction_fault", "lb200_set_warm_start", "lb200_set_warm_parents",
           "lb200_warm_alpha")


def last_error() -> str:
    """The calling thread's lb200_last_error() text."""
    load_library()
    buf = C.create_string_buffer(4096)
    _lib.lb200_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _check(rc: int, what: str):
    if rc != 0:
        buf = C.create_string_buffer(4096)
        _lib.lb200_last_error(buf, len(buf))
        raise EngineError(f"{what}: {buf.value.decode(errors='replace')}")


def describe_plan(graph, options: Options | None = None) -> dict:
    """The engine's plan for `graph` (lb200_describe_plan, host only): levels
    and, per backward start, its concretisation form and row windows."""
    import json
    load_library()
    desc = graph.desc()
    opt = options if options is not None else default_options()
    need = C.c_size_t()
    _check(_lib.lb200_describe_plan(C.byref(desc), C.byref(opt), None, 0, C.byref(need)), "lb200_describe_plan")
    buf = C.create_string_buffer(need.value)
    _check(_lib.lb200_describe_plan(C.byref(desc), C.byref(opt), buf, need.value, C.byref(need)),
           "lb200_describe_plan")
    return json.loads(buf.value.decode())


def shard_range(rank: int, world: int, n: int) -> tuple[int, int]:
    """[begin, end) of n boxes for `rank` (lb200_shard_range)."""
    load_library()
    a, b = C.c_int64(), C.c_int64()
    _check(_lib.lb200_shard_range(rank, world, n, C.byref(a), C.byref(b)), "lb200_shard_range")
    return a.value, b.value


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id, to be shared with every rank."""
    load_library()
    buf = (C.c_uint8 * 128)()
    _check(_lib.lb200_nccl_unique_id(buf), "lb200_nccl_unique_id")
    return bytes(buf)


class NcclComm:
    """An NCCL communicator over `world` ranks made by the engine library
    (lb200_nccl_comm_create); blocks until every rank has joined."""

    def __init__(self, uid: bytes, rank: int, world: int, device: int):
        load_library()
        if len(uid) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = C.c_void_p()
        _check(_lib.lb200_nccl_comm_create(buf, rank, world, device, C.byref(h)), "lb200_nccl_comm_create")
        self.handle, self.rank, self.world = h, rank, world

    def close(self):
        if self.handle:
            _check(_lib.lb200_nccl_comm_destroy(self.handle), "lb200_nccl_comm_destroy")
            self.handle = None


class Model:
    """One network on one GPU."""

    def __init__(self, graph, device: int = 0, options: Options | None = None):
        lib = load_library()
        self.graph = graph
        self._desc = graph.desc()
        h = C.c_void_p()
        _check(lib.lb200_model_create(C.byref(self._desc), device, C.byref(h)), "lb200_model_create")
        self._h = h
        self.options = options if options is not None else default_options()
        self.set_options(self.options)
        self.last_stats = Stats()

    def set_options(self, options: Options):
        self.options = options
        _check(_lib.lb200_set_options(self._h, C.byref(options)), "lb200_set_options")

    def set_profiling(self, on: bool):
        """Time the A.W contraction kernels with CUDA events (stats.ms_contractions)."""
        _check(_lib.lb200_set_profiling(self._h, int(on)), "lb200_set_profiling")

    def set_contraction_path(self, path: int):
        """0: tensor cores (3xTF32) where the shape allows, 224-column tiles on
        CTA pairs for wide N, split cross-term accumulation in the adjoint
        contractions; 1: SIMT fp32 only; 2: tensor cores on single CTAs;
        3: tensor-core forward, SIMT adjoint contractions; 4: as 0 without the
        split accumulation; 5: as 0 with it in the forward contractions too."""
        _check(_lib.lb200_set_contraction_path(self._h, int(path)), "lb200_set_contraction_path")

    def set_warm_start(self, keep: bool):
        """Retain every later alpha-CROWN call's final alphas (TorchModel::getState)
        for warm-starting the boxes of a following call; False drops them."""
        _check(_lib.lb200_set_warm_start(self._h, int(keep)), "lb200_set_warm_start")

    def set_warm_parents(self, parent):
        """The next call's box b starts from retained box parent[b]
        (TorchModel::loadState); -1 bounds it afresh."""
        p = np.ascontiguousarray(np.asarray(parent, np.int64).reshape(-1))
        _check(_lib.lb200_set_warm_parents(self._h, p.ctypes.data_as(C.POINTER(C.c_int64)), p.size),
               "lb200_set_warm_parents")

    def warm_alpha(self, level: int, start: int, box: int):
        """Retained alphas of one box (the alpha part of TorchModel::getState):
        ([2, rows, cols] fp32, creation set [cols] bool) for activation
        `level` and start `start` (lb200_warm_alpha)."""
        rows, cols = C.c_int64(), C.c_int64()
        _check(_lib.lb200_warm_alpha(self._h, int(level), int(start), int(box), None, 0, C.byref(rows),
                                     C.byref(cols), None), "lb200_warm_alpha")
        out = np.zeros((2, rows.value, cols.value), np.float32)
        aset = np.zeros(cols.value, np.uint8)
        _check(_lib.lb200_warm_alpha(self._h, int(level), int(start), int(box),
                                     out.ctypes.data_as(C.POINTER(C.c_float)), out.size, C.byref(rows),
                                     C.byref(cols), aset.ctypes.data_as(C.POINTER(C.c_uint8))), "lb200_warm_alpha")
        return out, aset.astype(bool)

    def compute_bounds(self, boxes, method: int, bound_lower: bool = True, bound_upper: bool = True,
                       out_lb: np.ndarray | None = None, out_ub: np.ndarray | None = None,
                       thresholds: np.ndarray | None = None):
        """Bound every box from host arrays; returns (lb, ub) as [B, nspec] fp32.
        With `thresholds` [nspec] a box is verified once some row's lower bound
        exceeds its threshold, and the STOP_*_ON_VERIFIED options apply."""
        xl = np.ascontiguousarray(boxes.lower, np.float32)
        xu = np.ascontiguousarray(boxes.upper, np.float32)
        Cm = np.ascontiguousarray(boxes.C, np.float32)
        B, nspec = xl.shape[0], Cm.shape[1]
        thr = None if thresholds is None else np.ascontiguousarray(thresholds, np.float32).reshape(nspec)
        lb = out_lb if out_lb is not None else np.empty((B, nspec), np.float32)
        ub = out_ub if out_ub is not None else np.empty((B, nspec), np.float32)
        st = Stats()
        _check(_lib.lb200_compute_bounds(self._h, method, fptr(xl), fptr(xu), B, fptr(Cm), Cm.shape[0],
                                         nspec, fptr(thr), int(bound_lower), int(bound_upper),
                                         fptr(lb), fptr(ub), C.byref(st)), "lb200_compute_bounds")
        self.last_stats = st
        return lb, ub

    def compute_property(self, prop, method: int, lower: np.ndarray | None = None,
                         upper: np.ndarray | None = None):
        """Bound boxes against a `vnnlib.Property` (lb200_compute_property):
        the property's own input box when `lower`/`upper` are None, else the
        boxes [B, n_in].  Returns (lb, ub, status) with lb, ub [B, rows] and
        status [B] (abi.STATUS_*)."""
        if (lower is None) != (upper is None):
            raise ValueError("give both lower and upper, or neither")
        if lower is None:
            B, xl, xu = 1, None, None
        else:
            xl = np.ascontiguousarray(lower, np.float32).reshape(-1, prop.n_in)
            xu = np.ascontiguousarray(upper, np.float32).reshape(-1, prop.n_in)
            B = xl.shape[0]
        rows = prop.nspec if prop.nspec > 0 else prop.n_out
        lb = np.empty((B, rows), np.float32)
        ub = np.empty((B, rows), np.float32)
        status = np.empty(B, np.int32)
        st = Stats()
        _check(_lib.lb200_compute_property(self._h, method, prop.handle, fptr(xl), fptr(xu), B, fptr(lb), fptr(ub),
                                           status.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(st)),
               "lb200_compute_property")
        self.last_stats = st
        return lb, ub, status

    def compute_property_ptr(self, prop, method: int, xl: int, xu: int, n_boxes: int, lb: int, ub: int,
                             status: int = 0, stream: int = 0):
        """Device-pointer variant of compute_property (pointers as ints, e.g.
        torch data_ptr()); status may be 0 (no verdicts)."""
        st = Stats()
        _check(_lib.lb200_compute_property_device(self._h, method, prop.handle, xl, xu, n_boxes, lb, ub,
                                                  status or None, stream or None, C.byref(st)),
               "lb200_compute_property_device")
        self.last_stats = st
        return st

    def shard_run(self, comm: NcclComm, boxes, method: int, timeout_ms: int = 60000):
        """Bound this rank's share of `boxes` and all-gather every rank's
        bounds over `comm` (lb200_shard_run); returns (lb, ub) [B, nspec] for
        the whole batch on every rank."""
        xl = np.ascontiguousarray(boxes.lower, np.float32)
        xu = np.ascontiguousarray(boxes.upper, np.float32)
        Cm = np.ascontiguousarray(boxes.C, np.float32)
        B, nspec = xl.shape[0], Cm.shape[1]
        lb = np.empty((B, nspec), np.float32)
        ub = np.empty((B, nspec), np.float32)
        st = Stats()
        rc = _lib.lb200_shard_run(self._h, comm.handle, comm.rank, comm.world, method, fptr(xl), fptr(xu), B,
                                  fptr(Cm), Cm.shape[0], nspec, fptr(lb), fptr(ub), timeout_ms, C.byref(st))
        if rc != 0 and "aborted" in last_error():
            comm.handle = None  # ncclCommAbort released it
        _check(rc, "lb200_shard_run")
        self.last_stats = st
        return lb, ub

    def compute_bounds_ptr(self, method: int, xl: int, xu: int, n_boxes: int, Cp: int, c_boxes: int,
                           nspec: int, lb: int, ub: int, stream: int = 0):
        """Device-pointer variant (pointers as ints, e.g. torch data_ptr())."""
        st = Stats()
        _check(_lib.lb200_compute_bounds_device(self._h, method, xl, xu, n_boxes, Cp, c_boxes, nspec,
                                                None, 1, 1, lb, ub, stream or None, C.byref(st)),
               "lb200_compute_bounds_device")
        self.last_stats = st
        return st

    def compute_bounds_host_ptr(self, method: int, xl: int, xu: int, n_boxes: int, Cp: int,
                                c_boxes: int, nspec: int, lb: int, ub: int):
        """Host-pointer variant (pointers as ints, e.g. pinned torch tensors)."""
        st = Stats()
        f = C.POINTER(C.c_float)
        _check(_lib.lb200_compute_bounds(self._h, method, C.cast(xl, f), C.cast(xu, f), n_boxes,
                                         C.cast(Cp, f), c_boxes, nspec, f(), 1, 1, C.cast(lb, f),
                                         C.cast(ub, f), C.byref(st)), "lb200_compute_bounds")
        self.last_stats = st
        return st

    def ibp_bounds_noalloc_ptr(self, xl: int, xu: int, n_boxes: int, Cp: int, c_boxes: int, nspec: int,
                               lb: int, ub: int, stream: int = 0):
        """IBP bounds through the allocation-free entry point (device pointers
        as ints).  Enqueues on `stream` and returns without waiting."""
        _check(_lib.lb200_ibp_bounds_noalloc(self._h, xl, xu, n_boxes, Cp, c_boxes, nspec, lb, ub,
                                             stream or None), "lb200_ibp_bounds_noalloc")

    def intermediate_bounds(self):
        """Pre-activation bounds of the last call, [B, sum of widths] lower and upper."""
        cnt = C.c_int64()
        _check(_lib.lb200_get_intermediate_bounds(self._h, None, None, C.byref(cnt)), "intermediate")
        lo = np.empty(cnt.value, np.float32)
        hi = np.empty(cnt.value, np.float32)
        _check(_lib.lb200_get_intermediate_bounds(self._h, fptr(lo), fptr(hi), C.byref(cnt)), "intermediate")
        return lo, hi

    def close(self):
        if getattr(self, "_h", None):
            _lib.lb200_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
