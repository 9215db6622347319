"""ctypes mirror of include/luna_b200.h (the engine's C ABI).

The structures here are laid out exactly as the C header declares them; the
header is the source of truth.  `Graph` owns the numpy buffers that the node
descriptors point into, so they stay alive as long as the descriptor.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

NODE_INPUT = 0
NODE_CONSTANT = 1
NODE_LINEAR = 2
NODE_RELU = 3
NODE_RESHAPE = 4
NODE_IDENTITY = 5
NODE_SUB = 6
NODE_FLATTEN = 7
NODE_ADD = 8
NODE_CONV = 9
NODE_BATCHNORM = 10
NODE_SIGMOID = 11
NODE_CONVTRANSPOSE = 12
NODE_CONCAT = 13
NODE_SLICE = 14

METHOD_IBP = 0
METHOD_CROWN = 1
METHOD_ALPHA_CROWN = 2

# lb200_status: the verdict on a VNN-LIB property for one box.
STATUS_UNKNOWN = 0
STATUS_UNSAT = 1  # verified: the counterexample region is unreachable
STATUS_SAT = 2    # every point of the box is a counterexample
STATUS_NAMES = {STATUS_UNKNOWN: "unknown", STATUS_UNSAT: "unsat", STATUS_SAT: "sat"}

_fp = C.POINTER(C.c_float)


class NodeDesc(C.Structure):
    _fields_ = [
        ("type", C.c_int32),
        ("num_inputs", C.c_int32),
        ("inputs", C.c_int32 * 4),
        ("in_features", C.c_int64),
        ("out_features", C.c_int64),
        ("scale", C.c_float),
        ("weight", _fp),
        ("bias", _fp),
        ("out_shape", C.c_int32 * 3),
        ("kernel", C.c_int32 * 2),
        ("stride", C.c_int32 * 2),
        ("padding", C.c_int32 * 2),
        ("output_padding", C.c_int32 * 2),
        ("running_mean", _fp),
        ("running_var", _fp),
        ("eps", C.c_float),
        ("constant", _fp),
        ("constant_second", C.c_int32),
        ("axis", C.c_int32),
        ("start", C.c_int64),
        ("end", C.c_int64),
        ("step", C.c_int64),
    ]


class GraphDesc(C.Structure):
    _fields_ = [
        ("num_nodes", C.c_int32),
        ("nodes", C.POINTER(NodeDesc)),
        ("input_index", C.c_int32),
        ("output_index", C.c_int32),
    ]


class Options(C.Structure):
    _fields_ = [
        ("alpha_iterations", C.c_uint32),
        ("alpha_lr", C.c_float),
        ("alpha_lr_decay", C.c_float),
        ("early_stop_patience", C.c_uint32),
        ("start_save_best", C.c_float),
        ("stabilize_intermediate_bounds", C.c_int32),
        ("recompute_intermediate_bounds", C.c_int32),
        ("optimize_lower", C.c_int32),
        ("optimize_upper", C.c_int32),
        ("stop_crown_on_verified", C.c_int32),
        ("stop_alpha_on_verified", C.c_int32),
        ("enable_first_linear_ibp", C.c_int32),
        ("use_patches_mode", C.c_int32),
    ]


class Stats(C.Structure):
    _fields_ = [
        ("ms_total", C.c_double),
        ("ms_device", C.c_double),
        ("kernel_launches", C.c_int64),
        ("backward_rows", C.c_int64),
        ("algorithmic_flops", C.c_double),
        ("alpha_iterations_run", C.c_int32),
        ("ms_contractions", C.c_double),
        ("contraction_launches", C.c_int64),
        ("contraction_flops", C.c_double),
    ]


class PropertyInfo(C.Structure):
    _fields_ = [
        ("n_in", C.c_int64),
        ("n_out", C.c_int64),
        ("nspec", C.c_int64),
        ("n_branches", C.c_int32),
        ("spec_dropped", C.c_int32),
        ("spec_error", C.c_char * 256),
    ]


def default_options(**overrides) -> Options:
    """Luna's LunaConfiguration defaults (src/configuration/LunaConfiguration.cpp:28-50)."""
    o = Options(
        alpha_iterations=20,
        alpha_lr=0.5,
        alpha_lr_decay=0.98,
        early_stop_patience=10,
        start_save_best=0.5,
        stabilize_intermediate_bounds=1,
        recompute_intermediate_bounds=1,
        optimize_lower=1,
        optimize_upper=0,
        stop_crown_on_verified=1,
        stop_alpha_on_verified=1,
        enable_first_linear_ibp=1,
        use_patches_mode=1,
    )
    for k, v in overrides.items():
        setattr(o, k, v)
    return o


def fptr(a: np.ndarray | None):
    if a is None:
        return _fp()
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


@dataclass
class Node:
    """One Bounded*Node: kind, producers, parameters and output shape (C, H, W)."""
    type: int
    inputs: list
    out_shape: tuple
    weight: np.ndarray | None = None
    bias: np.ndarray | None = None
    scale: float = 1.0
    kernel: tuple = (0, 0)
    stride: tuple = (1, 1)
    padding: tuple = (0, 0)
    output_padding: tuple = (0, 0)
    running_mean: np.ndarray | None = None
    running_var: np.ndarray | None = None
    eps: float = 1e-5
    # SUB with a constant: x - constant (constant_second) or constant - x.
    constant: np.ndarray | None = None
    constant_second: int = 1
    # SLICE (axis, start, end, step) and CONCAT (axis).
    axis: int = 1
    start: int = 0
    end: int = 0
    step: int = 1

    @property
    def size(self) -> int:
        return int(np.prod(self.out_shape))


@dataclass
class Graph:
    """A computation graph in TorchModel form: nodes indexed by id, one input, one output."""
    nodes: list
    input_index: int
    output_index: int
    _keep: list = field(default_factory=list, repr=False)

    @property
    def n_in(self) -> int:
        return self.nodes[self.input_index].size

    @property
    def n_out(self) -> int:
        return self.nodes[self.output_index].size

    def desc(self) -> GraphDesc:
        arr = (NodeDesc * len(self.nodes))()
        keep = []
        for i, n in enumerate(self.nodes):
            d = arr[i]
            d.type = n.type
            d.num_inputs = len(n.inputs)
            for k, p in enumerate(n.inputs):
                d.inputs[k] = p
            for k in range(3):
                d.out_shape[k] = int(n.out_shape[k])
            d.scale = n.scale
            if n.weight is not None:
                w = np.ascontiguousarray(n.weight, dtype=np.float32)
                keep.append(w)
                d.weight = fptr(w)
                if n.type == NODE_LINEAR:
                    d.out_features, d.in_features = w.shape
            if n.bias is not None:
                b = np.ascontiguousarray(n.bias, dtype=np.float32)
                keep.append(b)
                d.bias = fptr(b)
            for k in range(2):
                d.kernel[k] = n.kernel[k]
                d.stride[k] = n.stride[k]
                d.padding[k] = n.padding[k]
                d.output_padding[k] = n.output_padding[k]
            for name in ("running_mean", "running_var", "constant"):
                v = getattr(n, name)
                if v is not None:
                    v = np.ascontiguousarray(v, dtype=np.float32)
                    keep.append(v)
                    setattr(d, name, fptr(v))
            d.eps = n.eps
            d.constant_second = n.constant_second
            d.axis = n.axis
            d.start = n.start
            d.end = n.end
            d.step = n.step
        self._keep = [arr, keep]
        return GraphDesc(len(self.nodes), C.cast(arr, C.POINTER(NodeDesc)),
                         self.input_index, self.output_index)

    def activation_inputs(self) -> list:
        """Ids of the nodes that feed a ReLU or Sigmoid, ascending."""
        out = set()
        for n in self.nodes:
            if n.type in (NODE_RELU, NODE_SIGMOID):
                out.add(n.inputs[0])
        return sorted(out)
