"""Luna's Python API (`lunapy`, lunapy/lunapy.py in the Luna sources) over
this engine.

`TorchModel` keeps the method names, arguments and return types of
lunapy.TorchModel (lunapy/lunapy.py:48-228): input bounds and a
specification matrix are set on the model, `compute_bounds` runs IBP,
CROWN or alpha-CROWN and returns a `BoundedTensor`, and the last result is
kept for `getFinalAnalysisBounds`.  Two differences: the model is built from
a `luna_b200.abi.Graph` (node list and weights) rather than an ONNX file,
since the engine has no ONNX front end; and besides Luna's single box
(`[n_in]` bounds, `[nspec]` results) a batch of boxes (`[B, n_in]` bounds,
`[B, nspec]` results) is accepted, bounded in one engine call.

With `vnnlib_path` the input box and the specification (C, thresholds, OR
branches) come from the property file, as in
`TorchModel(onnx_path, vnnlib_path)`; `compute_bounds` then keeps the
thresholds, so Luna's early stops on verified boxes apply, and
`propertyStatus()` gives the CLI's verdict.  `setSpecificationMatrix`
replaces the property's specification (and drops its thresholds), as in
Luna.
"""
from __future__ import annotations

import numpy as np

from . import abi
from .engine import Model

_METHODS = {
    "IBP": abi.METHOD_IBP,
    "CROWN": abi.METHOD_CROWN,
    "alpha-CROWN": abi.METHOD_ALPHA_CROWN,
    "alpha_crown": abi.METHOD_ALPHA_CROWN,
    "AlphaCROWN": abi.METHOD_ALPHA_CROWN,
}


class BoundedTensor:
    """Lower and upper bounds (lunapy.BoundedTensor)."""

    def __init__(self, lower, upper):
        self._lower = np.asarray(lower, np.float32)
        self._upper = np.asarray(upper, np.float32)

    def lower(self):
        return self._lower

    def upper(self):
        return self._upper

    def __repr__(self):
        return f"<BoundedTensor shape={self._lower.shape}>"


class TorchModel:
    """A network with bound propagation on one GPU (lunapy.TorchModel)."""

    def __init__(self, graph, vnnlib_path=None, device: int = 0, options: abi.Options | None = None):
        if isinstance(graph, (str, bytes)):
            raise NotImplementedError("ONNX files are not read by this library; pass a luna_b200.abi.Graph")
        self._graph = graph
        self._options = options if options is not None else abi.default_options()
        self._device = device
        self._model = None  # the engine model, built on the first bound computation
        self._lower = self._upper = None
        self._C = None
        self._final = None
        self._property = None
        self._status = None
        if vnnlib_path is not None:
            from .vnnlib import Property
            self._property = Property.from_file(vnnlib_path, self.getInputSize(), self.getOutputSize())
            self._lower, self._upper = self._property.lower.copy(), self._property.upper.copy()

    # ---------------------------------------------------------------- sizes
    def getInputSize(self) -> int:
        return int(np.prod(self._graph.nodes[self._graph.input_index].out_shape))

    def getOutputSize(self) -> int:
        return int(np.prod(self._graph.nodes[self._graph.output_index].out_shape))

    def getNumNodes(self) -> int:
        return len(self._graph.nodes)

    # ---------------------------------------------------------------- inputs
    def setInputBounds(self, lower, upper):
        """Flat bounds of one box ([n_in]) or of a batch ([B, n_in])."""
        lower = np.asarray(lower, np.float32)
        upper = np.asarray(upper, np.float32)
        if lower.shape != upper.shape or lower.shape[-1] != self.getInputSize() or lower.ndim > 2:
            raise ValueError(f"input bounds must be [{self.getInputSize()}] or [B, {self.getInputSize()}]")
        if (lower > upper).any():
            raise ValueError("lower input bound above upper bound")
        self._lower, self._upper = lower, upper

    def getInputBounds(self) -> BoundedTensor:
        if self._lower is None:
            raise RuntimeError("input bounds are not set")
        return BoundedTensor(self._lower, self._upper)

    def hasInputBounds(self) -> bool:
        return self._lower is not None

    def forward(self, input_data):
        """The network's output at the given input(s) (fp32, on the CPU)."""
        import torch

        from .workloads import graph_forward
        x = np.asarray(input_data, np.float32)
        single = x.ndim == 1
        y = graph_forward(self._graph, torch.from_numpy(x.reshape(-1, self.getInputSize())))
        y = y.detach().numpy()
        return y[0] if single else y

    # --------------------------------------------------------- specification
    def setSpecificationMatrix(self, C):
        """C [nspec, n_out] (or [1, nspec, n_out]) for every box, or
        [B, nspec, n_out] with one specification per box."""
        self._C = self._spec(C)
        self._property = None

    def hasSpecificationMatrix(self) -> bool:
        return self._C is not None or (self._property is not None and self._property.has_spec)

    def _spec(self, C):
        C = np.asarray(C, np.float32)
        if C.ndim == 2:
            C = C[None]
        if C.ndim != 3 or C.shape[-1] != self.getOutputSize():
            raise ValueError(f"specification must be [nspec, {self.getOutputSize()}] or [B, nspec, "
                             f"{self.getOutputSize()}]")
        return np.ascontiguousarray(C)

    # ---------------------------------------------------------------- bounds
    def compute_bounds(self, method="CROWN", bound_lower=True, bound_upper=True, C=None) -> BoundedTensor:
        """Bounds of C . output over the input box(es).  Without C (and no
        specification matrix set) C is the identity: bounds of every output,
        as Luna's backward start from the output node does."""
        if method not in _METHODS:
            raise ValueError(f"unknown method {method!r}; one of {sorted(_METHODS)}")
        if self._lower is None:
            raise RuntimeError("input bounds are not set")
        spec = self._spec(C) if C is not None else self._C
        if spec is None and self._property is not None and self._property.has_spec:
            spec = self._property.C[None]
        if spec is None:
            spec = np.eye(self.getOutputSize(), dtype=np.float32)[None]
        single = self._lower.ndim == 1
        lo = self._lower.reshape(-1, self.getInputSize())
        hi = self._upper.reshape(-1, self.getInputSize())
        if self._model is None:
            self._model = Model(self._graph, device=self._device, options=self._options)
        self._status = None
        if C is None and self._property is not None and _METHODS[method] != abi.METHOD_IBP:
            # The property's specification with its thresholds (the CLI's path).
            lb, ub, self._status = self._model.compute_property(self._property, _METHODS[method], lo, hi)
        else:
            if spec.shape[0] not in (1, lo.shape[0]):
                raise ValueError("one specification for all boxes, or one per box")
            from .workloads import Boxes
            lb, ub = self._model.compute_bounds(Boxes(lo, hi, spec), _METHODS[method], bound_lower, bound_upper)
        self._final = BoundedTensor(lb[0] if single else lb, ub[0] if single else ub)
        return self._final

    def propertyStatus(self):
        """The CLI's verdict ('unsat' = verified, 'sat', 'unknown') of the last
        bound computation against the property file, per box."""
        if self._status is None:
            raise RuntimeError("no property analysis has run")
        names = [abi.STATUS_NAMES[int(v)] for v in self._status]
        return names[0] if self._lower.ndim == 1 else names

    def runCROWN(self) -> BoundedTensor:
        return self.compute_bounds("CROWN")

    def runAlphaCROWN(self, optimizeLower=True, optimizeUpper=False) -> BoundedTensor:
        if optimizeUpper:
            raise NotImplementedError("optimising upper bounds is not supported by this engine build")
        if not optimizeLower:
            return self.compute_bounds("CROWN")
        return self.compute_bounds("alpha-CROWN")

    def getFinalAnalysisBounds(self) -> BoundedTensor:
        if self._final is None:
            raise RuntimeError("no analysis has run")
        return self._final

    def hasFinalAnalysisBounds(self) -> bool:
        return self._final is not None

    def __repr__(self):
        return (f"<TorchModel nodes={self.getNumNodes()}, input_size={self.getInputSize()}, "
                f"output_size={self.getOutputSize()}>")
