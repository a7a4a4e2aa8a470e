"""CUDAExecutionProvider: the reference's operator API, executed on a B200.

Mirrors ``CPUExecutionProvider`` (src/Lokad.Onnx.Backend/CPUExecutionProvider.cs):
the same op names and argument meaning, and the same error behaviour -- a
validation or execution failure never raises but returns an ``OpResult``
with ``Status == "Failure"`` and a message (src/Lokad.Onnx.Backend/OpResult.cs:15-62).
Inputs are host arrays (the reference's ITensor); each call runs one node
through liblonnx_cuda.so, so the arithmetic is the CUDA kernels'.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import _native as N
from .graph import run_node
from .graphs import Node

SUPPORTED_OPS = ["Reshape", "Add", "Div", "Sub", "Mul", "Pow", "Conv", "Relu", "MaxPool", "MatMul", "Sqrt",
                 "Erf", "Transpose", "Constant", "Cast", "Concat", "Shape", "Gather", "Slice", "Unsqueeze",
                 "ReduceSum", "ReduceMean", "ReduceMax", "Softmax"]


@dataclass
class OpResult:
    Op: str
    Status: str  # "Success" | "Failure"
    Message: str | None = None
    Outputs: list = field(default_factory=list)

    @staticmethod
    def Success(op, *outputs):
        return OpResult(op, "Success", None, list(outputs))

    @staticmethod
    def Failure(op, message):
        return OpResult(op, "Failure", message, [])


def _run(op, inputs, attrs=None, opset=13):
    names = [f"in{i}" if x is not None else "" for i, x in enumerate(inputs)]
    while names and names[-1] == "":
        names.pop()
    feed = {n: np.asarray(x) for n, x in zip(names, inputs) if n}
    node = Node(op, names, ["out"], {k: v for k, v in (attrs or {}).items() if v is not None})
    try:
        r = run_node(node, feed, opset=opset)
        return OpResult.Success(op, r["out"])
    except N.LonnxError as e:
        return OpResult.Failure(op, e.message)


def _missing(op, name):
    return OpResult.Failure(op, f"The required input parameter {name} is missing or null.")


class CUDAExecutionProvider:
    SupportedOps = SUPPORTED_OPS

    @staticmethod
    def SupportsOp(op):
        return op in SUPPORTED_OPS

    @staticmethod
    def _binary(op, A, B):
        if A is None:
            return _missing(op, "A")
        if B is None:
            return _missing(op, "B")
        if np.asarray(A).dtype != np.asarray(B).dtype:
            return OpResult.Failure(op, "The input tensor for parameter B has the wrong type: Input tensors must be of the same type..")
        return _run(op, [A, B])

    Add = staticmethod(lambda A, B: CUDAExecutionProvider._binary("Add", A, B))
    Sub = staticmethod(lambda A, B: CUDAExecutionProvider._binary("Sub", A, B))
    Mul = staticmethod(lambda A, B: CUDAExecutionProvider._binary("Mul", A, B))
    Div = staticmethod(lambda A, B: CUDAExecutionProvider._binary("Div", A, B))
    Pow = staticmethod(lambda A, B: CUDAExecutionProvider._binary("Pow", A, B))

    @staticmethod
    def Relu(X):
        return _missing("Relu", "X") if X is None else _run("Relu", [X])

    @staticmethod
    def Sqrt(A):
        return _missing("Sqrt", "A") if A is None else _run("Sqrt", [A])

    @staticmethod
    def Erf(X):
        return _missing("Erf", "X") if X is None else _run("Erf", [X])

    @staticmethod
    def MatMul(A, B):
        if A is None:
            return _missing("MatMul", "A")
        if B is None:
            return _missing("MatMul", "B")
        return _run("MatMul", [A, B])

    @staticmethod
    def Conv(X, W, B=None, auto_pad=None, dilations=None, group=None, kernel_shape=None, pads=None,
             strides=None):
        if X is None:
            return _missing("Conv", "X")
        if W is None:
            return _missing("Conv", "W")
        attrs = dict(auto_pad=auto_pad, dilations=dilations, group=group, kernel_shape=kernel_shape, pads=pads,
                     strides=strides)
        return _run("Conv", [X, W, B], attrs)

    @staticmethod
    def MaxPool(X, auto_pad=None, ceil_mode=None, dilations=None, kernel_shape=None, pads=None,
                storage_order=None, strides=None):
        if X is None:
            return _missing("MaxPool", "X")
        attrs = dict(auto_pad=auto_pad, dilations=dilations, kernel_shape=kernel_shape, pads=pads, strides=strides)
        return _run("MaxPool", [X], attrs)

    @staticmethod
    def Softmax(input, axis=None):
        if input is None:
            return _missing("Softmax", "input")
        return _run("Softmax", [input], {"axis": axis})

    @staticmethod
    def _reduce(op, data, axes, keep_dims, noop=None):
        if data is None:
            return _missing(op, "data")
        return _run(op, [data, None if axes is None else np.asarray(axes, np.int64)], {"keepdims": keep_dims})

    ReduceSum = staticmethod(lambda data, axes=None, keep_dims=None, noop_with_empty_axes=None:
                             CUDAExecutionProvider._reduce("ReduceSum", data, axes, keep_dims))
    ReduceMean = staticmethod(lambda data, axes=None, keep_dims=None, noop_with_empty_axes=None:
                              CUDAExecutionProvider._reduce("ReduceMean", data, axes, keep_dims))
    ReduceMax = staticmethod(lambda data, axes=None, keep_dims=None:
                             CUDAExecutionProvider._reduce("ReduceMax", data, axes, keep_dims))

    @staticmethod
    def Gather(data, indices, axis=None):
        if data is None:
            return _missing("Gather", "data")
        if indices is None:
            return _missing("Gather", "indices")
        if np.asarray(indices).ndim > np.asarray(data).ndim:
            return OpResult.Failure("Gather", "The input tensor for parameter indices has the wrong shape.")
        return _run("Gather", [data, np.asarray(indices).astype(np.int64)], {"axis": axis})

    @staticmethod
    def Transpose(data, perm=None):
        if data is None:
            return _missing("Transpose", "data")
        return _run("Transpose", [data], {"perm": perm})

    @staticmethod
    def Reshape(input, shape, allow_zero=None):
        if input is None:
            return _missing("Reshape", "input")
        if shape is None:
            return _missing("Reshape", "shape")
        if np.asarray(shape).dtype != np.int64:
            return OpResult.Failure("Reshape", "The input tensor for parameter shape must be Int64.")
        return _run("Reshape", [input, shape], {"allowzero": None if allow_zero is None else int(allow_zero)})

    @staticmethod
    def Unsqueeze(data, axes):
        if data is None:
            return _missing("Unsqueeze", "data")
        if axes is None:
            return _missing("Unsqueeze", "axes")
        return _run("Unsqueeze", [data, np.asarray(axes, np.int64)])
