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
                 "ReduceSum", "ReduceMean", "ReduceMax", "Softmax",
                 # ONNX ops the reference names but does not dispatch (ResNet-50 coverage)
                 "Gemm", "BatchNormalization", "GlobalAveragePool", "Flatten"]


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
        # attributes passed to a provider method reach the op (the CPU
        # provider's Conv honours strides/dilations/group/kernel_shape)
        r = run_node(node, feed, opset=opset, honor_conv_attrs=True)
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
        if auto_pad == "NOTSET":
            if pads is None:
                return OpResult.Failure("Conv", "The required attribute pads is missing or null. When auto_pad is "
                                                "NOTSET pads must be specified")
            if any(p != pads[0] for p in pads):
                return OpResult.Failure("Conv", f"The attribute pads with value {list(pads)} is not supported for "
                                                "operation Conv. Asymmetric padding is not supported.")
        # CPUExecutionProvider.Conv reads pads only when auto_pad is NOTSET
        # (CPUExecutionProvider.cs:253-279); otherwise they do not reach the op
        attrs = dict(auto_pad=auto_pad, dilations=dilations, group=group, kernel_shape=kernel_shape,
                     pads=pads if auto_pad == "NOTSET" else None, strides=strides)
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

    @staticmethod
    def Constant(value):
        """CPUExecutionProvider.Constant (:435-449): a tensor, float, float
        list, int or int list becomes the op's output."""
        if value is None:
            return OpResult.Failure("Constant", "The required attribute value is missing or null. ")
        if isinstance(value, np.ndarray):
            return _run("Constant", [], {"value": value})
        if isinstance(value, float):
            return _run("Constant", [], {"value_float": value})
        if isinstance(value, int):
            return _run("Constant", [], {"value_int": value})
        if isinstance(value, (list, tuple)) and value and all(isinstance(v, float) for v in value):
            return _run("Constant", [], {"value_floats": list(value)})
        if isinstance(value, (list, tuple)) and all(isinstance(v, int) for v in value):
            return _run("Constant", [], {"value_ints": list(value)})
        return OpResult.Failure("Constant", "The operation Constant is not supported by the backend.")

    @staticmethod
    def Cast(input, to):
        if input is None:
            return _missing("Cast", "input")
        if int(to) not in (1, 6, 7, 9):
            return OpResult.Failure("Cast", f"The attribute to with value {to} is not supported for operation Cast. ")
        return _run("Cast", [input], {"to": int(to)})

    @staticmethod
    def Concat(inputs, axis=None):
        if inputs is None:
            return _missing("Concat", "inputs")
        arrs = [np.asarray(t) for t in inputs]
        if any(a.dtype != arrs[0].dtype for a in arrs):
            return OpResult.Failure("Concat", "The input tensor for parameter inputs has the wrong type: All tensors "
                                              "in a concat operation must have the same type..")
        return _run("Concat", arrs, {"axis": 0 if axis is None else int(axis)})

    @staticmethod
    def Shape(data, start=None, end=None):
        if data is None:
            return _missing("Shape", "data")
        return _run("Shape", [data], {"start": start, "end": end})

    @staticmethod
    def Slice(data, starts, ends, axes=None, steps=None):
        """CPUExecutionProvider.Slice (:548-600) with its validation messages."""
        op = "Slice"
        if data is None:
            return _missing(op, "data")
        if starts is None:
            return _missing(op, "starts")
        if ends is None:
            return _missing(op, "ends")
        d, s_, e = np.asarray(data), np.asarray(starts), np.asarray(ends)
        bad = lambda name, t, msg: OpResult.Failure(op, f"The input tensor for parameter {name} has shape "
                                                        f"{list(np.asarray(t).shape)}. {msg}.")
        if d.ndim == 0:
            return bad("data", d, "Cannot slice a tensor of rank 0")
        if s_.ndim != 1:
            return bad("starts", s_, "The rank of the starts tensor must be 1")
        if s_.size > d.ndim:
            return bad("starts", s_, "The length of the starts tensor must be less-than or equal to the rank of "
                                     "the data tensor.")
        if e.ndim != 1:
            return bad("ends", e, "The rank of the ends tensor must be 1")
        if s_.size != e.size:
            return bad("ends", e, "The ends tensor must be the same length as the start tensor.")
        for name, t in (("axes", axes), ("steps", steps)):
            if t is not None and (np.asarray(t).ndim != 1 or np.asarray(t).size != s_.size):
                return bad(name, t, f"The {name} tensor must be a rank 1 tensor with the same length as the start "
                                    "tensor.")
        ints = lambda t: None if t is None else np.asarray(t).astype(np.int64)
        return _run(op, [data, ints(starts), ints(ends), ints(axes), ints(steps)])

    # ---- ONNX ops beyond the CPU provider (ONNX operator semantics) ----

    @staticmethod
    def Gemm(A, B, C=None, alpha=None, beta=None, transA=None, transB=None):
        if A is None:
            return _missing("Gemm", "A")
        if B is None:
            return _missing("Gemm", "B")
        return _run("Gemm", [A, B, C], {"alpha": None if alpha is None else float(alpha),
                                        "beta": None if beta is None else float(beta),
                                        "transA": transA, "transB": transB})

    @staticmethod
    def BatchNormalization(X, scale, B, input_mean, input_var, epsilon=None):
        for name, t in (("X", X), ("scale", scale), ("B", B), ("input_mean", input_mean), ("input_var", input_var)):
            if t is None:
                return _missing("BatchNormalization", name)
        return _run("BatchNormalization", [X, scale, B, input_mean, input_var],
                    {"epsilon": None if epsilon is None else float(epsilon)})

    @staticmethod
    def GlobalAveragePool(X):
        return _missing("GlobalAveragePool", "X") if X is None else _run("GlobalAveragePool", [X])

    @staticmethod
    def Flatten(input, axis=None):
        return _missing("Flatten", "input") if input is None else _run("Flatten", [input], {"axis": axis})
