"""CPU oracle for the Lokad.Onnx float32 inference path -- TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm may import this module; the product (onnx_b200/) never does.

It restates the reference's operator layer (``CPUExecutionProvider`` and the
``Tensor<float>`` ops it calls) and its graph executor
(``ComputationalGraph.Execute``) on numpy arrays.  The arithmetic runs in
``liblonnx_oracle.so`` (lonnx_oracle.c, same loop and summation order as the
reference); shape logic, broadcasting and pure data movement (gather,
transpose, reshape) run in numpy, where they are exact.

References (paths inside the Lokad/Onnx project):
  src/Lokad.Onnx.Backend/CPUExecutionProvider.cs  operator API and validation
  src/Lokad.Onnx.Backend/Node.cs:121-181          which attributes reach each op
  src/Lokad.Onnx.Backend/ComputationalGraph.cs:199-272  executor loop
  src/Lokad.Onnx.Tensors/TensorOps.cs, MathOps.cs  the kernels
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build() -> str:
    """Compile liblonnx_oracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liblonnx_oracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liblonnx_oracle.so")
        src = os.path.join(_HERE, "lonnx_oracle.c")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(path)
        f32p = ctypes.POINTER(ctypes.c_float)
        i64p = ctypes.POINTER(ctypes.c_int64)
        i, i64 = ctypes.c_int, ctypes.c_int64
        L.oracle_mm.argtypes = [i, i, i, f32p, f32p, f32p]
        L.oracle_mm_batched.argtypes = [i, i64p, i64p, i64p, i, i, i, f32p, f32p, f32p]
        L.oracle_conv2d.argtypes = [f32p, i, i, i, i, i, i, i, i, i, i, i, i, i, i, i,
                                    f32p, f32p, i, f32p]
        L.oracle_conv2d.restype = i
        L.oracle_maxpool2d.argtypes = [f32p] + [i] * 12 + [f32p]
        L.oracle_reduce_inner.argtypes = [i, f32p, i64, i64, f32p]
        L.oracle_softmax.argtypes = [f32p, i64, i64, i64, f32p]
        L.oracle_unary.argtypes = [i, f32p, f32p, i64]
        L.oracle_binary.argtypes = [i, f32p, f32p, f32p, i64]
        _LIB = L
    return _LIB


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ip(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class OracleError(Exception):
    """An operator failure, the oracle's stand-in for OpResult.Failure
    (src/Lokad.Onnx.Backend/OpResult.cs:34-62)."""


# ----------------------------------------------------------------------------
# Shape helpers
# ----------------------------------------------------------------------------

def broadcast_shape(a, b):
    """Tensor<T>.Broadcast shape rule (TensorOps.cs:135-193): right-aligned,
    equal dims or a dim of 1; None when incompatible."""
    a, b = tuple(a), tuple(b)
    if a == b:
        return a
    if len(a) == 0:
        return b
    if len(b) == 0:
        return a
    r = max(len(a), len(b))
    a = (1,) * (r - len(a)) + a
    b = (1,) * (r - len(b)) + b
    out = []
    for x, y in zip(a, b):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            return None
    return tuple(out)


def _neg(rank, axis):
    """ArrayUtilities.HandleNegativeAxisOrIndex."""
    return axis + rank if axis < 0 else axis


def conv_output_info(pad_type, in_h, in_w, stride_h, stride_w, k_h, k_w, pad_value=None):
    """MathOps.GetConv2DOutputInfo (src/Lokad.Onnx.Tensors/MathOps.cs:36-89).

    Returns (out_h, out_w, top, left, bottom, right).  SAME_LOWER is handled as
    SAME_UPPER, as in the reference (MathOps.cs:54-73)."""
    if pad_type == "VALID":
        out_h = math.ceil((in_h - k_h + 1.0) / stride_h)
        out_w = math.ceil((in_w - k_w + 1.0) / stride_w)
        return out_h, out_w, 0, 0, 0, 0
    if pad_type in ("SAME_UPPER", "SAME_LOWER"):
        out_h = math.ceil(in_h / float(stride_h))
        out_w = math.ceil(in_w / float(stride_w))
        pad_h = (out_h - 1) * stride_h + k_h - in_h
        pad_w = (out_w - 1) * stride_w + k_w - in_w
        top = math.floor(pad_h / 2.0)
        left = math.floor(pad_w / 2.0)
        return out_h, out_w, top, left, pad_h - top, pad_w - left
    if pad_type == "VALUE":
        if pad_value is None:
            raise OracleError("padValue is required")
        p = pad_value
        out_h = math.floor((in_h - k_h + 2 * p * 1.0) / stride_h) + 1
        out_w = math.floor((in_w - k_w + 2 * p * 1.0) / stride_w) + 1
        return out_h, out_w, p, p, p, p
    raise OracleError(f"unknown pad type {pad_type}")


def _pad_mode(auto_pad, pads):
    """auto_pad string -> pad mode, CPUExecutionProvider.cs:253-279 / 326-352.
    An absent or empty auto_pad means VALID (explicit pads are then ignored)."""
    if not auto_pad:
        return "VALID", None
    if auto_pad == "VALID":
        return "VALID", None
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        return auto_pad, None
    if auto_pad == "NOTSET":
        if pads is None:
            raise OracleError("When auto_pad is NOTSET pads must be specified")
        if not all(p == pads[0] for p in pads):
            raise OracleError("Asymmetric padding is not supported.")
        return "VALUE", int(pads[0])
    return "VALID", None


# ----------------------------------------------------------------------------
# Operators (CPUExecutionProvider.<Op>)
# ----------------------------------------------------------------------------

_BIN = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3, "Pow": 4}


def binary(op, a, b):
    """Add/Sub/Mul/Div/Pow with numpy broadcasting (CPUExecutionProvider.cs:82-236)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.dtype != b.dtype:
        raise OracleError("Input tensors must be of the same type.")
    shape = broadcast_shape(a.shape, b.shape)
    if shape is None:
        raise OracleError(f"The tensors {a.shape} and {b.shape} are not compatible for broadcasting.")
    if a.dtype != np.float32:
        f = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply,
             "Div": np.floor_divide if a.dtype.kind in "iu" else np.divide, "Pow": np.power}[op]
        return f(a, b).astype(a.dtype)
    ba = _f32(np.broadcast_to(a, shape))
    bb = _f32(np.broadcast_to(b, shape))
    y = np.empty(shape, np.float32)
    lib().oracle_binary(_BIN[op], _fp(ba), _fp(bb), _fp(y), y.size)
    return y


def unary(op, x):
    code = {"Relu": 0, "Sqrt": 1, "Erf": 2, "Exp": 3}[op]
    x = _f32(x)
    y = np.empty_like(x)
    lib().oracle_unary(code, _fp(x), _fp(y), x.size)
    return y


def matmul(a, b):
    """Tensor<float>.MatMul (TensorOps.cs:600-704)."""
    a = _f32(a)
    b = _f32(b)
    if a.ndim == 0 or b.ndim == 0:
        raise OracleError("The rank of each tensor in matrix multiplication must be greater than 1.")
    if a.ndim >= 2 and b.ndim >= 2:
        if a.shape[-1] != b.shape[-2]:
            raise OracleError("The number of columns in the first matrix is not equal to the number of rows in the second matrix.")
        lead = broadcast_shape(a.shape[:-2], b.shape[:-2])
        if lead is None:
            raise OracleError("The tensor shapes are not compatible for broadcasting.")
        m, n = a.shape[-2], a.shape[-1]
        k = b.shape[-1]
        ba = np.broadcast_to(a, lead + (m, n))
        bb = np.broadcast_to(b, lead + (n, k))
        nb = int(np.prod(lead)) if lead else 1
        # storage offsets of each batch (stride 0 on broadcast dims)
        idx = np.indices(lead).reshape(len(lead), -1).T if lead else np.zeros((1, 0), np.int64)
        sa = np.array(ba.strides[:-2], np.int64) // 4
        sb = np.array(bb.strides[:-2], np.int64) // 4
        offa = np.ascontiguousarray((idx * sa).sum(1) if lead else np.zeros(1), np.int64)
        offb = np.ascontiguousarray((idx * sb).sum(1) if lead else np.zeros(1), np.int64)
        offc = np.ascontiguousarray(np.arange(nb, dtype=np.int64) * m * k)
        c = np.empty(lead + (m, k), np.float32)
        lib().oracle_mm_batched(nb, _ip(offa), _ip(offb), _ip(offc), m, n, k, _fp(a), _fp(b), _fp(c))
        return c
    if a.ndim < 2 and b.ndim < 2:
        a2 = a.reshape(1, -1)
        b2 = b.reshape(-1, 1)
        return matmul(a2, b2).reshape(1)
    shape = broadcast_shape(a.shape, b.shape)
    if shape is None:
        raise OracleError(f"The shapes {a.shape} and {b.shape} are not compatible for broadcasting.")
    return matmul(np.broadcast_to(a, shape), np.broadcast_to(b, shape))


def conv(x, w, b=None, auto_pad=None, dilations=None, group=None, kernel_shape=None,
         pads=None, strides=None):
    """CPUExecutionProvider.Conv -> Tensor<float>.Conv2D -> MathOps.Conv2D
    (CPUExecutionProvider.cs:237-291, TensorOps.cs:903-962, MathOps.cs:791-877)."""
    x = _f32(x)
    w = _f32(w)
    if x.ndim != 4 or w.ndim != 4:
        raise OracleError("Conv inputs must be of rank 4")
    mode, pv = _pad_mode(auto_pad, pads)
    strides = list(strides) if strides is not None else [1, 1]
    dilations = list(dilations) if dilations is not None else [1, 1]
    group = int(group) if group is not None else 1
    n, c, h, wd = x.shape
    m = w.shape[0]
    kh = kernel_shape[0] if kernel_shape is not None else w.shape[2]
    kw = kernel_shape[1] if kernel_shape is not None else w.shape[3]
    ekh = kh if dilations[0] <= 1 else kh + (kh - 1) * (dilations[0] - 1)
    ekw = kw if dilations[1] <= 1 else kw + (kw - 1) * (dilations[1] - 1)
    oh, ow, top, left, bottom, right = conv_output_info(mode, h, wd, strides[0], strides[1], ekh, ekw, pv)
    # the reference passes (left, top, right, bottom) as (padY, padX, padH, padW)
    pad_y, pad_x, pad_h, pad_w = left, top, right, bottom
    dst_h = (h + pad_y + pad_h - (dilations[0] * (kh - 1) + 1)) // strides[0] + 1
    dst_w = (wd + pad_x + pad_w - (dilations[1] * (kw - 1) + 1)) // strides[1] + 1
    if (dst_h, dst_w) != (oh, ow):
        # the reference allocates [N, M, oh, ow] but MathOps.Conv2D writes
        # dst_h x dst_w planes; they agree for every pad mode with square pads
        raise OracleError("conv output geometry mismatch")
    y = np.zeros((n, m, oh, ow), np.float32)
    bias = _f32(b) if b is not None else None
    rc = lib().oracle_conv2d(_fp(x), n, c, h, wd, kh, kw, dilations[0], dilations[1],
                             strides[0], strides[1], pad_y, pad_x, pad_h, pad_w, group,
                             _fp(w), _fp(y), m, _fp(bias) if bias is not None else None)
    if rc != 0:
        raise OracleError("conv: out of memory")
    return y


def maxpool(x, auto_pad=None, ceil_mode=None, dilations=None, kernel_shape=None, pads=None,
            storage_order=None, strides=None):
    """CPUExecutionProvider.MaxPool -> Tensor<float>.MaxPool2D
    (CPUExecutionProvider.cs:311-357, TensorOps.cs:1025-1099)."""
    x = _f32(x)
    if x.ndim != 4:
        raise OracleError("MaxPool input must be of rank 4")
    if kernel_shape is None:
        raise OracleError("kernelshape")
    mode, pv = _pad_mode(auto_pad, pads)
    strides = list(strides) if strides is not None else list(kernel_shape)
    dilations = list(dilations) if dilations is not None else [1, 1]
    n, c, h, w = x.shape
    kh, kw = kernel_shape
    ekh = kh if dilations[0] <= 1 else kh + (kh - 1) * (dilations[0] - 1)
    ekw = kw if dilations[1] <= 1 else kw + (kw - 1) * (dilations[1] - 1)
    oh, ow, top, left, _, _ = conv_output_info(mode, h, w, strides[0], strides[1], ekh, ekw, pv)
    y = np.empty((n, c, oh, ow), np.float32)
    lib().oracle_maxpool2d(_fp(x), n, c, h, w, kh, kw, strides[0], strides[1], top, left, oh, ow, _fp(y))
    return y


def _reduce(code, x, axes, keepdims):
    """ReduceSum/ReduceMax/ReduceMean (TensorOps.cs:1610-1839): transpose the
    reduced axes innermost in the given order, reduce sequentially."""
    x = _f32(x)
    r = x.ndim
    ax = list(range(r)) if axes is None or len(axes) == 0 else [_neg(r, int(a)) for a in axes]
    keep = [d for d in range(r) if d not in ax]
    perm = keep + ax
    xp = _f32(np.transpose(x, perm))
    outer_shape = tuple(x.shape[d] for d in keep)
    red = int(np.prod([x.shape[d] for d in ax])) if ax else 1
    outer = int(np.prod(outer_shape)) if outer_shape else 1
    y = np.empty(outer, np.float32)
    lib().oracle_reduce_inner(code, _fp(xp), outer, red, _fp(y))
    y = y.reshape(outer_shape)
    if keepdims:
        y = y.reshape(tuple(1 if d in ax else x.shape[d] for d in range(r)))
    return y


def reduce_sum(x, axes=None, keepdims=1):
    return _reduce(0, x, axes, keepdims)


def reduce_max(x, axes=None, keepdims=1):
    return _reduce(1, x, axes, keepdims)


def reduce_mean(x, axes=None, keepdims=1):
    return _reduce(2, x, axes, keepdims)


def softmax(x, axis=-1):
    """Tensor<float>.Softmax (TensorOps.cs:1312-1330)."""
    x = _f32(x)
    ax = _neg(x.ndim, axis)
    if ax >= x.ndim:
        raise OracleError("The specified axis must be less than the rank of the tensor.")
    outer = int(np.prod(x.shape[:ax])) if ax > 0 else 1
    inner = int(np.prod(x.shape[ax + 1:])) if ax + 1 < x.ndim else 1
    y = np.empty_like(x)
    lib().oracle_softmax(_fp(x), outer, x.shape[ax], inner, _fp(y))
    return y


def gather(data, indices, axis=None):
    """Tensor<T>.Gather (TensorOps.cs:1410-1446): np.take semantics with
    negative indices wrapped once; indices converted to int32 first
    (ITensor.cs:172-183)."""
    data = np.asarray(data)
    idx = np.asarray(indices)
    if idx.ndim > data.ndim:
        raise OracleError("indices rank exceeds data rank")
    idx = idx.astype(np.int32)
    ax = _neg(data.ndim, axis if axis is not None else 0)
    dim = data.shape[ax]
    w = np.where(idx < 0, idx + dim, idx)
    if np.any(w < 0) or np.any(w >= dim):
        raise OracleError("Index was outside the bounds of the array.")
    return np.take(data, w, axis=ax)


def transpose(x, perm=None):
    x = np.asarray(x)
    if perm is None:
        perm = list(range(x.ndim))[::-1]
    if x.ndim <= 1:
        return x
    return np.ascontiguousarray(np.transpose(x, [_neg(x.ndim, p) for p in perm]))


def reshape(x, shape, allow_zero=False):
    """Tensor<T>.Reshape (TensorOps.cs:1256-1310)."""
    shape = [int(s) for s in np.asarray(shape).reshape(-1)]
    out = []
    for i, s in enumerate(shape):
        out.append(x.shape[i] if (s == 0 and not allow_zero) else s)
    return np.asarray(x).reshape(out)


def unsqueeze(x, axes):
    x = np.asarray(x)
    r = x.ndim + len(axes)
    ax = sorted(_neg(r, int(a)) for a in axes)
    for a in ax:
        x = np.expand_dims(x, a)
    return x


_ONNX_DTYPES = {1: np.float32, 6: np.int32, 7: np.int64, 9: np.bool_, 11: np.float64, 2: np.uint8}


# ----------------------------------------------------------------------------
# ONNX ops the reference names but does not implement (OpType.cs:17,51,57,58;
# absent from CPUExecutionProvider.SupportedOps, CPUExecutionProvider.cs:24-50).
# Restated from the ONNX operator specification, every step a float32 op
# rounded once, composed from the reference's own kernels where one exists
# (the GEMM order of MathOps.cs:380-410, ReduceMean = ReduceSum then divide).
# Parity on these is against the ONNX semantics, not a reference binary.
# ----------------------------------------------------------------------------

def gemm(a, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0):
    """ONNX Gemm: Y = alpha * op(A) . op(B) + beta * C (C broadcast to [M, N])."""
    a = _f32(a)
    b = _f32(b)
    if a.ndim != 2 or b.ndim != 2:
        raise OracleError("Gemm inputs must be of rank 2")
    if trans_a:
        a = _f32(a.T)
    if trans_b:
        b = _f32(b.T)
    y = matmul(a, b)
    if alpha != 1.0:
        y = (np.float32(alpha) * y).astype(np.float32)
    if c is not None and beta != 0.0:
        cc = _f32(c)
        if beta != 1.0:
            cc = (np.float32(beta) * cc).astype(np.float32)
        y = binary("Add", y, cc)
    return y


def batch_norm(x, scale, bias, mean, var, epsilon=1e-5):
    """ONNX BatchNormalization (inference): (x - mean) / sqrt(var + eps) * scale + B
    over axis 1, each step a float32 operation."""
    x = _f32(x)
    shp = (1, -1) + (1,) * (x.ndim - 2)
    m, v, s, b = (_f32(t).reshape(shp) for t in (mean, var, scale, bias))
    den = np.sqrt((v + np.float32(epsilon)).astype(np.float32)).astype(np.float32)
    return ((((x - m).astype(np.float32) / den).astype(np.float32) * s).astype(np.float32) + b).astype(np.float32)


def global_average_pool(x):
    """ONNX GlobalAveragePool: ReduceMean over every spatial axis, kept as 1s."""
    x = _f32(x)
    return reduce_mean(x, list(range(2, x.ndim)), 1)


def flatten(x, axis=1):
    x = np.asarray(x)
    axis = _neg(x.ndim, axis) if axis < 0 else axis
    outer = int(np.prod(x.shape[:axis])) if axis > 0 else 1
    return x.reshape(outer, -1 if outer else 0)


def slice_(data, starts, ends, axes=None, steps=None):
    """Slice (CPUExecutionProvider.Slice, CPUExecutionProvider.cs:548-600):
    numpy slicing with ONNX clamping of starts/ends."""
    data = np.asarray(data)
    starts = [int(v) for v in np.asarray(starts).reshape(-1)]
    ends = [int(v) for v in np.asarray(ends).reshape(-1)]
    axes = list(range(len(starts))) if axes is None else [int(v) for v in np.asarray(axes).reshape(-1)]
    steps = [1] * len(starts) if steps is None else [int(v) for v in np.asarray(steps).reshape(-1)]
    sl = [slice(None)] * data.ndim
    for s, e, a, st in zip(starts, ends, axes, steps):
        sl[_neg(data.ndim, a)] = slice(s, e, st)
    return np.ascontiguousarray(data[tuple(sl)])


# ----------------------------------------------------------------------------
# Graph executor: ComputationalGraph.Execute (ComputationalGraph.cs:199-272)
# ----------------------------------------------------------------------------

def run_node(node, get, opset=13, honor_conv_attrs=False):
    """Node.ExecuteCPU (src/Lokad.Onnx.Backend/Node.cs:121-181).

    ``honor_conv_attrs=False`` reproduces the reference, whose Conv reads its
    INTS attributes as int[] while the loader stores long[] (Node.cs:137-138,
    NodeUtil.cs:13-14), so strides/pads/dilations/kernel_shape/group arrive as
    null.  True applies them (ONNX semantics), used for models the reference
    cannot run correctly (documented deviation)."""
    op, a = node.op, node.attrs
    ins = [get(n) if n else None for n in node.inputs]
    I = lambda i: ins[i] if i < len(ins) else None
    if op in _BIN:
        return [binary(op, I(0), I(1))]
    if op in ("Relu", "Sqrt", "Erf"):
        return [unary(op, I(0))]
    if op == "MatMul":
        return [matmul(I(0), I(1))]
    if op == "Conv":
        if honor_conv_attrs:
            # ONNX: an absent auto_pad is NOTSET, i.e. the explicit pads apply
            ap = a.get("auto_pad") or ("NOTSET" if a.get("pads") is not None else None)
            return [conv(I(0), I(1), I(2), ap, a.get("dilations"), a.get("group"),
                         a.get("kernel_shape"), a.get("pads"), a.get("strides"))]
        return [conv(I(0), I(1), I(2), a.get("auto_pad"))]
    if op == "MaxPool":
        return [maxpool(I(0), a.get("auto_pad"), None, a.get("dilations"), a.get("kernel_shape"),
                        a.get("pads"), None, a.get("strides"))]
    if op == "Softmax":
        return [softmax(I(0), a.get("axis", -1))]
    if op in ("ReduceMean", "ReduceSum", "ReduceMax"):
        if op == "ReduceMean" and opset < 13:
            axes = a["axes"]
        else:
            axes = None if I(1) is None else [int(v) for v in np.asarray(I(1)).reshape(-1)]
            if axes is None and "axes" in a:
                axes = a["axes"]
        keep = a.get("keepdims", 1)
        f = {"ReduceMean": reduce_mean, "ReduceSum": reduce_sum, "ReduceMax": reduce_max}[op]
        return [f(I(0), axes, keep)]
    if op == "Gather":
        return [gather(I(0), I(1), a.get("axis"))]
    if op == "Transpose":
        return [transpose(I(0), a.get("perm"))]
    if op == "Reshape":
        return [reshape(I(0), I(1), bool(a.get("allow_zero", 0)))]
    if op == "Unsqueeze":
        axes = a["axes"] if opset < 13 else [int(v) for v in np.asarray(I(1)).reshape(-1)]
        return [unsqueeze(I(0), axes)]
    if op == "Cast":
        return [np.asarray(I(0)).astype(_ONNX_DTYPES[int(a["to"])])]
    if op == "Constant":
        for key in ("value", "value_float", "value_floats", "value_int", "value_ints"):
            if key in a:
                v = a[key]
                dt = np.float32 if key.startswith("value_float") else (np.int64 if key.startswith("value_int") else None)
                return [np.asarray(v, dt) if dt is not None else np.asarray(v)]
        raise OracleError("The required attribute value is missing or null.")
    if op == "Shape":
        return [np.array(np.asarray(I(0)).shape, np.int64)]
    if op == "Concat":
        return [np.concatenate([np.asarray(t) for t in ins], axis=a["axis"])]
    if op == "Slice":
        return [slice_(I(0), I(1), I(2), I(3), I(4))]
    if op == "Gemm":
        return [gemm(I(0), I(1), I(2), a.get("alpha", 1.0), a.get("beta", 1.0), a.get("transA", 0),
                     a.get("transB", 0))]
    if op == "BatchNormalization":
        return [batch_norm(I(0), I(1), I(2), I(3), I(4), a.get("epsilon", 1e-5))]
    if op == "GlobalAveragePool":
        return [global_average_pool(I(0))]
    if op == "Flatten":
        return [flatten(I(0), a.get("axis", 1))]
    if op in ("Identity", "Dropout"):
        x = np.asarray(I(0))
        return [x, np.ones(x.shape, bool)]
    raise OracleError(f"The operation {op} is not supported by the backend.")


# ----------------------------------------------------------------------------
# Pre-processing before the model (src/Lokad.Onnx.Data)
# ----------------------------------------------------------------------------

def image_to_array_f(rgba):
    """Images.ImageToArrayF (Images.cs:92-103): RGBA8 [H, W, 4] ->
    float [1, 1, H, W], pixel[y, x] = ((R + G + B) / 3.0f) / 255.0f, the
    byte sum exact, each division one float32 rounding."""
    a = np.asarray(rgba, dtype=np.uint8)
    s = a[..., 0].astype(np.int32) + a[..., 1] + a[..., 2]
    px = (s.astype(np.float32) / np.float32(3.0)) / np.float32(255.0)
    return px.astype(np.float32).reshape(1, 1, a.shape[0], a.shape[1])


def roberta_pad(sequences, pad_id=1):
    """The padding loop of Text.RobertaTokenize over a string array
    (Text.cs:126-140): every sequence right-padded to the longest; input_ids
    with 1, attention_mask ones then zeros, token_type_ids zeros."""
    seqs = [list(map(int, s)) for s in sequences]
    maxl = max((len(s) for s in seqs), default=0)
    ids, mask, types = [], [], []
    for s in seqs:
        pad = maxl - len(s)
        ids.append(s + [pad_id] * pad)
        mask.append([1] * len(s) + [0] * pad)
        types.append([0] * maxl)
    shape = (len(seqs), maxl)
    return (np.array(ids, np.int64).reshape(shape), np.array(mask, np.int64).reshape(shape),
            np.array(types, np.int64).reshape(shape))


def execute(graph, inputs, honor_conv_attrs=False):
    """Run ``graph`` (nodes in file order) on ``inputs`` (name -> array).

    Tensors are resolved from inputs, then initializers, then intermediate
    outputs (ComputationalGraph.cs:39-41).  Returns a dict of graph outputs."""
    env = {}
    env.update(graph.initializers)
    env.update(inputs)

    def get(name):
        if name not in env:
            raise OracleError(f"The required input parameter {name} is missing or null.")
        return env[name]

    for node in graph.nodes:
        outs = run_node(node, get, graph.opset, honor_conv_attrs)
        for name, t in zip(node.outputs, outs):
            env[name] = t
    return {name: env[name] for name in graph.outputs}
