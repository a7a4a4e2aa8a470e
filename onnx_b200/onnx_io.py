"""ONNX model files: read a ``.onnx`` protobuf into a ``GraphDef`` and write
one back.

This is the loading step the reference performs with OnnxSharp in
``Model.Parse`` / ``Model.Load`` (src/Lokad.Onnx.Backend/Model.cs:14-63),
``TensorUtil.ToTensor`` (src/Lokad.Onnx.Backend/TensorUtil.cs:14-55) and
``NodeUtil.ToNode`` (src/Lokad.Onnx.Backend/NodeUtil.cs:9-57): nodes in file
order with their attributes, initializers as arrays, the graph's inputs
(minus those an initializer provides, as ``useInitializers`` does,
ComputationalGraph.cs:48-73) and outputs, and the default-domain opset.

The ``onnx`` Python package is not used (nor available): the protobuf wire
format is decoded and encoded here for the message fields an inference graph
needs.  Field numbers are those of onnx/onnx.proto (ModelProto, GraphProto,
NodeProto, AttributeProto, TensorProto, ValueInfoProto), a file format that
has to be matched exactly.
"""
from __future__ import annotations

import struct

import numpy as np

from .graphs import GraphDef, Node

# TensorProto.DataType -> numpy
_NP = {1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16, 6: np.int32, 7: np.int64, 9: np.bool_,
       10: np.float16, 11: np.float64, 12: np.uint32, 13: np.uint64}
_CODE = {np.dtype(v): k for k, v in _NP.items()}

# AttributeProto.AttributeType
_A_FLOAT, _A_INT, _A_STRING, _A_TENSOR, _A_FLOATS, _A_INTS, _A_STRINGS = 1, 2, 3, 4, 6, 7, 8


class OnnxFormatError(ValueError):
    pass


# ---------------------------------------------------------------------------
# wire format

def _varint(buf, i):
    shift = v = 0
    while True:
        if i >= len(buf):
            raise OnnxFormatError("truncated varint")
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if b < 0x80:
            return v, i
        shift += 7
        if shift > 70:
            raise OnnxFormatError("varint too long")


def _fields(buf):
    """(field number, wire type, value) of each field of one message."""
    i, n = 0, len(buf)
    while i < n:
        key, i = _varint(buf, i)
        fn, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(buf, i)
        elif wt == 1:
            v, i = buf[i:i + 8], i + 8
        elif wt == 2:
            ln, i = _varint(buf, i)
            v, i = buf[i:i + ln], i + ln
        elif wt == 5:
            v, i = buf[i:i + 4], i + 4
        else:
            raise OnnxFormatError(f"unsupported wire type {wt}")
        if i > n:
            raise OnnxFormatError("truncated field")
        yield fn, wt, v


def _signed(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(wt, v):
    if wt != 2:
        return [_signed(v)]
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(_signed(x))
    return out


def _floats(wt, v):
    return list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]


def _doubles(wt, v):
    return list(struct.unpack(f"<{len(v) // 8}d", v)) if wt == 2 else [struct.unpack("<d", v)[0]]


# ---------------------------------------------------------------------------
# reader

def read_tensor(buf) -> tuple[str, np.ndarray]:
    """TensorProto -> (name, array)."""
    dims, dtype, name, raw = [], 1, "", None
    f32, i32, i64, f64, u64 = [], [], [], [], []
    for fn, wt, v in _fields(buf):
        if fn == 1:
            dims += _ints(wt, v)
        elif fn == 2:
            dtype = v
        elif fn == 4:
            f32 += _floats(wt, v)
        elif fn == 5:
            i32 += _ints(wt, v)
        elif fn == 7:
            i64 += _ints(wt, v)
        elif fn == 8:
            name = bytes(v).decode()
        elif fn == 9:
            raw = bytes(v)
        elif fn == 10:
            f64 += _doubles(wt, v)
        elif fn == 11:
            u64 += _ints(wt, v)
        elif fn == 14 and v == 1:
            raise OnnxFormatError(f"tensor {name!r} stores its data externally (not supported)")
    if dtype not in _NP:
        raise OnnxFormatError(f"tensor {name!r}: unsupported data type {dtype}")
    npt = np.dtype(_NP[dtype])
    if raw is not None:
        arr = np.frombuffer(raw, dtype=npt.newbyteorder("<")).astype(npt)
    elif dtype == 1:
        arr = np.array(f32, npt)
    elif dtype == 11:
        arr = np.array(f64, npt)
    elif dtype == 7:
        arr = np.array(i64, npt)
    elif dtype in (12, 13):
        arr = np.array([x & ((1 << 64) - 1) for x in u64], npt)
    elif dtype == 10:
        arr = np.array(i32, np.uint16).view(np.float16)
    else:  # int32 and the narrower integer / bool types live in int32_data
        arr = np.array(i32, npt)
    count = int(np.prod(dims)) if dims else 1
    if arr.size != count:
        raise OnnxFormatError(f"tensor {name!r}: {arr.size} values for dims {dims}")
    return name, arr.reshape(dims)


def _read_attribute(buf):
    name, atype = "", 0
    f = i = s = t = None
    floats, ints, strings = [], [], []
    for fn, wt, v in _fields(buf):
        if fn == 1:
            name = bytes(v).decode()
        elif fn == 2:
            f = struct.unpack("<f", v)[0]
        elif fn == 3:
            i = _signed(v)
        elif fn == 4:
            s = bytes(v).decode(errors="replace")
        elif fn == 5:
            t = read_tensor(v)[1]
        elif fn == 7:
            floats += _floats(wt, v)
        elif fn == 8:
            ints += _ints(wt, v)
        elif fn == 9:
            strings.append(bytes(v).decode(errors="replace"))
        elif fn == 20:
            atype = v
    by_type = {_A_FLOAT: f, _A_INT: i, _A_STRING: s, _A_TENSOR: t, _A_FLOATS: floats, _A_INTS: ints,
               _A_STRINGS: strings}
    if atype in by_type:
        return name, by_type[atype]
    # files without the type field: take whichever value is present
    for v in (t, f, i, s):
        if v is not None:
            return name, v
    return name, floats or ints or strings


def _read_node(buf) -> Node:
    ins, outs, op, attrs = [], [], "", {}
    for fn, wt, v in _fields(buf):
        if fn == 1:
            ins.append(bytes(v).decode())
        elif fn == 2:
            outs.append(bytes(v).decode())
        elif fn == 4:
            op = bytes(v).decode()
        elif fn == 5:
            k, val = _read_attribute(v)
            attrs[k] = val
    return Node(op, ins, outs, attrs)


def _value_info_name(buf):
    for fn, wt, v in _fields(buf):
        if fn == 1:
            return bytes(v).decode()
    return ""


def loads(data: bytes) -> GraphDef:
    """Parse a serialized ModelProto."""
    buf = memoryview(data)
    graph, opset = None, None
    for fn, wt, v in _fields(buf):
        if fn == 7:
            graph = v
        elif fn == 8:
            domain, version = "", 0
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    domain = bytes(v2).decode()
                elif f2 == 2:
                    version = v2
            if domain in ("", "ai.onnx"):
                opset = version
    if graph is None:
        raise OnnxFormatError("no graph in the model")
    nodes, inits, inputs, outputs = [], {}, [], []
    for fn, wt, v in _fields(graph):
        if fn == 1:
            nodes.append(_read_node(v))
        elif fn == 5:
            k, arr = read_tensor(v)
            inits[k] = arr
        elif fn == 11:
            inputs.append(_value_info_name(v))
        elif fn == 12:
            outputs.append(_value_info_name(v))
    inputs = [n for n in inputs if n not in inits]
    return GraphDef(nodes, inits, inputs, outputs, int(opset or 13))


def load(path: str) -> GraphDef:
    """Read a ``.onnx`` file (Model.Load)."""
    with open(path, "rb") as f:
        return loads(f.read())


# ---------------------------------------------------------------------------
# writer

def _enc_varint(v):
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fn, wt):
    return _enc_varint((fn << 3) | wt)


def _f_varint(fn, v):
    return _key(fn, 0) + _enc_varint(int(v))


def _f_bytes(fn, b):
    b = b.encode() if isinstance(b, str) else bytes(b)
    return _key(fn, 2) + _enc_varint(len(b)) + b


def _f_float(fn, v):
    return _key(fn, 5) + struct.pack("<f", float(v))


def write_tensor(name: str, arr: np.ndarray) -> bytes:
    """array -> TensorProto (dims, data_type, name, raw_data little-endian)."""
    a = np.asarray(arr)  # (ascontiguousarray would turn a 0-d scalar into shape [1])
    if not a.flags.c_contiguous:
        a = a.copy()
    if a.dtype not in _CODE:
        raise OnnxFormatError(f"tensor {name!r}: unsupported dtype {a.dtype}")
    out = b"".join(_f_varint(1, d) for d in a.shape)
    out += _f_varint(2, _CODE[a.dtype]) + _f_bytes(8, name)
    out += _f_bytes(9, a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())
    return out


def _write_attribute(name, v) -> bytes:
    out = _f_bytes(1, name)
    if isinstance(v, np.ndarray):
        return out + _f_bytes(5, write_tensor("", v)) + _f_varint(20, _A_TENSOR)
    if isinstance(v, str):
        return out + _f_bytes(4, v) + _f_varint(20, _A_STRING)
    if isinstance(v, (bool, int, np.integer)):
        return out + _f_varint(3, int(v)) + _f_varint(20, _A_INT)
    if isinstance(v, (float, np.floating)):
        return out + _f_float(2, v) + _f_varint(20, _A_FLOAT)
    if isinstance(v, (list, tuple)):
        if v and all(isinstance(x, str) for x in v):
            return out + b"".join(_f_bytes(9, x) for x in v) + _f_varint(20, _A_STRINGS)
        if v and any(isinstance(x, (float, np.floating)) for x in v):
            packed = struct.pack(f"<{len(v)}f", *[float(x) for x in v])
            return out + _f_bytes(7, packed) + _f_varint(20, _A_FLOATS)
        packed = b"".join(_enc_varint(int(x)) for x in v)
        return out + _f_bytes(8, packed) + _f_varint(20, _A_INTS)
    raise OnnxFormatError(f"attribute {name!r}: unsupported value {type(v).__name__}")


def _write_value_info(name, arr=None) -> bytes:
    out = _f_bytes(1, name)
    if arr is not None:
        dims = b"".join(_f_bytes(1, _f_varint(1, d)) for d in arr.shape)
        tt = _f_varint(1, _CODE[np.dtype(arr.dtype)]) + _f_bytes(2, dims)
        out += _f_bytes(2, _f_bytes(1, tt))
    return out


def dumps(g: GraphDef, name: str = "graph", producer: str = "onnx_b200") -> bytes:
    """Serialize a GraphDef as a ModelProto (IR version 8, default-domain opset g.opset)."""
    graph = b""
    for i, n in enumerate(g.nodes):
        node = b"".join(_f_bytes(1, x) for x in n.inputs) + b"".join(_f_bytes(2, x) for x in n.outputs)
        node += _f_bytes(3, f"{n.op}_{i}") + _f_bytes(4, n.op)
        node += b"".join(_f_bytes(5, _write_attribute(k, v)) for k, v in n.attrs.items())
        graph += _f_bytes(1, node)
    graph += _f_bytes(2, name)
    for k, arr in g.initializers.items():
        graph += _f_bytes(5, write_tensor(k, np.asarray(arr)))
    for k in g.inputs:
        graph += _f_bytes(11, _write_value_info(k))
    for k in g.outputs:
        graph += _f_bytes(12, _write_value_info(k))
    opset = _f_bytes(1, "") + _f_varint(2, g.opset)
    return _f_varint(1, 8) + _f_bytes(2, producer) + _f_bytes(7, graph) + _f_bytes(8, opset)


def save(g: GraphDef, path: str, name: str = "graph") -> None:
    with open(path, "wb") as f:
        f.write(dumps(g, name))
