"""Generate tests/golden/mnist8.npz + mnist8_graph.json from the reference's
own test model and images (run once in a container that has the reference
checkout; the outputs are committed, the reference is not needed afterwards).

Inputs (paths within the Lokad/Onnx project):
  tests/Lokad.Onnx.Backend.Tests/models/mnist-8.onnx
  tests/Lokad.Onnx.Backend.Tests/images/mnist{4,2,5}.png

The ONNX protobuf is decoded with a minimal wire-format reader written here
(the `onnx` package is not installed).  Images are converted as
src/Lokad.Onnx.Data/Images.cs:166-183 does: grayscale, resize to 28x28,
pixel = mean(R,G,B)/255.  The reference resizes with ImageSharp's default
resampler; Pillow's bicubic stands in for it (the end-to-end known answers,
GraphTests.cs:15-30, are class probabilities with wide margins).

Usage: python tests/golden/make_mnist8_fixture.py <reference_root>
"""
import json
import os
import struct
import sys

import numpy as np


def _varint(buf, i):
    shift = 0
    v = 0
    while True:
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if b < 0x80:
            return v, i
        shift += 7


def fields(buf):
    """Yield (field_number, wire_type, value) of one protobuf message."""
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        fn, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(buf, i)
        elif wt == 1:
            v = buf[i:i + 8]
            i += 8
        elif wt == 2:
            n, i = _varint(buf, i)
            v = buf[i:i + n]
            i += n
        elif wt == 5:
            v = buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"wire type {wt}")
        yield fn, wt, v


def _packed_varints(v):
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        if x >= 1 << 63:
            x -= 1 << 64
        out.append(x)
    return out


def tensor(buf):
    """TensorProto -> (name, ndarray): dims=1, data_type=2, float_data=4,
    int64_data=7, name=8, raw_data=9."""
    dims, dtype, name, raw, fdata, idata = [], 1, "", None, [], []
    for fn, wt, v in fields(buf):
        if fn == 1:
            dims += _packed_varints(v) if wt == 2 else [v]
        elif fn == 2:
            dtype = v
        elif fn == 8:
            name = v.decode()
        elif fn == 9:
            raw = bytes(v)
        elif fn == 4:
            fdata += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif fn == 7:
            idata += _packed_varints(v) if wt == 2 else [v]
    npt = {1: np.float32, 7: np.int64, 6: np.int32}[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=npt).copy()
    else:
        arr = np.array(fdata if dtype == 1 else idata, dtype=npt)
    return name, arr.reshape(dims)


def attribute(buf):
    """AttributeProto: name=1, f=2, i=3, s=4, t=5, floats=7, ints=8, type=20."""
    name, val, ints, floats = "", None, [], []
    for fn, wt, v in fields(buf):
        if fn == 1:
            name = v.decode()
        elif fn == 2:
            val = struct.unpack("<f", v)[0]
        elif fn == 3:
            val = v - (1 << 64) if v >= 1 << 63 else v
        elif fn == 4:
            val = v.decode()
        elif fn == 5:
            val = tensor(v)[1].tolist()
        elif fn == 7:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif fn == 8:
            ints += _packed_varints(v) if wt == 2 else [v]
    if ints:
        val = ints
    if floats:
        val = floats
    return name, val


def load_model(path):
    buf = open(path, "rb").read()
    opset = 0
    graph = None
    for fn, wt, v in fields(buf):
        if fn == 7:
            graph = v
        elif fn == 8:  # opset_import
            for f2, _, v2 in fields(v):
                if f2 == 2:
                    opset = v2
    nodes, inits, inputs, outputs = [], {}, [], []
    for fn, wt, v in fields(graph):
        if fn == 1:
            node = {"op": "", "inputs": [], "outputs": [], "attrs": {}}
            for f2, _, v2 in fields(v):
                if f2 == 1:
                    node["inputs"].append(v2.decode())
                elif f2 == 2:
                    node["outputs"].append(v2.decode())
                elif f2 == 4:
                    node["op"] = v2.decode()
                elif f2 == 5:
                    k, val = attribute(v2)
                    node["attrs"][k] = val
            nodes.append(node)
        elif fn == 5:
            k, arr = tensor(v)
            inits[k] = arr
        elif fn in (11, 12):
            for f2, _, v2 in fields(v):
                if f2 == 1:
                    (inputs if fn == 11 else outputs).append(v2.decode())
    inputs = [n for n in inputs if n not in inits]
    return {"opset": opset, "nodes": nodes, "inputs": inputs, "outputs": outputs}, inits


def load_image(path):
    from PIL import Image
    im = Image.open(path).convert("RGBA").convert("L").resize((28, 28), Image.BICUBIC)
    g = np.asarray(im.convert("RGB"), dtype=np.float32)
    px = ((g[..., 0] + g[..., 1] + g[..., 2]) / 3.0) / 255.0
    return px.astype(np.float32).reshape(1, 1, 28, 28)


def main(root):
    here = os.path.dirname(os.path.abspath(__file__))
    tdir = os.path.join(root, "tests", "Lokad.Onnx.Backend.Tests")
    g, inits = load_model(os.path.join(tdir, "models", "mnist-8.onnx"))
    arrays = {"init/" + k: v for k, v in inits.items()}
    for d in (4, 2, 5):
        arrays[f"image/mnist{d}"] = load_image(os.path.join(tdir, "images", f"mnist{d}.png"))
    np.savez_compressed(os.path.join(here, "mnist8.npz"), **arrays)
    with open(os.path.join(here, "mnist8_graph.json"), "w") as f:
        json.dump(g, f, indent=1)
    print(json.dumps(g["nodes"], indent=None)[:2000])


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
