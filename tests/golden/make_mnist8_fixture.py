"""Generate tests/golden/mnist8.npz + mnist8_graph.json from the reference's
own test model and images (run once in a container that has the reference
checkout; the outputs are committed, the reference is not needed afterwards).

Inputs (paths within the Lokad/Onnx project):
  tests/Lokad.Onnx.Backend.Tests/models/mnist-8.onnx
  tests/Lokad.Onnx.Backend.Tests/images/mnist{4,2,5}.png

The ONNX protobuf is decoded with the library's own reader
(onnx_b200/onnx_io.py; the `onnx` package is not installed), and the model
file and the three images are copied beside the fixtures for the loader tests.  Images are converted as
src/Lokad.Onnx.Data/Images.cs:166-183 does: grayscale, resize to 28x28,
pixel = mean(R,G,B)/255.  The reference resizes with ImageSharp's default
resampler; Pillow's bicubic stands in for it (the end-to-end known answers,
GraphTests.cs:15-30, are class probabilities with wide margins).

Usage: python tests/golden/make_mnist8_fixture.py <reference_root>
"""
import json
import os
import shutil
import sys

import numpy as np


def load_model(path):
    """The model through the library's own ONNX reader (onnx_b200/onnx_io.py),
    as the node-list JSON and initializer arrays the tests load."""
    from onnx_b200 import onnx_io
    g = onnx_io.load(path)
    nodes = [{"op": n.op, "inputs": n.inputs, "outputs": n.outputs,
              "attrs": {k: (v.tolist() if isinstance(v, np.ndarray) else v) for k, v in n.attrs.items()}}
             for n in g.nodes]
    return {"opset": g.opset, "nodes": nodes, "inputs": g.inputs, "outputs": g.outputs}, g.initializers


def load_image(path):
    from PIL import Image
    im = Image.open(path).convert("RGBA").convert("L").resize((28, 28), Image.BICUBIC)
    g = np.asarray(im.convert("RGB"), dtype=np.float32)
    px = ((g[..., 0] + g[..., 1] + g[..., 2]) / 3.0) / 255.0
    return px.astype(np.float32).reshape(1, 1, 28, 28)


def main(root):
    here = os.path.dirname(os.path.abspath(__file__))
    tdir = os.path.join(root, "tests", "Lokad.Onnx.Backend.Tests")
    model = os.path.join(tdir, "models", "mnist-8.onnx")
    shutil.copyfile(model, os.path.join(here, "mnist-8.onnx"))  # the model file itself, for the loader tests
    g, inits = load_model(model)
    arrays = {"init/" + k: v for k, v in inits.items()}
    for d in (4, 2, 5):
        png = os.path.join(tdir, "images", f"mnist{d}.png")
        arrays[f"image/mnist{d}"] = load_image(png)
        shutil.copyfile(png, os.path.join(here, f"mnist{d}.png"))  # the image files, for the loader tests
    np.savez_compressed(os.path.join(here, "mnist8.npz"), **arrays)
    with open(os.path.join(here, "mnist8_graph.json"), "w") as f:
        json.dump(g, f, indent=1)
    print(json.dumps(g["nodes"], indent=None)[:2000])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_mnist8_fixture.py <root of a Lokad/Onnx checkout>")
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    main(sys.argv[1])
