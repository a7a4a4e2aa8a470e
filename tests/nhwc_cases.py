"""Graphs for the NHWC conv-chain tests (test_conv_nhwc_gpu.py), built the
same way in the test process (for the oracle) and in the child processes
that run them on the GPU with the layout pass on and off.

- resnet50_small: ResNet-50 v1 at 2 x 3 x 64 x 64 (stem, MaxPool, the 16
  bottlenecks with projection and identity residuals, the H x W mean, FC).
- mixed_readers: conv outputs read by something other than a conv chain --
  a graph output that also feeds a conv (stays NCHW), an NHWC value feeding
  a conv small enough for the direct kernel (converted back) and a
  tensor-core conv whose output must be NCHW, a MaxPool whose
  output is not NHWC-eligible (its NHWC input converted), a ReduceMax over
  {2, 3} with keepdims, a ReduceSum over channels, a Softmax.
- pool_shapes: MaxPool 3x3/2 pad 1 and 2x2/2 over NHWC values of odd
  sizes (17 x 23 -> 9 x 12 -> 4 x 6) between convs, then the H x W mean.
- projection_residual: two bottlenecks at 14 x 14 (stride-2 1x1 on both
  branches, a 3x3, residual Adds fused into the last 1x1 convs), then the
  H x W mean: the whole chain NHWC.
"""
import numpy as np

from onnx_b200 import graphs as G
from onnx_b200.graphs import GraphDef, Node


def _conv(nodes, inits, rng, name, x, cin, cout, k, s, relu=True, gamma=1.0):
    attrs = {"kernel_shape": [k, k], "strides": [s, s], "pads": [k // 2] * 4, "auto_pad": "NOTSET", "group": 1,
             "dilations": [1, 1]}
    inits[name + ".w"] = (rng.standard_normal((cout, cin, k, k)) * gamma * np.sqrt(2.0 / (cin * k * k))).astype(
        np.float32)
    inits[name + ".b"] = (rng.standard_normal(cout) * 0.01).astype(np.float32)
    nodes.append(Node("Conv", [x, name + ".w", name + ".b"], [name], attrs))
    if not relu:
        return name
    nodes.append(Node("Relu", [name], [name + ".r"]))
    return name + ".r"


def build(case):
    """(GraphDef, feed, output names) of a test case."""
    rng = np.random.default_rng(11)
    if case == "resnet50_small":
        g = G.resnet50(seed=3)
        x = rng.uniform(0, 1, (2, 3, 64, 64)).astype(np.float32)
        return g, {"data": x}, ["logits"]
    nodes, inits = [], {}
    if case == "mixed_readers":
        r1 = _conv(nodes, inits, rng, "c1", "x", 32, 64, 3, 1)
        r2 = _conv(nodes, inits, rng, "c2", r1, 64, 64, 1, 1)
        nodes.append(Node("MaxPool", [r2], ["p"], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1],
                                                   "auto_pad": "NOTSET"}))
        inits["ax1"] = np.array([1], np.int64)
        inits["ax23"] = np.array([2, 3], np.int64)
        nodes.append(Node("ReduceSum", ["p", "ax1"], ["rsum"], {"keepdims": 1}))
        nodes.append(Node("ReduceMax", [r2, "ax23"], ["gmax"], {"keepdims": 1}))
        r3 = _conv(nodes, inits, rng, "c3", r2, 64, 4, 1, 1)  # below the tensor-core size: direct kernel
        nodes.append(Node("Softmax", [r3], ["sm"], {"axis": 1}))
        r4 = _conv(nodes, inits, rng, "c4", r2, 64, 64, 3, 1)  # NHWC in, NCHW out (read by a Softmax)
        nodes.append(Node("Softmax", [r4], ["sm4"], {"axis": 1}))
        x = rng.standard_normal((2, 32, 20, 20)).astype(np.float32)
        outs = [r1, "rsum", "gmax", "sm", "sm4"]
        return GraphDef(nodes, inits, ["x"], outs, opset=18), {"x": x}, outs
    if case == "projection_residual":
        a = _conv(nodes, inits, rng, "a1", "x", 128, 64, 1, 2)
        b = _conv(nodes, inits, rng, "b1", a, 64, 64, 3, 1)
        c = _conv(nodes, inits, rng, "c1", b, 64, 256, 1, 1, relu=False, gamma=0.2)
        sc = _conv(nodes, inits, rng, "s1", "x", 128, 256, 1, 2, relu=False, gamma=0.5)
        nodes += [Node("Add", [c, sc], ["y.sum"]), Node("Relu", ["y.sum"], ["y"])]
        a = _conv(nodes, inits, rng, "a2", "y", 256, 64, 1, 1)
        b = _conv(nodes, inits, rng, "b2", a, 64, 64, 3, 1)
        c = _conv(nodes, inits, rng, "c2", b, 64, 256, 1, 1, relu=False, gamma=0.2)
        nodes += [Node("Add", [c, "y"], ["z.sum"]), Node("Relu", ["z.sum"], ["z"])]
        inits["ax23"] = np.array([2, 3], np.int64)
        nodes.append(Node("ReduceMean", ["z", "ax23"], ["gap"], {"keepdims": 0}))
        x = rng.uniform(0, 1, (4, 128, 28, 28)).astype(np.float32)
        return GraphDef(nodes, inits, ["x"], ["gap"], opset=18), {"x": x}, ["gap"]
    if case == "pool_shapes":
        a = _conv(nodes, inits, rng, "p1", "x", 32, 64, 3, 1)
        nodes.append(Node("MaxPool", [a], ["mp1"], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1],
                                                    "auto_pad": "NOTSET"}))
        b = _conv(nodes, inits, rng, "p2", "mp1", 64, 128, 1, 1)
        nodes.append(Node("MaxPool", [b], ["mp2"], {"kernel_shape": [2, 2], "strides": [2, 2], "pads": [0, 0, 0, 0],
                                                    "auto_pad": "NOTSET"}))
        c = _conv(nodes, inits, rng, "p3", "mp2", 128, 64, 3, 1)
        inits["ax23"] = np.array([2, 3], np.int64)
        nodes.append(Node("ReduceMean", [c, "ax23"], ["gap"], {"keepdims": 0}))
        x = rng.standard_normal((3, 32, 17, 23)).astype(np.float32)
        return GraphDef(nodes, inits, ["x"], ["gap"], opset=18), {"x": x}, ["gap"]
    raise ValueError(case)


def has_3x3(case):
    """Whether a 3x3 conv of the case reads an NHWC-eligible value (NCHW
    mode then transposes its input; NHWC mode does not)."""
    return case in ("resnet50_small", "projection_residual", "pool_shapes")
