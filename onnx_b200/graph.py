"""Host-side mirror of the reference's graph API on top of the native executor.

``ComputationalGraph`` mirrors src/Lokad.Onnx.Backend/ComputationalGraph.cs
(``Execute`` :199, ``Reset`` :336, ``Outputs``), with ``provider="CUDA"``
being the only provider: every node runs through liblonnx_cuda.so's graph
executor (lonnx_graph_*), activations stay in HBM, and a host copy happens
only when an output is read.  ``run_node`` mirrors the reference's Python
backend entry ``LokadOnnxBackend.run_node`` (src/interop/backend.py:149-187):
one node wrapped into a one-node graph and executed.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .graphs import GraphDef, Node
from .tensor import Context, DeviceTensor, ONNX_DTYPE, NP_DTYPE


def _cstrs(names):
    arr = (ctypes.c_char_p * max(len(names), 1))(*[n.encode() for n in names])
    return arr


class ComputationalGraph:
    """A GraphDef loaded onto one GPU."""

    def __init__(self, graph: GraphDef, ctx: Context | None = None, fuse: bool = True,
                 honor_conv_attrs: bool = False):
        self.ctx = ctx or Context.default(0)
        self.graph = graph
        h = ctypes.c_void_p()
        N.check(N.lib.lonnx_graph_create(self.ctx.handle, ctypes.byref(h)))
        self.handle = h
        g = h
        N.check(N.lib.lonnx_graph_set_opset(g, int(graph.opset)))
        for name, arr in graph.initializers.items():
            a = np.ascontiguousarray(arr)
            if a.dtype == np.float64:
                a = a.astype(np.float32)
            shp = N.shape_arr(a.shape)
            N.check(N.lib.lonnx_graph_add_initializer(g, name.encode(), ONNX_DTYPE[a.dtype], shp, a.ndim,
                                                      a.ctypes.data))
        for node in graph.nodes:
            N.check(N.lib.lonnx_graph_add_node(g, node.op.encode(), _cstrs(node.inputs), len(node.inputs),
                                               _cstrs(node.outputs), len(node.outputs)))
            for k, v in node.attrs.items():
                if isinstance(v, str):
                    N.check(N.lib.lonnx_graph_attr_string(g, k.encode(), v.encode()))
                elif isinstance(v, float):
                    N.check(N.lib.lonnx_graph_attr_float(g, k.encode(), v))
                elif isinstance(v, (list, tuple)):
                    if v and isinstance(v[0], float):
                        raise ValueError(f"float-list attribute {k} is not supported")
                    arr = (ctypes.c_int64 * max(len(v), 1))(*[int(x) for x in v])
                    N.check(N.lib.lonnx_graph_attr_ints(g, k.encode(), arr, len(v)))
                else:
                    N.check(N.lib.lonnx_graph_attr_int(g, k.encode(), int(v)))
        for o in graph.outputs:
            N.check(N.lib.lonnx_graph_add_output(g, o.encode()))
        flags = (1 if fuse else 0) | (2 if honor_conv_attrs else 0)
        N.check(N.lib.lonnx_graph_prepare(g, flags))
        self._device_inputs = []

    @property
    def num_steps(self) -> int:
        return N.lib.lonnx_graph_num_steps(self.handle)

    def set_inputs(self, inputs: dict):
        self._device_inputs = []
        for name, val in inputs.items():
            if isinstance(val, DeviceTensor):
                shp = N.shape_arr(val.shape)
                N.check(N.lib.lonnx_graph_set_input_device(self.handle, name.encode(), ONNX_DTYPE[val.dtype], shp,
                                                           len(val.shape), val.ptr))
                self._device_inputs.append(val)
            else:
                a = np.ascontiguousarray(val)
                shp = N.shape_arr(a.shape)
                N.check(N.lib.lonnx_graph_set_input(self.handle, name.encode(), ONNX_DTYPE[a.dtype], shp, a.ndim,
                                                    a.ctypes.data))

    def run(self):
        """Enqueue one execution of the whole graph (no host synchronisation)."""
        N.check(N.lib.lonnx_graph_execute(self.handle))

    def capture(self):
        """Record one execution as a CUDA graph (inputs must already be set)."""
        N.check(N.lib.lonnx_graph_capture(self.handle))

    def replay(self):
        """Re-run the captured execution with a single graph launch."""
        N.check(N.lib.lonnx_graph_replay(self.handle))

    def output_shape(self, name):
        shp = (ctypes.c_int64 * 8)()
        r = ctypes.c_int()
        N.check(N.lib.lonnx_graph_output_shape(self.handle, name.encode(), shp, ctypes.byref(r)))
        return tuple(shp[i] for i in range(r.value))

    def output(self, name, dtype=np.float32) -> np.ndarray:
        out = np.empty(self.output_shape(name), dtype)
        N.check(N.lib.lonnx_graph_get_output(self.handle, name.encode(), out.ctypes.data, out.nbytes))
        return out

    def output_device_ptr(self, name) -> int:
        p = ctypes.c_void_p()
        N.check(N.lib.lonnx_graph_output_device(self.handle, name.encode(), ctypes.byref(p)))
        return p.value

    def execute(self, inputs: dict) -> dict:
        """ComputationalGraph.Execute: run and return the graph outputs on the host."""
        self.set_inputs(inputs)
        self.run()
        return {o: self.output(o) for o in self.graph.outputs}

    def reset(self):
        N.check(N.lib.lonnx_graph_reset(self.handle))

    def __del__(self):
        try:
            if self.handle:
                N.lib.lonnx_graph_destroy(self.handle)
        except Exception:
            pass


def run_node(node: Node, inputs: dict, ctx: Context | None = None, opset: int = 13,
             initializers: dict | None = None) -> dict:
    """Execute one node on the GPU (the reference's backend.run_node form):
    ``inputs`` maps the node's input names to host arrays; returns name -> array."""
    inits = dict(initializers or {})
    gd = GraphDef([node], inits, [n for n in node.inputs if n and n not in inits], list(node.outputs), opset)
    g = ComputationalGraph(gd, ctx, fuse=False)
    g.set_inputs({k: v for k, v in inputs.items()})
    g.run()
    res = {}
    for o in node.outputs:
        shp = g.output_shape(o)
        dt = np.float32
        # outputs keep the dtype of their producing op: integer for shape ops / int gathers
        if node.op in ("Shape",):
            dt = np.int64
        elif node.op in ("Gather", "Reshape", "Unsqueeze", "Transpose", "Concat", "Slice") and inputs:
            first = inputs.get(node.inputs[0], inits.get(node.inputs[0]))
            dt = np.asarray(first).dtype
        elif node.op == "Cast":
            dt = NP_DTYPE[int(node.attrs["to"])]
        out = np.empty(shp, dt)
        N.check(N.lib.lonnx_graph_get_output(g.handle, o.encode(), out.ctypes.data, out.nbytes))
        res[o] = out
    return res
