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


def _set_attr(g, k, v):
    """One attribute of the last added node, by Python type: str, float,
    int, list of ints / floats, or a numpy array (a TENSOR attribute)."""
    name = k.encode()
    if isinstance(v, str):
        N.check(N.lib.lonnx_graph_attr_string(g, name, v.encode()))
    elif isinstance(v, np.ndarray):
        a = np.ascontiguousarray(v)
        if a.dtype == np.float64:
            a = a.astype(np.float32)
        N.check(N.lib.lonnx_graph_attr_tensor(g, name, ONNX_DTYPE[a.dtype], N.shape_arr(a.shape), a.ndim,
                                              a.ctypes.data))
    elif isinstance(v, (float, np.floating)):
        N.check(N.lib.lonnx_graph_attr_float(g, name, float(v)))
    elif isinstance(v, (list, tuple)):
        if v and isinstance(v[0], (float, np.floating)):
            arr = (ctypes.c_float * len(v))(*[float(x) for x in v])
            N.check(N.lib.lonnx_graph_attr_floats(g, name, arr, len(v)))
        else:
            arr = (ctypes.c_int64 * max(len(v), 1))(*[int(x) for x in v])
            N.check(N.lib.lonnx_graph_attr_ints(g, name, arr, len(v)))
    else:
        N.check(N.lib.lonnx_graph_attr_int(g, name, int(v)))


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
                _set_attr(g, k, v)
        for o in graph.outputs:
            N.check(N.lib.lonnx_graph_add_output(g, o.encode()))
        flags = (1 if fuse else 0) | (2 if honor_conv_attrs else 0)
        N.check(N.lib.lonnx_graph_prepare(g, flags))
        self._device_inputs = []

    @classmethod
    def load(cls, path: str, ctx: Context | None = None, **kw) -> "ComputationalGraph":
        """Model.Load (src/Lokad.Onnx.Backend/Model.cs:30-63): read a .onnx
        file and load its graph onto the GPU."""
        from . import onnx_io
        return cls(onnx_io.load(path), ctx, **kw)

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

    def output_dtype(self, name) -> np.dtype:
        d = ctypes.c_int()
        N.check(N.lib.lonnx_graph_output_dtype(self.handle, name.encode(), ctypes.byref(d)))
        return NP_DTYPE[d.value]

    def output(self, name, dtype=None) -> np.ndarray:
        out = np.empty(self.output_shape(name), dtype or self.output_dtype(name))
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
             initializers: dict | None = None, honor_conv_attrs: bool = False) -> dict:
    """Execute one node on the GPU (the reference's backend.run_node form):
    ``inputs`` maps the node's input names to host arrays; returns name -> array
    (each output in the element type the executor produced)."""
    inits = dict(initializers or {})
    outs = [o for o in node.outputs if o]
    gd = GraphDef([node], inits, [n for n in node.inputs if n and n not in inits], outs, opset)
    g = ComputationalGraph(gd, ctx, fuse=False, honor_conv_attrs=honor_conv_attrs)
    g.set_inputs({k: v for k, v in inputs.items()})
    g.run()
    return {o: g.output(o) for o in outs}
