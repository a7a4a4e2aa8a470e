"""The library's ONNX reader/writer (onnx_b200/onnx_io.py, the Model.Load
step of src/Lokad.Onnx.Backend/Model.cs:14-63): the reference's own
mnist-8.onnx decodes to the committed fixture, and every graph this
repository builds survives a write -> read round trip unchanged.  The GPU
tests load the .onnx file straight into the executor."""
import os

import numpy as np
import pytest

from onnx_b200 import graphs as G
from onnx_b200 import onnx_io

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MNIST = os.path.join(GOLDEN, "mnist-8.onnx")


def _same_graph(a, b):
    assert a.opset == b.opset and a.inputs == b.inputs and a.outputs == b.outputs
    assert len(a.nodes) == len(b.nodes)
    for x, y in zip(a.nodes, b.nodes):
        assert (x.op, x.inputs, x.outputs) == (y.op, y.inputs, y.outputs)
        assert x.attrs.keys() == y.attrs.keys()
        for k in x.attrs:
            u, v = x.attrs[k], y.attrs[k]
            if isinstance(u, np.ndarray) or isinstance(v, np.ndarray):
                assert np.array_equal(np.asarray(u), np.asarray(v)) and np.asarray(u).dtype == np.asarray(v).dtype
            elif isinstance(u, float) or (isinstance(u, list) and u and isinstance(u[0], float)):
                assert np.allclose(np.float32(u), np.float32(v), rtol=0, atol=0)
            else:
                assert u == v, (k, u, v)
    assert a.initializers.keys() == b.initializers.keys()
    for k in a.initializers:
        u, v = np.asarray(a.initializers[k]), np.asarray(b.initializers[k])
        assert u.dtype == v.dtype and u.shape == v.shape and np.array_equal(u, v), k


def test_reads_reference_mnist8_model_like_the_fixture():
    g = onnx_io.load(MNIST)
    arr = dict(np.load(os.path.join(GOLDEN, "mnist8.npz")))
    ref = G.from_json(os.path.join(GOLDEN, "mnist8_graph.json"), arr)
    _same_graph(g, ref)
    assert g.opset == 8 and len(g.nodes) == 12 and g.inputs == ["Input3"]
    assert [n.op for n in g.nodes].count("Conv") == 2


@pytest.mark.parametrize("build", ["mnist8", "e5", "resnet_onnx"])
def test_write_read_round_trip(build):
    g = {"mnist8": lambda: G.mnist8(seed=3),
         "e5": lambda: G.e5_encoder(layers=2, vocab=100, seq=16, seed=3),
         "resnet_onnx": lambda: G.resnet50(num_classes=10, seed=3, onnx_ops=True)}[build]()
    _same_graph(onnx_io.loads(onnx_io.dumps(g)), g)


def test_attribute_kinds_round_trip():
    t = np.arange(6, dtype=np.int64).reshape(2, 3)
    g = G.GraphDef([G.Node("Constant", [], ["c"], {"value": t}),
                    G.Node("Foo", ["c", ""], ["y"], {"f": 0.5, "fs": [1.5, -2.0], "i": -3, "is": [1, -1, 1 << 40],
                                                     "s": "SAME_UPPER", "ss": ["a", "b"]})],
                   {"w": np.ones((2, 2), np.float64), "b": np.array([True, False])}, ["x"], ["y"], opset=17)
    _same_graph(onnx_io.loads(onnx_io.dumps(g)), g)


def test_rejects_malformed_files():
    with pytest.raises(onnx_io.OnnxFormatError):
        onnx_io.loads(b"\x0a")              # truncated length-delimited field
    with pytest.raises(onnx_io.OnnxFormatError):
        onnx_io.loads(b"\x08\x08")          # a model with no graph
    data = open(MNIST, "rb").read()
    with pytest.raises(onnx_io.OnnxFormatError):
        onnx_io.loads(data[: len(data) // 2])


@pytest.mark.gpu
def test_gpu_runs_reference_mnist8_file(ctx):
    """The reference's mnist-8.onnx loaded by ComputationalGraph.load and run
    on the GPU gives the reference's end-to-end known answers
    (tests/Lokad.Onnx.Backend.Tests/GraphTests.cs:15-30)."""
    from onnx_b200.graph import ComputationalGraph
    from oracle import oracle as O
    cg = ComputationalGraph.load(MNIST, ctx)
    arr = dict(np.load(os.path.join(GOLDEN, "mnist8.npz")))
    for digit, thresh in ((4, 0.9), (2, 0.9), (5, 0.48)):
        out = cg.execute({"Input3": arr[f"image/mnist{digit}"]})["Plus214_Output_0"]
        p = O.softmax(out.reshape(-1))
        assert p.argmax() == digit and p[digit] > thresh


@pytest.mark.gpu
def test_gpu_file_round_trip_matches_in_memory_graph(ctx, tmp_path):
    """An e5 encoder and an ONNX-style ResNet written to .onnx files and
    loaded back run bit-identically to the in-memory graphs."""
    from onnx_b200.graph import ComputationalGraph
    e = G.e5_encoder(layers=2, vocab=2000, seq=32, seed=4)
    onnx_io.save(e, str(tmp_path / "e5.onnx"))
    inp = G.e5_inputs(3, 32, 2000, seed=4)
    a = ComputationalGraph(e, ctx).execute(inp)
    b = ComputationalGraph.load(str(tmp_path / "e5.onnx"), ctx).execute(inp)
    for k in e.outputs:
        assert np.array_equal(a[k], b[k])
    r = G.resnet50(num_classes=10, seed=4, onnx_ops=True)
    onnx_io.save(r, str(tmp_path / "r.onnx"))
    x = np.random.default_rng(4).uniform(0, 1, (1, 3, 64, 64)).astype(np.float32)
    a = ComputationalGraph(r, ctx, honor_conv_attrs=True).execute({"data": x})["logits"]
    b = ComputationalGraph.load(str(tmp_path / "r.onnx"), ctx, honor_conv_attrs=True).execute({"data": x})["logits"]
    assert np.array_equal(a, b)
