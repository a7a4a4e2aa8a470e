"""The ONNX ops the reference names but does not dispatch (Gemm,
BatchNormalization, GlobalAveragePool, Flatten; OpType.cs:17,51,57,58 vs
CPUExecutionProvider.cs:24-50), plus Identity/Dropout and tensor-valued
Constant, on the GPU against the oracle's ONNX-spec restatement -- as single
nodes, inside fused graphs (Gemm as one GEMM step, Conv + BatchNormalization
folded at prepare), and as a whole ONNX-style ResNet-50."""
import numpy as np
import pytest

from conftest import close
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _graph(nodes, inits, inputs, outputs, opset=13):
    from onnx_b200.graphs import GraphDef
    return GraphDef(nodes, inits, inputs, outputs, opset)


C_SHAPES = {"none": None, "row": lambda m, n: (n,), "row2d": lambda m, n: (1, n), "full": lambda m, n: (m, n),
            "col": lambda m, n: (m, 1), "scalar": lambda m, n: ()}


@pytest.mark.parametrize("c_kind", list(C_SHAPES))
@pytest.mark.parametrize("ta,tb,alpha,beta", [(0, 0, 1.0, 1.0), (0, 1, 1.0, 1.0), (1, 0, 0.5, 2.0), (1, 1, 1.0, 0.25)])
@pytest.mark.parametrize("c_init", [True, False])
def test_gemm_node_vs_oracle(ctx, c_kind, ta, tb, alpha, beta, c_init):
    """Gemm with every transpose / alpha / beta combination and every C shape
    ONNX allows to broadcast, C as an initializer (the fused GEMM step when it
    is a row bias and alpha = 1, transA = 0) or as a graph input (the node
    kernel).  Large enough (256 x 384 x 320) for the tensor-core path."""
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    rng = np.random.default_rng(ta * 8 + tb * 4 + int(c_init))
    M, K, N = 256, 384, 320
    a = rng.uniform(-1, 1, (K, M) if ta else (M, K)).astype(np.float32)
    w = rng.uniform(-1, 1, (N, K) if tb else (K, N)).astype(np.float32)
    inits = {"w": w}
    feeds = {"a": a}
    ins = ["a", "w"]
    if C_SHAPES[c_kind] is not None:
        c = rng.uniform(-1, 1, C_SHAPES[c_kind](M, N)).astype(np.float32)
        (inits if c_init else feeds)["c"] = c
        ins.append("c")
    g = _graph([Node("Gemm", ins, ["y"], {"alpha": alpha, "beta": beta, "transA": ta, "transB": tb})], inits,
               list(feeds), ["y"])
    cg = ComputationalGraph(g, ctx)
    fused = c_init and ta == 0 and alpha == 1.0 and c_kind in ("none", "row", "row2d")
    got = cg.execute(feeds)["y"]
    ref = O.execute(g, feeds)["y"]
    close(got, ref)
    if fused:
        assert cg.num_steps == 1


def test_gemm_small_node_bit_exact(ctx):
    """Below the tensor-core threshold Gemm runs the exact-order FFMA kernel:
    bit-exact against the oracle (the reference's GEMM summation order)."""
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (4, 2048)).astype(np.float32)
    w = rng.uniform(-1, 1, (10, 2048)).astype(np.float32)
    c = rng.uniform(-1, 1, 10).astype(np.float32)
    g = _graph([Node("Gemm", ["a", "w", "c"], ["y"], {"transB": 1})], {"w": w, "c": c}, ["a"], ["y"])
    got = ComputationalGraph(g, ctx, fuse=False).execute({"a": a})["y"]
    assert np.array_equal(got, O.execute(g, {"a": a})["y"])


@pytest.mark.parametrize("shape", [(2, 64, 28, 28), (3, 16, 7, 5), (4, 32), (2, 8, 3, 3, 3)])
def test_batchnorm_node_bit_exact(ctx, shape):
    """Unfused BatchNormalization computes the ONNX formula with each step
    rounded once in order: bit-exact against the oracle's float32 numpy."""
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    rng = np.random.default_rng(len(shape))
    C = shape[1]
    x = rng.standard_normal(shape).astype(np.float32)
    params = {"s": rng.uniform(0.5, 1.5, C), "b": rng.standard_normal(C), "m": rng.standard_normal(C) * 0.3,
              "v": rng.uniform(0.2, 2.0, C)}
    params = {k: v.astype(np.float32) for k, v in params.items()}
    g = _graph([Node("BatchNormalization", ["x", "s", "b", "m", "v"], ["y"], {"epsilon": 1e-3})], params, ["x"],
               ["y"])
    got = ComputationalGraph(g, ctx).execute({"x": x})["y"]
    assert np.array_equal(got, O.execute(g, {"x": x})["y"])


@pytest.mark.parametrize("with_bias,relu,residual", [(False, True, False), (True, False, False),
                                                     (False, True, True)])
def test_conv_batchnorm_fold_vs_oracle(ctx, with_bias, relu, residual):
    """Conv -> BatchNormalization [-> Add(residual)] [-> Relu]: the BN is
    folded into the conv's weights and bias at prepare, then the conv fuses
    the residual and the Relu -- within the parity tolerance of the
    unfolded chain."""
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    rng = np.random.default_rng(7)
    M, C = 128, 64
    inits = {"w": (rng.standard_normal((M, C, 3, 3)) / 24).astype(np.float32),
             "s": rng.uniform(0.5, 1.5, M).astype(np.float32), "B": rng.standard_normal(M).astype(np.float32) * 0.1,
             "m": rng.standard_normal(M).astype(np.float32) * 0.1, "v": rng.uniform(0.5, 1.5, M).astype(np.float32)}
    cin = ["x", "w"]
    if with_bias:
        inits["cb"] = rng.standard_normal(M).astype(np.float32) * 0.1
        cin.append("cb")
    nodes = [Node("Conv", cin, ["c"], {"pads": [1, 1, 1, 1], "kernel_shape": [3, 3]}),
             Node("BatchNormalization", ["c", "s", "B", "m", "v"], ["bn"], {"epsilon": 1e-5})]
    last = "bn"
    feeds = {"x": rng.uniform(-1, 1, (2, C, 20, 20)).astype(np.float32)}
    if residual:
        feeds["r"] = rng.uniform(-1, 1, (2, M, 20, 20)).astype(np.float32)
        nodes.append(Node("Add", ["bn", "r"], ["sum"]))
        last = "sum"
    if relu:
        nodes.append(Node("Relu", [last], ["y"]))
        last = "y"
    g = _graph(nodes, inits, list(feeds), [last])
    cg = ComputationalGraph(g, ctx, honor_conv_attrs=True)
    assert cg.num_steps == 1, "Conv + BN (+ Add + Relu) should be one step"
    got = cg.execute(feeds)[last]
    ref = O.execute(g, feeds, honor_conv_attrs=True)[last]
    close(got, ref)


def test_global_avg_pool_flatten_identity_dropout(ctx):
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 2048, 7, 7)).astype(np.float32)
    nodes = [Node("Identity", ["x"], ["i"]), Node("GlobalAveragePool", ["i"], ["p"]),
             Node("Dropout", ["p"], ["d"]), Node("Flatten", ["d"], ["f"], {"axis": 1})]
    g = _graph(nodes, {}, ["x"], ["p", "f"])
    got = ComputationalGraph(g, ctx).execute({"x": x})
    ref = O.execute(g, {"x": x})
    assert got["p"].shape == (4, 2048, 1, 1) and got["f"].shape == (4, 2048)
    close(got["p"], ref["p"])
    close(got["f"], ref["f"])


def test_constant_tensor_and_float_list_attributes(ctx):
    """Constant with a TENSOR attribute (float and int64) and value_floats."""
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import Node
    t = np.arange(12, dtype=np.float32).reshape(3, 4) / 7
    nodes = [Node("Constant", [], ["c"], {"value": t}),
             Node("Constant", [], ["s"], {"value": np.array([4, 3], np.int64)}),
             Node("Constant", [], ["f"], {"value_floats": [0.5, 1.5, 2.5, 3.5]}),
             Node("Add", ["x", "c"], ["y0"]), Node("Mul", ["y0", "f"], ["y1"]),
             Node("Reshape", ["y1", "s"], ["y"])]
    g = _graph(nodes, {}, ["x"], ["y", "s"])
    x = np.ones((3, 4), np.float32)
    got = ComputationalGraph(g, ctx).execute({"x": x})
    assert got["s"].dtype == np.int64 and list(got["s"]) == [4, 3]
    assert np.array_equal(got["y"], ((x + t) * np.array([0.5, 1.5, 2.5, 3.5], np.float32)).reshape(4, 3))


@pytest.mark.parametrize("fuse", [True, False])
def test_resnet50_onnx_ops_vs_oracle(ctx, fuse):
    """ResNet-50 laid out as an ONNX export: Conv (no bias) ->
    BatchNormalization -> Relu, GlobalAveragePool, Flatten, Gemm(transB=1).
    Fused: every BN folded into its conv; unfused: every node on its own
    kernel.  Both against the oracle's node-by-node ONNX semantics."""
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    g = G.resnet50(seed=2, onnx_ops=True)
    x = np.random.default_rng(2).uniform(0, 1, (2, 3, 96, 96)).astype(np.float32)
    cg = ComputationalGraph(g, ctx, fuse=fuse, honor_conv_attrs=True)
    got = cg.execute({"data": x})["logits"]
    ref = O.execute(g, {"data": x}, honor_conv_attrs=True)["logits"]
    close(got, ref)
    if fuse:
        assert cg.num_steps < len(g.nodes) // 2


def test_provider_shape_ops_return_op_results():
    """CUDAExecutionProvider's Constant/Cast/Concat/Shape/Slice (the five the
    CPU provider has at CPUExecutionProvider.cs:435-600) return OpResults
    with the oracle's values, and failures instead of exceptions."""
    from onnx_b200.provider import CUDAExecutionProvider as P
    x = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    r = P.Constant(x)
    assert r.Status == "Success" and np.array_equal(r.Outputs[0], x)
    r = P.Constant(2.5)
    assert r.Status == "Success" and float(r.Outputs[0]) == 2.5
    r = P.Constant([1, 2, 3])
    assert r.Outputs[0].dtype == np.int64 and list(r.Outputs[0]) == [1, 2, 3]
    r = P.Cast(np.array([[1, -2], [3, 4]], np.int64), 1)
    assert r.Status == "Success" and r.Outputs[0].dtype == np.float32 and r.Outputs[0][0, 1] == -2.0
    r = P.Concat([x, x + 1], 1)
    assert np.array_equal(r.Outputs[0], np.concatenate([x, x + 1], 1))
    r = P.Shape(x)
    assert list(r.Outputs[0]) == [2, 3, 4]
    r = P.Shape(x, 1, -1)
    assert list(r.Outputs[0]) == [3]
    st, en, ax, sp = (np.array(v, np.int64) for v in ([0, 3], [2, 0], [1, 2], [1, -1]))
    r = P.Slice(x, st, en, ax, sp)
    assert r.Status == "Success"
    assert np.array_equal(r.Outputs[0], O.slice_(x, st, en, ax, sp))
    bad = P.Slice(x, np.array([[0]], np.int64), np.array([1], np.int64), None, None)
    assert bad.Status == "Failure" and "rank of the starts tensor must be 1" in bad.Message
    assert P.Concat(None).Status == "Failure"
    assert P.Concat([x, x.astype(np.int64)], 0).Status == "Failure"


def test_provider_onnx_ops_vs_oracle():
    from onnx_b200.provider import CUDAExecutionProvider as P
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (8, 16)).astype(np.float32)
    b = rng.uniform(-1, 1, (12, 16)).astype(np.float32)
    c = rng.uniform(-1, 1, 12).astype(np.float32)
    r = P.Gemm(a, b, c, transB=1)
    assert r.Status == "Success"
    close(r.Outputs[0], O.gemm(a, b, c, trans_b=1))
    x = rng.standard_normal((2, 4, 3, 3)).astype(np.float32)
    p = [rng.uniform(0.5, 1.5, 4).astype(np.float32) for _ in range(4)]
    r = P.BatchNormalization(x, *p)
    assert np.array_equal(r.Outputs[0], O.batch_norm(x, *p))
    r = P.GlobalAveragePool(x)
    close(r.Outputs[0], O.global_average_pool(x))
    assert P.Flatten(x, 2).Outputs[0].shape == (8, 9)
    assert P.Gemm(a, None).Status == "Failure"


def test_provider_conv_honours_explicit_attributes():
    """CPUExecutionProvider.Conv applies the strides/kernel_shape it is given
    and reads pads only with auto_pad NOTSET (CPUExecutionProvider.cs:237-291)."""
    from onnx_b200.provider import CUDAExecutionProvider as P
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (1, 3, 11, 11)).astype(np.float32)
    w = rng.uniform(-1, 1, (4, 3, 3, 3)).astype(np.float32)
    r = P.Conv(x, w, None, "NOTSET", None, None, [3, 3], [1, 1, 1, 1], [2, 2])
    ref = O.conv(x, w, None, "NOTSET", None, None, [3, 3], [1, 1, 1, 1], [2, 2])
    assert r.Status == "Success" and r.Outputs[0].shape == ref.shape == (1, 4, 6, 6)
    assert np.array_equal(r.Outputs[0], ref)
    r = P.Conv(x, w, None, None, None, None, None, [1, 1, 1, 1], [2, 2])  # pads ignored without NOTSET
    assert r.Outputs[0].shape == O.conv(x, w, None, None, None, None, None, None, [2, 2]).shape == (1, 4, 5, 5)
    assert P.Conv(x, w, None, "NOTSET", None, None, None, [1, 0, 1, 0], None).Status == "Failure"
