"""Pin the CPU oracle against the reference's own known answers (no GPU).

Sources (inside the Lokad/Onnx project):
  tests/Lokad.Onnx.Tensors.Tests/MathTests.cs:82-168  Conv2D / MaxPool2D / MatMul values
  tests/python/test_backend.py:208-220,379-442,792-876  Erf, Gather, Softmax rows
  tests/Lokad.Onnx.Backend.Tests/GraphTests.cs:15-30  mnist-8 end to end (classes 4, 2, 5)
"""
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_conv2d_known_answers():
    X = np.arange(25, dtype=np.float32).reshape(1, 1, 5, 5)
    W = np.ones((1, 1, 3, 3), np.float32)
    y = O.conv(X, W, auto_pad="NOTSET", pads=[1, 1, 1, 1])
    assert np.array_equal(y[0, 0], [[12, 21, 27, 33, 24], [33, 54, 63, 72, 51], [63, 99, 108, 117, 81],
                                    [93, 144, 153, 162, 111], [72, 111, 117, 123, 84]])
    y = O.conv(X, W, auto_pad="VALID")
    assert np.array_equal(y[0, 0], [[54, 63, 72], [99, 108, 117], [144, 153, 162]])
    X7 = np.arange(35, dtype=np.float32).reshape(1, 1, 7, 5)
    y = O.conv(X7, W, auto_pad="NOTSET", pads=[1, 1, 1, 1], strides=[2, 2])
    assert np.array_equal(y[0, 0], [[12, 27, 24], [63, 108, 81], [123, 198, 141], [112, 177, 124]])


def test_maxpool_known_answers():
    X = np.array([[[[12, 20, 30, 0], [8, 12, 2, 0], [34, 70, 37, 4], [112, 100, 25, 12]]]], np.float32)
    y = O.maxpool(X, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[2, 2])
    assert np.array_equal(y[0, 0], [[20, 30], [112, 37]])
    y = O.maxpool(X, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[1, 1])
    assert np.array_equal(y[0, 0], [[20, 30, 30], [70, 70, 37], [112, 100, 37]])


def test_matmul_known_answers():
    a = np.ones((1, 1, 5, 6), np.float32)
    assert O.matmul(a, np.ones((3, 6, 7), np.float32)).shape == (1, 3, 5, 7)
    assert O.matmul(np.ones((4, 1, 5, 6), np.float32), np.ones((4, 2, 6, 7), np.float32)).shape == (4, 2, 5, 7)
    a = np.arange(16, dtype=np.float32).reshape(2, 2, 4)
    b = np.arange(64, dtype=np.float32).reshape(2, 4, 8)
    assert O.matmul(a, b)[0, 1, 1] == 326.0
    a = np.arange(16, dtype=np.float32).reshape(2, 2, 4)
    b = np.arange(16, dtype=np.float32).reshape(2, 4, 2)
    assert O.matmul(a, b)[0, 1, 1] == 98.0


def test_softmax_known_answers():
    np.testing.assert_almost_equal(O.softmax(np.array([[-1, 0, 1]], np.float32)),
                                   [[0.09003058, 0.24472848, 0.66524094]], decimal=7)
    x = np.array([[0, 1, 2, 3], [10000, 10001, 10002, 10003]], np.float32)
    e = [0.032058604, 0.08714432, 0.23688284, 0.6439143]
    np.testing.assert_almost_equal(O.softmax(x), [e, e], decimal=7)


def test_erf_vs_math_erf():
    x = np.linspace(-4, 4, 2001).astype(np.float32)
    ref = np.array([math.erf(float(v)) for v in x])
    np.testing.assert_allclose(O.unary("Erf", x), ref, rtol=1e-6, atol=1e-6)


def test_gather_known_answers():
    x = np.random.default_rng(0).standard_normal((10, 10)).astype(np.float32)
    y = np.array([[0, 1], [1, 2]])
    assert np.array_equal(O.gather(x, y), np.take(x, y, axis=0))
    assert np.array_equal(O.gather(x, np.array([[-10, -9], [1, -8]])), np.take(x, y, axis=0))
    d = np.arange(10, dtype=np.float32)
    assert np.array_equal(O.gather(d, np.array([0, -9, -10]), 0), d[[0, 1, 0]])
    with pytest.raises(O.OracleError):
        O.gather(d, np.array([10]))


def test_mm_order_is_sequential_separate_mul_add():
    """The reference accumulates C[i,:] += A[i,j]*B[j,:] in j order with a
    separate multiply and add (MathOps.cs:380-410); the oracle must equal a
    float32 loop in that order, not an FMA or a pairwise sum."""
    rng = np.random.default_rng(1)
    A = rng.standard_normal((3, 50)).astype(np.float32)
    B = rng.standard_normal((50, 4)).astype(np.float32)
    C = np.zeros((3, 4), np.float32)
    for j in range(50):
        C = (C + (A[:, j:j + 1] * B[j:j + 1, :]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(O.matmul(A, B), C)


def test_reducemax_reference_defect():
    assert O.reduce_max(-np.ones((2, 3), np.float32), [1], 1).tolist() == [[0.0], [0.0]]


def test_mnist8_reference_model_classifies_reference_images():
    from onnx_b200 import graphs as G
    arr = dict(np.load(os.path.join(GOLDEN, "mnist8.npz")))
    g = G.from_json(os.path.join(GOLDEN, "mnist8_graph.json"), arr)
    for digit, thresh in ((4, 0.9), (2, 0.9), (5, 0.48)):
        out = O.execute(g, {"Input3": arr[f"image/mnist{digit}"]})["Plus214_Output_0"]
        p = O.softmax(out.reshape(-1))
        assert p.argmax() == digit and p[digit] > thresh


def test_mnist8_fixture_topology():
    """The committed fixture is the reference's 12-node mnist-8 graph (opset 8)."""
    import json
    g = json.load(open(os.path.join(GOLDEN, "mnist8_graph.json")))
    assert g["opset"] == 8
    assert [n["op"] for n in g["nodes"]] == ["Reshape", "Conv", "Add", "Relu", "MaxPool", "Conv", "Add", "Relu",
                                             "MaxPool", "Reshape", "MatMul", "Add"]


def test_broadcast_shape_reference_known_answers():
    """tests/Lokad.Onnx.Tensors.Tests/ShapeTests.cs:24-45 (Tensor<int>.BroadcastShape),
    through the oracle and through the library's host-side lonnx_broadcast_shape."""
    import ctypes
    cases = [((1, 1), (2,), (1, 2)), ((4, 1, 1), (2,), (4, 1, 2)), ((1, 2), (2,), (1, 2)),
             ((1, 3), (2,), None), ((4, 3, 3), (2,), None), ((2, 1), (2,), (2, 2)), ((2, 1), (2, 3), (2, 3))]
    try:
        from onnx_b200 import _native as N
    except ImportError:
        N = None
    for a, b, exp in cases:
        assert O.broadcast_shape(a, b) == exp
        if N is None:
            continue
        out = (ctypes.c_int64 * 8)()
        r = ctypes.c_int()
        rc = N.lib.lonnx_broadcast_shape(N.shape_arr(a), len(a), N.shape_arr(b), len(b), out, ctypes.byref(r))
        if exp is None:
            assert rc == -2
        else:
            assert rc == 0 and tuple(out[:r.value]) == exp


def test_reshape_reference_known_answers():
    """tests/Lokad.Onnx.Tensors.Tests/ShapeTests.cs:80-106 (Tensor<int>.Reshape):
    explicit shapes, -1 inferred, 0 copies the input dimension."""
    X = np.ones((2, 3, 4), np.int32)
    for s, exp in [([4, 2, 3], (4, 2, 3)), ([2, 4, 3], (2, 4, 3)), ([2, 12], (2, 12)), ([2, -1, 2], (2, 6, 2)),
                   ([-1, 2, 3, 4], (1, 2, 3, 4)), ([2, 0, 1, -1], (2, 3, 1, 4))]:
        assert O.reshape(X, np.array(s, np.int64)).shape == exp


def test_transpose_reference_known_answers():
    """tests/Lokad.Onnx.Tensors.Tests/ShapeTests.cs:109-120: default reverses
    the axes; an explicit permutation moves them."""
    X = np.ones((2, 3, 4), np.int32)
    assert O.transpose(X).shape[2] == 2
    t = O.transpose(X, [2, 0, 1])
    assert t.shape[0] == 4 and t.shape[2] == 3
