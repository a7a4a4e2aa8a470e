"""Per-op parity on the GPU: every op of the path, run through the provider
(one-node graphs through liblonnx_cuda.so, the reference's run_node form,
src/interop/backend.py:149-187) and through the direct C ABI, compared with
the oracle on the same seeded inputs.  Data movement (Gather, Transpose,
Reshape, Slice, Concat) must be bit-exact; float math within
|gpu - ref| <= 1e-4 + 1e-4 |ref|."""
import numpy as np
import pytest

from conftest import close
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def P():
    from onnx_b200.provider import CUDAExecutionProvider
    return CUDAExecutionProvider


def ok(r):
    assert r.Status == "Success", r.Message
    return r.Outputs[0]


@pytest.mark.parametrize("op", ["Add", "Sub", "Mul", "Div", "Pow"])
@pytest.mark.parametrize("sa,sb", [((1, 8, 28, 28), (8, 1, 1)), ((64, 384), (384,)), ((384,), (64, 384)),
                                   ((3, 4, 5), ()), ((), (3, 4, 5)), ((2, 12, 16, 16), (2, 1, 1, 16)),
                                   ((5, 1, 7), (1, 6, 1)), ((37,), (37,)), ((4, 16, 384), (4, 16, 1)),
                                   ((4, 16, 1), (4, 16, 384)), ((3, 5, 6), (3, 1, 1)), ((3, 5, 7), (3, 5, 1))])
def test_binary_broadcast(P, op, sa, sb):
    rng = np.random.default_rng(hash((op, sa, sb)) % 2**32)
    a = rng.uniform(0.5, 2.0, sa).astype(np.float32)
    b = rng.uniform(0.5, 2.0, sb).astype(np.float32)
    if op == "Pow":
        b = np.full(sb, 2.0, np.float32)
    got = ok(getattr(P, op)(a, b))
    ref = O.binary(op, a, b)
    assert got.shape == ref.shape
    if op == "Pow":
        # x**2 is x*x rounded once on the GPU; glibc's powf (the reference's
        # MathF.Pow on Linux) is not correctly rounded, so allow 1 ulp
        np.testing.assert_array_max_ulp(got, ref, maxulp=1)
    else:
        assert np.array_equal(got, ref), "IEEE element-wise ops must match exactly"


def test_binary_incompatible(P):
    r = P.Add(np.zeros((3, 4), np.float32), np.zeros((5,), np.float32))
    assert r.Status == "Failure" and "broadcast" in r.Message


def test_binary_type_mismatch(P):
    r = P.Add(np.zeros(3, np.float32), np.zeros(3, np.int64))
    assert r.Status == "Failure"


@pytest.mark.parametrize("op", ["Relu", "Sqrt", "Erf"])
@pytest.mark.parametrize("n", [1, 5, 1000, 1 << 17])
def test_unary(P, op, n):
    rng = np.random.default_rng(n)
    x = rng.uniform(-4, 4, n).astype(np.float32)
    if op == "Sqrt":
        x = np.abs(x)
    got = ok(getattr(P, op)(x))
    ref = O.unary(op, x)
    if op == "Erf":
        close(got, ref, atol=1e-6, rtol=1e-6)
    else:
        assert np.array_equal(got, ref)


@pytest.mark.parametrize("shape,axis", [((3, 4, 5), 0), ((3, 4, 5), 1), ((3, 4, 5), 2), ((3, 4, 5), -1),
                                        ((2, 12, 128, 128), -1), ((7, 1000), -1), ((4, 2000), 1), ((1, 3), -1)])
def test_softmax(P, shape, axis):
    rng = np.random.default_rng(len(shape) * 10 + axis)
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    close(ok(P.Softmax(x, axis)), O.softmax(x, axis), atol=1e-6, rtol=1e-5)


def test_softmax_known_answers(P):
    """tests/python/test_backend.py:815-827."""
    y = ok(P.Softmax(np.array([[-1, 0, 1]], np.float32), None))
    np.testing.assert_almost_equal(y, [[0.09003058, 0.24472848, 0.66524094]], decimal=7)
    x = np.array([[0, 1, 2, 3], [10000, 10001, 10002, 10003]], np.float32)
    e = [0.032058604, 0.08714432, 0.23688284, 0.6439143]
    np.testing.assert_almost_equal(ok(P.Softmax(x, None)), [e, e], decimal=7)


@pytest.mark.parametrize("op", ["ReduceSum", "ReduceMean", "ReduceMax"])
@pytest.mark.parametrize("shape,axes,keep", [((4, 16, 384), [-1], 1), ((4, 16, 384), [1], 0), ((4, 16, 384), None, 1),
                                             ((3, 4, 5, 6), [0, 2], 1), ((3, 4, 5, 6), [3, 1], 0),
                                             ((2, 3), [0], 1)])
def test_reduce(P, op, shape, axes, keep):
    rng = np.random.default_rng(len(shape) + (len(axes) if axes else 0))
    x = rng.standard_normal(shape).astype(np.float32)
    got = ok(getattr(P, op)(x, axes, keep))
    ref = {"ReduceSum": O.reduce_sum, "ReduceMean": O.reduce_mean, "ReduceMax": O.reduce_max}[op](x, axes, keep)
    assert got.shape == ref.shape
    close(got, ref, atol=1e-5, rtol=1e-5)


def test_reducemax_starts_at_zero(P):
    """Reference defect kept for parity: ReduceMax's running max starts at 0
    (src/Lokad.Onnx.Tensors/TensorOps.cs:1820)."""
    x = -np.ones((2, 3), np.float32)
    assert np.array_equal(ok(P.ReduceMax(x, [1], 1)), np.zeros((2, 1), np.float32))


def test_conv_known_answers(P):
    """tests/Lokad.Onnx.Tensors.Tests/MathTests.cs:127-151 (ONNX Conv doc
    values), via the conv kernel with explicit pads/strides."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import Context, DeviceTensor
    ctx = Context.default(0)

    def conv(x, w, pads, stride):
        dx, dw = DeviceTensor.from_host(ctx, x), DeviceTensor.from_host(ctx, w)
        H, W = x.shape[2:]
        Ho = (H + 2 * pads - 3) // stride + 1
        Wo = (W + 2 * pads - 3) // stride + 1
        y = DeviceTensor(ctx, (1, 1, Ho, Wo), np.float32)
        N.check(N.lib.lonnx_conv2d_f32(ctx.handle, dx.ptr, dw.ptr, None, y.ptr, 1, 1, H, W, 1, 3, 3, stride, stride,
                                       pads, pads, pads, pads, 1, 1, 1, 0))
        return y.to_host()

    X = np.arange(25, dtype=np.float32).reshape(1, 1, 5, 5)
    Wt = np.ones((1, 1, 3, 3), np.float32)
    assert np.array_equal(conv(X, Wt, 1, 1)[0, 0], [[12, 21, 27, 33, 24], [33, 54, 63, 72, 51], [63, 99, 108, 117, 81],
                                                    [93, 144, 153, 162, 111], [72, 111, 117, 123, 84]])
    assert np.array_equal(conv(X, Wt, 0, 1)[0, 0], [[54, 63, 72], [99, 108, 117], [144, 153, 162]])
    X7 = np.arange(35, dtype=np.float32).reshape(1, 1, 7, 5)
    assert np.array_equal(conv(X7, Wt, 1, 2)[0, 0], [[12, 27, 24], [63, 108, 81], [123, 198, 141], [112, 177, 124]])


@pytest.mark.parametrize("xs,ws,auto_pad", [((1, 1, 28, 28), (8, 1, 5, 5), "SAME_UPPER"),
                                            ((1, 8, 14, 14), (16, 8, 5, 5), "SAME_UPPER"),
                                            ((2, 3, 9, 11), (4, 3, 3, 3), "VALID"), ((2, 3, 9, 9), (4, 3, 3, 3), None)])
def test_conv_provider_vs_oracle(P, xs, ws, auto_pad):
    rng = np.random.default_rng(xs[1] * 10 + ws[0])
    x = rng.uniform(0, 1, xs).astype(np.float32)
    w = (rng.standard_normal(ws) * 0.1).astype(np.float32)
    b = (rng.standard_normal(ws[0]) * 0.1).astype(np.float32)
    got = ok(P.Conv(x, w, b, auto_pad=auto_pad))
    ref = O.conv(x, w, b, auto_pad=auto_pad)
    assert np.array_equal(got, ref), "direct conv follows the reference summation order exactly"


def test_maxpool_known_answers(P):
    """tests/Lokad.Onnx.Tensors.Tests/MathTests.cs:154-168."""
    X = np.array([[[[12, 20, 30, 0], [8, 12, 2, 0], [34, 70, 37, 4], [112, 100, 25, 12]]]], np.float32)
    y = ok(P.MaxPool(X, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[2, 2]))
    assert np.array_equal(y[0, 0], [[20, 30], [112, 37]])
    y = ok(P.MaxPool(X, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[1, 1]))
    assert np.array_equal(y[0, 0], [[20, 30, 30], [70, 70, 37], [112, 100, 37]])


@pytest.mark.parametrize("xs,k,s,ap,pads", [((1, 8, 28, 28), 2, 2, "NOTSET", [0, 0, 0, 0]),
                                            ((1, 16, 14, 14), 3, 3, "NOTSET", [0, 0, 0, 0]),
                                            ((2, 4, 11, 11), 3, 2, "NOTSET", [1, 1, 1, 1]),
                                            ((2, 4, 10, 10), 3, 2, "SAME_UPPER", None)])
def test_maxpool_vs_oracle(P, xs, k, s, ap, pads):
    x = np.random.default_rng(k * s).standard_normal(xs).astype(np.float32)
    got = ok(P.MaxPool(x, auto_pad=ap, kernel_shape=[k, k], pads=pads, strides=[s, s]))
    ref = O.maxpool(x, auto_pad=ap, kernel_shape=[k, k], pads=pads, strides=[s, s])
    assert np.array_equal(got, ref)


def test_gather_reference_cases(P):
    """tests/python/test_backend.py:379-442, including negative indices."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((10, 10)).astype(np.float32)
    y = np.array([[0, 1], [1, 2]])
    assert np.array_equal(ok(P.Gather(x, y)), np.take(x, y, axis=0))
    assert np.array_equal(ok(P.Gather(x, np.array([[-10, -9], [1, -8]]))), np.take(x, y, axis=0))
    data = rng.standard_normal((5, 4, 3, 2)).astype(np.float32)
    for axis in (0, 1):
        assert np.array_equal(ok(P.Gather(data, np.array([0, 1, 3]), axis)), np.take(data, [0, 1, 3], axis=axis))
    d2 = rng.standard_normal((3, 3)).astype(np.float32)
    assert np.array_equal(ok(P.Gather(d2, np.array([[0, 2]]), 1)), np.take(d2, [[0, 2]], axis=1))
    d3 = np.arange(10, dtype=np.float32)
    assert np.array_equal(ok(P.Gather(d3, np.array([0, -9, -10]), 0)), np.take(d3, [0, -9, -10]))


def test_gather_embedding_rows_bit_exact(ctx):
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(2)
    table = rng.standard_normal((50000, 384)).astype(np.float32)
    idx = rng.integers(-50000, 50000, size=(32, 128)).astype(np.int64)
    dt, di = DeviceTensor.from_host(ctx, table), DeviceTensor.from_host(ctx, idx)
    y = DeviceTensor(ctx, (32, 128, 384), np.float32)
    N.check(N.lib.lonnx_gather(ctx.handle, dt.ptr, 4, 1, 50000, 384, di.ptr, idx.size, y.ptr))
    ctx.sync()
    assert np.array_equal(y.to_host(), O.gather(table, idx, 0))


def test_gather_out_of_range_reports_oob(ctx):
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    table = np.ones((10, 8), np.float32)
    idx = np.array([1, 10], np.int64)
    dt, di = DeviceTensor.from_host(ctx, table), DeviceTensor.from_host(ctx, idx)
    y = DeviceTensor(ctx, (2, 8), np.float32)
    N.check(N.lib.lonnx_gather(ctx.handle, dt.ptr, 4, 1, 10, 8, di.ptr, 2, y.ptr))
    with pytest.raises(N.LonnxError) as e:
        ctx.sync()
    assert e.value.code == -6
    ctx.sync()  # flag cleared; the context stays usable
    out = y.to_host()
    assert np.array_equal(out[0], np.ones(8)) and np.array_equal(out[1], np.zeros(8))


@pytest.mark.parametrize("shape,perm", [((2, 128, 12, 32), [0, 2, 1, 3]), ((2, 128, 12, 32), [0, 2, 3, 1]),
                                        ((3, 4), None), ((2, 3, 4, 5, 6), [4, 0, 3, 1, 2])])
def test_transpose_bit_exact(P, shape, perm):
    x = np.random.default_rng(1).standard_normal(shape).astype(np.float32)
    assert np.array_equal(ok(P.Transpose(x, perm)), O.transpose(x, perm))


_TRANSPOSE_CASES = [((2, 128, 12, 32), [0, 2, 1, 3]), ((2, 128, 12, 32), [0, 2, 3, 1]), ((33, 65), [1, 0]),
                    ((1, 5, 1, 7), [3, 2, 1, 0]), ((4, 5, 6), [0, 1, 2]), ((2, 1, 3), [2, 1, 0]),
                    ((3, 40, 7, 33), [1, 3, 0, 2]), ((2, 3, 4, 5, 6, 7), [5, 4, 3, 2, 1, 0]),
                    ((2, 2, 2, 2, 2, 2, 2, 3), [7, 6, 5, 4, 3, 2, 1, 0]), ((6, 4, 5, 3), [0, 1, 3, 2]),
                    ((7, 9, 3), [1, 0, 2])]


@pytest.mark.parametrize("dtype", [np.float32, np.uint8, np.int16, np.float64])
@pytest.mark.parametrize("shape,perm", _TRANSPOSE_CASES)
def test_transpose_c_abi_all_element_sizes(ctx, shape, perm, dtype):
    """lonnx_transpose for 1/2/4/8-byte elements: run copies (innermost axis
    kept, vectorised), 32x32 shared-memory tiles (innermost axis moved), size-1
    dimensions and merged adjacent dimensions, an identity permutation; bit-exact."""
    import ctypes
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    x = (np.random.default_rng(len(shape)).standard_normal(shape) * 100).astype(dtype)
    dx = DeviceTensor.from_host(ctx, x)
    ref = np.ascontiguousarray(np.transpose(x, perm))
    dy = DeviceTensor(ctx, ref.shape, dtype)
    sh = (ctypes.c_int64 * len(shape))(*shape)
    pm = (ctypes.c_int64 * len(perm))(*perm)
    N.check(N.lib.lonnx_transpose(ctx.handle, dx.ptr, x.itemsize, sh, len(shape), pm, dy.ptr))
    ctx.sync()
    assert np.array_equal(dy.to_host(), ref)


def test_maxpool_many_planes_and_resnet_shape(P):
    """More (n, c) planes than one grid dimension holds, and ResNet-50's
    3x3/2 pad-1 pool; bit-exact against the oracle."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 40000, 3, 3)).astype(np.float32)
    got = ok(P.MaxPool(x, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0], strides=[1, 1]))
    assert np.array_equal(got, O.maxpool(x, auto_pad="NOTSET", kernel_shape=[2, 2], pads=[0, 0, 0, 0],
                                         strides=[1, 1]))
    x = rng.standard_normal((2, 8, 112, 112)).astype(np.float32)
    got = ok(P.MaxPool(x, auto_pad="NOTSET", kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2]))
    assert np.array_equal(got, O.maxpool(x, auto_pad="NOTSET", kernel_shape=[3, 3], pads=[1, 1, 1, 1],
                                         strides=[2, 2]))


@pytest.mark.parametrize("xs,pads", [((2, 3, 9, 12), [1, 1, 1, 1]), ((1, 70, 20, 40), [1, 1, 1, 1]),
                                     ((3, 5, 16, 16), [1, 1, 1, 1]), ((1, 1, 4, 4), [1, 1, 1, 1]),
                                     ((2, 33, 7, 20), [1, 1, 1, 1])])
def test_maxpool_3x3_s2_strip_kernel(P, xs, pads):
    """The 3x3 / stride-2 / pad-1 strip kernel (W % 4 == 0, Wo == W / 2):
    odd heights, output heights that are not a multiple of the strip, column
    pairs that do not divide a warp (halo loads on lane 0, warps spanning
    strips and planes), ReLU zeros and infinities; bit-exact."""
    rng = np.random.default_rng(sum(xs))
    x = np.maximum(rng.standard_normal(xs), 0).astype(np.float32)
    x.flat[::97] = np.inf
    x.flat[5::89] = -np.inf
    got = ok(P.MaxPool(x, auto_pad="NOTSET", kernel_shape=[3, 3], pads=pads, strides=[2, 2]))
    ref = O.maxpool(x, auto_pad="NOTSET", kernel_shape=[3, 3], pads=pads, strides=[2, 2])
    assert np.array_equal(got, ref)


def test_gelu_unary_matches_node_chain(ctx):
    """The fused Erf-GELU (lonnx_unary_f32 op 4) against the exported node
    chain Div(sqrt 2) -> Erf -> Add(1) -> Mul(x) -> Mul(0.5) on the oracle,
    over a wide range including tiny, subnormal, huge and infinite inputs.
    Erf's exp differs from the host's by an ulp, hence the Erf tolerance."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(9)
    x = np.concatenate([rng.uniform(-6, 6, 1 << 16), rng.standard_normal(4096) * 1e-30,
                        np.array([0.0, -0.0, 1e-45, -1e-45, 1e-38, 3e38, -3e38, np.inf, -np.inf, 1.0, -1.0])]
                       ).astype(np.float32)
    dx = DeviceTensor.from_host(ctx, x)
    dy = DeviceTensor(ctx, x.shape, np.float32)
    N.check(N.lib.lonnx_unary_f32(ctx.handle, 4, dx.ptr, dy.ptr, x.size))
    ctx.sync()
    got = dy.to_host()
    with np.errstate(all="ignore"):
        a = x / np.float32(1.41421353816986083984375)
        e = O.unary("Erf", a)
        ref = ((x * (e + np.float32(1.0))).astype(np.float32) * np.float32(0.5)).astype(np.float32)
    fin = np.isfinite(ref)
    close(got[fin], ref[fin], atol=1e-6, rtol=1e-6)
    assert np.array_equal(np.isnan(got), np.isnan(ref))


def test_reshape_and_unsqueeze(P):
    x = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    assert ok(P.Reshape(x, np.array([0, -1], np.int64))).shape == (2, 12)
    assert ok(P.Unsqueeze(x, [0, 3])).shape == (1, 2, 3, 1, 4)
    r = P.Reshape(x, np.array([5, -1], np.int64))
    assert r.Status == "Failure"


def test_layernorm_direct(ctx):
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(4)
    for rows, cols in [(1000, 384), (7, 100), (33, 1024), (5, 3000)]:
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        r = rng.standard_normal((rows, cols)).astype(np.float32)
        gm = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
        bt = (0.1 * rng.standard_normal(cols)).astype(np.float32)
        eps = np.float32(1e-12)
        s = O.binary("Add", x, r)
        mean = O.reduce_mean(s, [-1], 1)
        d = O.binary("Sub", s, mean)
        var = O.reduce_mean(O.binary("Pow", d, np.float32(2)), [-1], 1)
        ref = O.binary("Add", O.binary("Mul", O.binary("Div", d, O.unary("Sqrt", O.binary("Add", var, eps))), gm), bt)
        dx, dr, dg, db = (DeviceTensor.from_host(ctx, a) for a in (x, r, gm, bt))
        y = DeviceTensor(ctx, (rows, cols), np.float32)
        N.check(N.lib.lonnx_layernorm_f32(ctx.handle, dx.ptr, dr.ptr, dg.ptr, db.ptr, eps, y.ptr, rows, cols))
        ctx.sync()
        close(y.to_host(), ref, atol=1e-5, rtol=1e-5)


def test_attention_direct(ctx):
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(8)
    B, S, h, dh = 3, 128, 12, 32
    H = h * dh
    qkv = rng.standard_normal((B, S, 3 * H)).astype(np.float32)
    mask = np.zeros((B, 1, 1, S), np.float32)
    mask[1, ..., 100:] = np.finfo(np.float32).min
    q, k, v = qkv[..., :H], qkv[..., H:2 * H], qkv[..., 2 * H:]
    split = lambda t, p: O.transpose(t.reshape(B, S, h, dh), p)
    s = O.matmul(split(q, [0, 2, 1, 3]), split(k, [0, 2, 3, 1]))
    p = O.softmax(O.binary("Add", O.binary("Div", s, np.float32(np.sqrt(dh))), mask), -1)
    ref = O.transpose(O.matmul(p, split(v, [0, 2, 1, 3])), [0, 2, 1, 3]).reshape(B, S, H)
    dq = DeviceTensor.from_host(ctx, qkv)
    dm = DeviceTensor.from_host(ctx, mask)
    out = DeviceTensor(ctx, (B, S, H), np.float32)
    N.check(N.lib.lonnx_attention_f32(ctx.handle, dq.ptr, dq.ptr + 4 * H, dq.ptr + 8 * H, 3 * H, dm.ptr, out.ptr,
                                      B, S, h, dh, np.float32(np.sqrt(dh))))
    ctx.sync()
    close(out.to_host(), ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("S,packed,masked", [(128, False, True), (77, True, True), (1, True, False),
                                             (100, False, False), (33, True, True)])
def test_attention_direct_shapes(ctx, S, packed, masked):
    """The TMA-fed tensor-core attention at sequence lengths below 128 (the
    128-row TMA box then reaches into the next sequence, or past the end of
    the tensor for the last one), with Q/K/V packed in one [B, S, 3H] buffer
    or in three [B, S, H] buffers, with and without the additive mask."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(S)
    B, h, dh = 5, 12, 32
    H = h * dh
    qkv = rng.standard_normal((B, S, 3 * H)).astype(np.float32)
    mask = np.zeros((B, 1, 1, S), np.float32)
    if masked:
        for bb in range(B):
            mask[bb, ..., S - rng.integers(0, S):] = np.finfo(np.float32).min
    q, k, v = qkv[..., :H], qkv[..., H:2 * H], qkv[..., 2 * H:]
    split = lambda t, p: O.transpose(t.reshape(B, S, h, dh), p)
    sc = O.matmul(split(q, [0, 2, 1, 3]), split(k, [0, 2, 3, 1]))
    sc = O.binary("Div", sc, np.float32(np.sqrt(dh)))
    if masked:
        sc = O.binary("Add", sc, mask)
    p = O.softmax(sc, -1)
    ref = O.transpose(O.matmul(p, split(v, [0, 2, 1, 3])), [0, 2, 1, 3]).reshape(B, S, H)
    out = DeviceTensor(ctx, (B, S, H), np.float32)
    dm = DeviceTensor.from_host(ctx, mask) if masked else None
    mp = dm.ptr if masked else None
    if packed:
        dq = DeviceTensor.from_host(ctx, qkv)
        args = (dq.ptr, dq.ptr + 4 * H, dq.ptr + 8 * H, 3 * H)
    else:
        dq, dk, dv = (DeviceTensor.from_host(ctx, np.ascontiguousarray(a)) for a in (q, k, v))
        args = (dq.ptr, dk.ptr, dv.ptr, H)
    N.check(N.lib.lonnx_attention_f32(ctx.handle, *args, mp, out.ptr, B, S, h, dh, np.float32(np.sqrt(dh))))
    ctx.sync()
    close(out.to_host(), ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("xs,ws,stride,pad,relu", [((4, 64, 28, 28), (128, 64, 3, 3), 1, 1, 1),
                                                   ((2, 3, 64, 64), (64, 3, 7, 7), 2, 3, 1),
                                                   ((4, 256, 14, 14), (512, 256, 1, 1), 2, 0, 0),
                                                   ((3, 32, 17, 19), (48, 32, 3, 3), 1, 1, 0),
                                                   ((8, 512, 7, 7), (2048, 512, 1, 1), 1, 0, 1),
                                                   ((5, 128, 9, 13), (72, 128, 3, 3), 2, 2, 0),
                                                   ((2, 6, 40, 40), (200, 6, 5, 5), 1, 2, 1),
                                                   ((2, 8, 30, 30), (64, 8, 9, 9), 1, 4, 0)])
def test_conv_tensor_core_path_vs_oracle(ctx, xs, ws, stride, pad, relu):
    """Convs large enough for the tensor-core implicit GEMM (rows = output
    pixels gathered from NCHW in the kernel, 3xTF32, bias + ReLU epilogue,
    NCHW written directly; 7x7 maps put several images in one row tile; the
    9x9 kernel has more taps than the tap table takes, so it gathers through
    the per-stage shuffle path)."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(xs[1] + ws[0])
    x = rng.uniform(-1, 1, xs).astype(np.float32)
    w = (rng.standard_normal(ws) * np.sqrt(2.0 / np.prod(ws[1:]))).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, ws[0]).astype(np.float32)
    ref = O.conv(x, w, b, auto_pad="NOTSET", pads=[pad] * 4, strides=[stride] * 2)
    if relu:
        ref = O.unary("Relu", ref)
    dx, dw, db = (DeviceTensor.from_host(ctx, a) for a in (x, w, b))
    y = DeviceTensor(ctx, ref.shape, np.float32)
    N.check(N.lib.lonnx_conv2d_f32(ctx.handle, dx.ptr, dw.ptr, db.ptr, y.ptr, xs[0], xs[1], xs[2], xs[3], ws[0],
                                   ws[2], ws[3], stride, stride, pad, pad, pad, pad, 1, 1, 1, relu))
    ctx.sync()
    close(y.to_host(), ref)


@pytest.mark.parametrize("dil,pads,c,k", [((2, 2), (2, 2, 2, 2), 40, 3), ((1, 3), (1, 0, 2, 3), 40, 3),
                                          ((2, 2), (2, 2, 2, 2), 64, 3), ((1, 3), (1, 0, 2, 3), 32, 5),
                                          ((1, 1), (0, 0, 0, 0), 96, 2)])
def test_conv_tensor_core_dilation_asymmetric_pads(ctx, dil, pads, c, k):
    """Dilated taps and asymmetric pads through the implicit-GEMM gather
    (from NCHW for C = 40; from the NHWC copy, tap-major weights, for C a
    multiple of 32), against a float64 direct convolution (tolerance of the
    3xTF32 GEMM)."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(11)
    n, h, w, m = 3, 23, 21, 96
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((m, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
    pt, pl, pb, pr = pads
    ho = (h + pt + pb - (dil[0] * (k - 1) + 1)) + 1
    wo = (w + pl + pr - (dil[1] * (k - 1) + 1)) + 1
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    ref = np.zeros((n, m, ho, wo))
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, :, ky * dil[0]:ky * dil[0] + ho, kx * dil[1]:kx * dil[1] + wo]
            ref += np.einsum("nchw,mc->nmhw", patch, wt[:, :, ky, kx].astype(np.float64))
    dx, dw = DeviceTensor.from_host(ctx, x), DeviceTensor.from_host(ctx, wt)
    y = DeviceTensor(ctx, (n, m, ho, wo), np.float32)
    N.check(N.lib.lonnx_conv2d_f32(ctx.handle, dx.ptr, dw.ptr, None, y.ptr, n, c, h, w, m, k, k, 1, 1, pt, pl, pb, pr,
                                   dil[0], dil[1], 1, 0))
    ctx.sync()
    close(y.to_host(), ref.astype(np.float32), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("c,k,stride,dil,pads,m", [(3, 7, 2, (1, 1), (3, 3, 3, 3), 64),
                                                   (1, 5, 1, (1, 1), (2, 2, 2, 2), 32),
                                                   (2, 3, 1, (2, 3), (1, 0, 2, 3), 96),
                                                   (4, 3, 2, (1, 1), (1, 1, 1, 1), 64),
                                                   (3, 8, 1, (1, 1), (0, 0, 0, 0), 64)])
def test_conv_few_channels_tensor_core(ctx, c, k, stride, dil, pads, m):
    """Convs of 1-4 input channels (the RGB stem's class) on the tensor-core
    implicit GEMM: K = C x taps is not a multiple of 32, so stages straddle
    channels and the last one is zero-filled past K; the 8 x 8 kernel (64
    taps) has more taps than the per-pixel validity mask holds and gathers
    through the per-stage shuffle path.  Strides, dilations and asymmetric
    pads against a float64 direct convolution at the 3xTF32 tolerance."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(c * 100 + k)
    n, h, w = 5, 45, 38
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((m, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, m).astype(np.float32)
    pt, pl, pb, pr = pads
    ho = (h + pt + pb - (dil[0] * (k - 1) + 1)) // stride + 1
    wo = (w + pl + pr - (dil[1] * (k - 1) + 1)) // stride + 1
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    ref = np.zeros((n, m, ho, wo)) + b.astype(np.float64)[None, :, None, None]
    for ky in range(k):
        for kx in range(k):
            y0, x0 = ky * dil[0], kx * dil[1]
            patch = xp[:, :, y0:y0 + stride * (ho - 1) + 1:stride, x0:x0 + stride * (wo - 1) + 1:stride]
            ref += np.einsum("nchw,mc->nmhw", patch, wt[:, :, ky, kx].astype(np.float64))
    ref = np.maximum(ref, 0.0)
    dx, dw, db = (DeviceTensor.from_host(ctx, a) for a in (x, wt, b))
    y = DeviceTensor(ctx, (n, m, ho, wo), np.float32)
    N.check(N.lib.lonnx_conv2d_f32(ctx.handle, dx.ptr, dw.ptr, db.ptr, y.ptr, n, c, h, w, m, k, k, stride, stride, pt,
                                   pl, pb, pr, dil[0], dil[1], 1, 1))
    ctx.sync()
    close(y.to_host(), ref.astype(np.float32), atol=1e-5, rtol=1e-5)
