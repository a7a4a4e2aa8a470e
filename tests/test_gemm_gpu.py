"""GEMM / MatMul parity on the GPU, through the C ABI (lonnx_gemm_f32,
lonnx_matmul_f32), against the oracle's restatement of the reference's
mm_unsafe_vectorized (src/Lokad.Onnx.Tensors/MathOps.cs:380-410) and, for the
largest benchmark shape, against a float64 product (the oracle would take
minutes there).  Tolerance: |gpu - ref| <= 1e-4 + 1e-4 |ref|."""
import ctypes

import numpy as np
import pytest

from conftest import close
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _gemm(ctx, A, B, bias=None, transB=0, epi=0, alpha=1.0, beta=1.0, batch=1, sA=0, sB=0, sC=0, M=None,
          N=None, K=None):
    from onnx_b200 import _native as N_
    from onnx_b200.tensor import DeviceTensor
    dA = DeviceTensor.from_host(ctx, A)
    dB = DeviceTensor.from_host(ctx, B)
    db = DeviceTensor.from_host(ctx, bias) if bias is not None else None
    M = M or A.shape[-2]
    K = K or A.shape[-1]
    N = N or (B.shape[-2] if transB else B.shape[-1])
    out = DeviceTensor(ctx, (batch, M, N) if batch > 1 else (M, N), np.float32)
    N_.check(N_.lib.lonnx_gemm_f32(ctx.handle, dA.ptr, dB.ptr, db.ptr if db else None, out.ptr, batch, M, N, K,
                                   sA, sB, sC, transB, alpha, beta, epi))
    ctx.sync()
    return out.to_host()


SWEEP = [(128, 384, 384), (4096, 384, 1536), (4096, 1536, 384)]


@pytest.mark.parametrize("M,K,N", SWEEP)
@pytest.mark.parametrize("transB", [0, 1])
def test_gemm_sweep_vs_oracle(ctx, M, K, N, transB):
    rng = np.random.default_rng(M + K + N + transB)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    ref = O.binary("Add", O.matmul(A, B), bias)  # MatMul node then Add node
    got = _gemm(ctx, A, np.ascontiguousarray(B.T) if transB else B, bias, transB=transB)
    close(got, ref)


def test_gemm_largest_vs_fp64(ctx):
    M, K, N = 8192, 1024, 4096
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    ref = A.astype(np.float64) @ B.astype(np.float64) + bias
    got = _gemm(ctx, A, np.ascontiguousarray(B.T), bias, transB=1)
    close(got, ref)


@pytest.mark.parametrize("M,K,N", [(1, 4, 1), (3, 5, 7), (130, 36, 200), (257, 300, 129), (1000, 64, 1000),
                                   (300, 1028, 260)])
def test_gemm_ragged_shapes(ctx, M, K, N):
    """Shapes that are not tile multiples (TMA zero fill, masked epilogue) and
    unaligned K (FFMA path)."""
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    ref = O.matmul(A, B)
    got = _gemm(ctx, A, B, None)
    close(got, ref)


def test_gemm_small_is_bit_exact(ctx):
    """Small GEMMs run the FFMA kernel in the reference's summation order."""
    rng = np.random.default_rng(3)
    A = rng.standard_normal((5, 256)).astype(np.float32)
    B = rng.standard_normal((256, 10)).astype(np.float32)
    assert np.array_equal(_gemm(ctx, A, B), O.matmul(A, B))


def test_gemm_gelu_epilogue(ctx):
    rng = np.random.default_rng(11)
    M, K, N = 1024, 384, 1536
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N) * 0.05).astype(np.float32)
    y = O.binary("Add", O.matmul(A, W), b)
    # the exported GELU node chain, step by step in the oracle
    ref = O.binary("Mul", O.binary("Mul", y, O.binary("Add", O.unary("Erf", O.binary("Div", y, np.float32(np.sqrt(2)))),
                                                       np.float32(1))), np.float32(0.5))
    got = _gemm(ctx, A, np.ascontiguousarray(W.T), b, transB=1, epi=2)
    close(got, ref)


def test_gemm_tensor_core_accuracy_3xtf32(ctx):
    """3xTF32 must be far more accurate than a single TF32 product: error
    against float64 stays at fp32 level over K = 1536."""
    rng = np.random.default_rng(5)
    M, K, N = 2048, 1536, 512
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    got = _gemm(ctx, A, np.ascontiguousarray(B.T), transB=1)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel < 2e-6, rel


def test_matmul_batched_broadcast(ctx):
    from onnx_b200 import _native as N_
    from onnx_b200.tensor import DeviceTensor
    rng = np.random.default_rng(1)
    for sa, sb in [((4, 1, 5, 6), (4, 2, 6, 7)), ((2, 3, 5, 6), (3, 6, 7)), ((1, 1, 5, 6), (3, 6, 7)),
                   ((2, 12, 128, 32), (2, 12, 32, 128)), ((8, 128, 384), (384, 384))]:
        a = rng.standard_normal(sa).astype(np.float32)
        b = rng.standard_normal(sb).astype(np.float32)
        ref = O.matmul(a, b)
        da, db = DeviceTensor.from_host(ctx, a), DeviceTensor.from_host(ctx, b)
        out = DeviceTensor(ctx, ref.shape, np.float32)
        N_.check(N_.lib.lonnx_matmul_f32(ctx.handle, da.ptr, N_.shape_arr(sa), len(sa), db.ptr, N_.shape_arr(sb),
                                         len(sb), out.ptr))
        ctx.sync()
        close(out.to_host(), ref)


def test_matmul_known_answer(ctx):
    """tests/Lokad.Onnx.Tensors.Tests/MathTests.cs:117-123: arange MatMul -> c[0,1,1] == 326."""
    from onnx_b200.provider import CUDAExecutionProvider as P
    a = np.arange(0, 16, dtype=np.float32).reshape(2, 2, 4)
    b = np.arange(0, 64, dtype=np.float32).reshape(2, 4, 8)
    r = P.MatMul(a, b)
    assert r.Status == "Success", r.Message
    assert r.Outputs[0][0, 1, 1] == 326.0


def test_tf32_operand_truncation(ctx):
    """The kernel uses the raw fp32 activation tile as the high part of the
    split, relying on the tensor core reading an fp32 operand as its tf32
    truncation.  Inputs whose low part is 3/4 of a tf32 ulp discriminate: a
    rounding tensor core would take hi + 1 ulp and the result would be off by
    ~1e-3 relative; truncation gives fp32 accuracy."""
    rng = np.random.default_rng(12)
    M, K, N = 512, 256, 512
    base = rng.uniform(1, 2, (M, K)).astype(np.float32)
    base = (base.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)  # tf32-exact
    A = (base * np.float32(1 + 0.75 * 2.0 ** -10)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    got = _gemm(ctx, A, np.ascontiguousarray(B.T), transB=1)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel < 2e-6, rel


@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_split_k_epilogue(ctx, epi):
    """Few output tiles (M = 256, N = 200 -> 4 tiles) with a long K take the
    split-K path: partial tiles in a workspace, summed in split order, then
    alpha, beta * bias and the activation -- against float64."""
    import math
    rng = np.random.default_rng(17 + epi)
    M, K, N = 256, 3072, 200
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    W = (rng.uniform(-1, 1, (N, K)) * 0.05).astype(np.float32)
    b = rng.uniform(-1, 1, N).astype(np.float32)
    y = 0.5 * (A.astype(np.float64) @ W.T.astype(np.float64)) + 2.0 * b
    if epi == 1:
        y = np.maximum(y, 0)
    elif epi == 2:
        y = 0.5 * y * (1 + np.vectorize(math.erf)(y / math.sqrt(2)))
    got = _gemm(ctx, A, W, b, transB=1, epi=epi, alpha=0.5, beta=2.0)
    close(got, y.astype(np.float32))


def test_gemm_96_wide_tiles_vs_fp64():
    """The 96-wide tile (accumulator warps in 32-column groups; the tile-width
    model picks it for N = 384 at small M), forced via LONNX_GEMM_BN=96 in a
    child process (the switch is read once per process), on the encoder's
    batch-32 FFN2 shape, a ragged one and a GELU epilogue, against float64;
    and bit-identical to the 128-wide tile (the width changes no element's
    summation order)."""
    import os
    import subprocess
    import sys
    code = r'''
import numpy as np, sys
sys.path.insert(0, %r)
from onnx_b200.tensor import Context, DeviceTensor
from onnx_b200 import _native as N
ctx = Context(0)
out = []
for (M, K, N_, tb, epi) in [(4096, 1536, 384, 0, 0), (700, 520, 200, 1, 0), (1000, 384, 96, 0, 2)]:
    rng = np.random.default_rng(M)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (N_, K) if tb else (K, N_)).astype(np.float32)
    b = rng.uniform(-1, 1, N_).astype(np.float32)
    ref = A.astype(np.float64) @ (B.T if tb else B).astype(np.float64) + b
    if epi == 2:
        from math import erf, sqrt
        ref = 0.5 * ref * (1 + np.vectorize(erf)(ref / sqrt(2)))
    dA, dB, db = (DeviceTensor.from_host(ctx, x) for x in (A, B, b))
    y = DeviceTensor(ctx, (M, N_), np.float32)
    N.check(N.lib.lonnx_gemm_f32(ctx.handle, dA.ptr, dB.ptr, db.ptr, y.ptr, 1, M, N_, K, 0, 0, 0, tb, 1.0, 1.0, epi))
    ctx.sync()
    got = y.to_host()
    err = np.abs(got - ref) - (1e-4 + 1e-4 * np.abs(ref))
    assert err.max() <= 0, (M, K, N_, float(err.max()))
    out.append(got)
np.save(sys.argv[1], np.concatenate([o.ravel() for o in out]))
print("ok")
''' % os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    import tempfile
    import numpy as np
    res = {}
    with tempfile.TemporaryDirectory() as d:
        for bn in ("96", "128"):
            f = os.path.join(d, bn + ".npy")
            env = dict(os.environ, LONNX_GEMM_BN=bn)
            r = subprocess.run([sys.executable, "-c", code, f], env=env, capture_output=True, text=True, timeout=300)
            assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
            res[bn] = np.load(f)
    assert np.array_equal(res["96"], res["128"])
