"""lonnx_gemm_f32_noalloc: the GEMM for callers that cannot allocate device
memory (a callback or plugin running inside a runtime that owns the device's
memory pool, or code without a lonnx_ctx).  Its weight split lives in a fixed
device array inside the library instead of allocated scratch.  It must give
the same results as lonnx_gemm_f32 (within the parity tolerance) on two calls
in a row -- the second call reuses the array the first one left behind --
and refuse weights larger than the array.

This file sorts last so that a run stopping at the first failure has already
run every other test."""
import numpy as np
import pytest

from conftest import close

pytestmark = pytest.mark.gpu


def _run(ctx, fn_name, A, B, bias, transB, epi, batch=1, sA=0, sB=0, sC=0, M=None, Nn=None, K=None):
    """One call of `fn_name`; A, B are flat or 2-D host arrays, the output
    holds batch * M * Nn floats (sC apart)."""
    from onnx_b200 import _native as N
    from onnx_b200.tensor import DeviceTensor
    if M is None:
        M, K = A.shape
        Nn = B.shape[0] if transB else B.shape[1]
    dA, dB, db = (DeviceTensor.from_host(ctx, x) for x in (A, B, bias))
    out = DeviceTensor(ctx, (max(batch, 1) * M * Nn,), np.float32)
    first = ctx.handle if fn_name == "lonnx_gemm_f32" else ctx.stream
    N.check(getattr(N.lib, fn_name)(first, dA.ptr, dB.ptr, db.ptr, out.ptr, batch, M, Nn, K, sA, sB, sC, transB,
                                    1.0, 1.0, epi))
    if fn_name != "lonnx_gemm_f32":
        N.check(N.lib.lonnx_gemm_f32_noalloc_status(ctx.stream))  # no pipeline wait expired
    ctx.sync()
    return out.to_host()


@pytest.mark.parametrize("M,K,N,transB,epi", [(4096, 384, 1536, 1, 0), (2048, 1536, 384, 0, 2), (100, 36, 70, 0, 0)])
def test_noalloc_matches_allocating_gemm_twice(ctx, M, K, N, transB, epi):
    rng = np.random.default_rng(M + K + N)
    for call in range(2):  # two calls in a row: the shared array keeps the previous call's contents
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        B = rng.uniform(-1, 1, (N, K) if transB else (K, N)).astype(np.float32)
        bias = rng.uniform(-1, 1, N).astype(np.float32)
        ref = _run(ctx, "lonnx_gemm_f32", A, B, bias, transB, epi)
        got = _run(ctx, "lonnx_gemm_f32_noalloc", A, B, bias, transB, epi)
        close(got, ref)


@pytest.mark.parametrize("shared", [False, True])
def test_noalloc_batched_matches_allocating_gemm(ctx, shared):
    """batch = 3 on the tensor-core path.  With a weight per batch
    (strideB != 0) every batch re-splits its weight into the same array,
    which is correct only because the split waits in stream order for the
    previous batch's GEMM; with a shared weight (strideB = 0) and strideA
    != M*K, the batches do not fold into one tall GEMM and reuse one split."""
    M, K, Nn, batch = 512, 384, 384, 3
    rng = np.random.default_rng(17 + shared)
    sA = M * K + 64  # padded: never folds
    A = rng.uniform(-1, 1, batch * sA).astype(np.float32)
    sB = 0 if shared else K * Nn
    B = rng.uniform(-1, 1, max(sB * batch, K * Nn)).astype(np.float32)
    bias = rng.uniform(-1, 1, Nn).astype(np.float32)
    for call in range(2):
        kw = dict(batch=batch, sA=sA, sB=sB, sC=M * Nn, M=M, Nn=Nn, K=K)
        ref = _run(ctx, "lonnx_gemm_f32", A, B, bias, 0, 0, **kw)
        got = _run(ctx, "lonnx_gemm_f32_noalloc", A, B, bias, 0, 0, **kw)
        close(got, ref)
        A = A[::-1].copy()


def test_noalloc_large_weight_on_ffma_path(ctx):
    """The size limit binds only the tensor-core path: a GEMM whose K is not
    a multiple of 4 (so TMA cannot address it) with a weight larger than the
    array runs on the FFMA kernel, which needs no scratch, and matches
    lonnx_gemm_f32."""
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (4, 2047)).astype(np.float32)
    B = rng.uniform(-1, 1, (2047, 4096)).astype(np.float32)
    bias = rng.uniform(-1, 1, 4096).astype(np.float32)
    ref = _run(ctx, "lonnx_gemm_f32", A, B, bias, 0, 0)
    got = _run(ctx, "lonnx_gemm_f32_noalloc", A, B, bias, 0, 0)
    close(got, ref)


def test_noalloc_rejects_oversized_weight(ctx):
    from onnx_b200 import _native as N
    rc = N.lib.lonnx_gemm_f32_noalloc(ctx.stream, 16, 16, None, 16, 1, 8, 4096, 2048, 0, 0, 0, 1, 1.0, 1.0, 0)
    assert rc == -1
    assert "exceeds the fixed scratch" in N.lib.lonnx_last_error().decode()
