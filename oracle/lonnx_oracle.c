/*
 * lonnx_oracle.c -- CPU restatement of Lokad.Onnx's float32 operator kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in onnx_b200/ and the timed CPU baseline of bench.py.  Nothing in the
 * product path loads it.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference arm may call it.
 *
 * Each function restates one routine of the reference (C#, .NET 8) with the
 * same loop order and the same float32 summation order, so that it reproduces
 * the reference's results bit for bit where the reference is deterministic:
 *
 *   - separate multiply and add (compile with -ffp-contract=off): the default
 *     reference float path (HardwareConfig.UseIntrinsics=false,
 *     src/Lokad.Onnx.Base/HardwareConfig.cs:7) uses Vector<float> `c + a*b`,
 *     which .NET does not contract into an FMA;
 *   - every reduction is a sequential float32 sum in index order.
 *
 * Parity is pinned against the reference's own known answers
 * (tests/Lokad.Onnx.Tensors.Tests/MathTests.cs:82-168,
 *  tests/python/test_backend.py:379-442,792-876) and against the mnist-8
 * end-to-end classification (tests/Lokad.Onnx.Backend.Tests/GraphTests.cs:15-30);
 * see tests/test_oracle_golden.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

/* MathOps.mm_unsafe_vectorized (src/Lokad.Onnx.Tensors/MathOps.cs:380-410).
 * Reference naming: M = rows of A, N = inner dimension, K = columns of B.
 * C is zero-initialised (the reference writes into a fresh DenseTensor) and
 * accumulated row by row: C[i,:] += A[i,j] * B[j,:] for j = 0..N-1. */
ORACLE_API void oracle_mm(int M, int N, int K, const float *A, const float *B, float *C)
{
    for (int i = 0; i < M; ++i) {
        float *Cp = C + (int64_t)i * K;
        const float *Ap = A + (int64_t)i * N;
        for (int k = 0; k < K; ++k) Cp[k] = 0.0f;
        for (int j = 0; j < N; ++j) {
            const float a = Ap[j];
            const float *Bp = B + (int64_t)j * K;
            for (int k = 0; k < K; ++k) {
                float prod = a * Bp[k];
                Cp[k] = Cp[k] + prod;
            }
        }
    }
}

/* Batched form of Tensor<float>.MatMul (src/Lokad.Onnx.Tensors/TensorOps.cs:600-672):
 * one mm call per leading index with the broadcast storage offsets the caller
 * computed (stride 0 on broadcast dimensions, TensorOps.cs:621-631,648). */
ORACLE_API void oracle_mm_batched(int nbatch, const int64_t *offA, const int64_t *offB,
                                  const int64_t *offC, int M, int N, int K,
                                  const float *A, const float *B, float *C)
{
    for (int b = 0; b < nbatch; ++b)
        oracle_mm(M, N, K, A + offA[b], B + offB[b], C + offC[b]);
}

/* MathOps.Im2col (src/Lokad.Onnx.Tensors/MathOps.cs:654-709): buffer laid out
 * as [C * kY * kX, dstH * dstW], zero outside the padded input. */
static void im2col(const float *src, int srcC, int srcH, int srcW, int kY, int kX,
                   int dilY, int dilX, int strY, int strX, int padY, int padX,
                   int padH, int padW, float *buf)
{
    const int dstH = (srcH + padY + padH - (dilY * (kY - 1) + 1)) / strY + 1;
    const int dstW = (srcW + padX + padW - (dilX * (kX - 1) + 1)) / strX + 1;
    for (int c = 0; c < srcC; ++c)
        for (int ky = 0; ky < kY; ++ky)
            for (int kx = 0; kx < kX; ++kx)
                for (int dy = 0; dy < dstH; ++dy) {
                    const int sy = ky * dilY - padY + dy * strY;
                    for (int dx = 0; dx < dstW; ++dx) {
                        const int sx = kx * dilX - padX + dx * strX;
                        float v = 0.0f;
                        if (sy >= 0 && sy < srcH && sx >= 0 && sx < srcW)
                            v = src[((int64_t)c * srcH + sy) * srcW + sx];
                        *buf++ = v;
                    }
                }
}

/* MathOps.Conv2D(float*) (src/Lokad.Onnx.Tensors/MathOps.cs:791-877).
 * Per image: im2col, then per group a scalar i-k-j product
 * dst[m, p] = sum_k W[m, k] * buf[k, p] (zero-initialised, sequential in k,
 * MathOps.cs:821-846), then the bias is added in a separate pass (:862-872).
 * Argument order follows the reference call (TensorOps.cs:937):
 * padY, padX, padH, padW receive the pad info's left, top, right, bottom. */
ORACLE_API int oracle_conv2d(const float *src, int batch, int srcC, int srcH, int srcW,
                             int kY, int kX, int dilY, int dilX, int strY, int strX,
                             int padY, int padX, int padH, int padW, int group,
                             const float *weight, float *dst, int dstC, const float *bias)
{
    const int dstH = (srcH + padY + padH - (dilY * (kY - 1) + 1)) / strY + 1;
    const int dstW = (srcW + padX + padW - (dilX * (kX - 1) + 1)) / strX + 1;
    const int M = dstC / group;
    const int64_t N = (int64_t)dstH * dstW;
    const int64_t K = (int64_t)srcC * kY * kX / group;
    float *buf = (float *)malloc(sizeof(float) * (size_t)srcC * kY * kX * N);
    if (!buf) return -1;
    for (int b = 0; b < batch; ++b) {
        im2col(src, srcC, srcH, srcW, kY, kX, dilY, dilX, strY, strX, padY, padX, padH, padW, buf);
        for (int g = 0; g < group; ++g) {
            const float *Wg = weight + (int64_t)M * K * g;
            const float *Bg = buf + N * K * g;
            float *Cg = dst + (int64_t)M * N * g;
            for (int i = 0; i < M; ++i) {
                float *Cp = Cg + i * N;
                const float *Ap = Wg + i * K;
                for (int64_t j = 0; j < N; ++j) Cp[j] = 0.0f;
                for (int64_t k = 0; k < K; ++k) {
                    const float a = Ap[k];
                    const float *Bp = Bg + k * N;
                    for (int64_t j = 0; j < N; ++j) {
                        float prod = a * Bp[j];
                        Cp[j] = Cp[j] + prod;
                    }
                }
            }
        }
        if (bias) {
            for (int i = 0; i < dstC; ++i) {
                float *pd = dst + (int64_t)i * N;
                for (int64_t j = 0; j < N; ++j) pd[j] = pd[j] + bias[i];
            }
        }
        src += (int64_t)srcC * srcH * srcW;
        dst += (int64_t)dstC * dstH * dstW;
    }
    free(buf);
    return 0;
}

/* Tensor<float>.MaxPool2D window loop (src/Lokad.Onnx.Tensors/TensorOps.cs:1025-1099):
 * window clipped to the input, max starting from -inf, early exit from the
 * row loop while the max is still -inf; dilation is not applied to the window. */
ORACLE_API void oracle_maxpool2d(const float *x, int N, int C, int H, int W, int kH, int kW,
                                 int sH, int sW, int padTop, int padLeft, int outH, int outW,
                                 float *y)
{
    for (int n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c) {
            const float *xp = x + ((int64_t)n * C + c) * H * W;
            float *yp = y + ((int64_t)n * C + c) * outH * outW;
            for (int yr = 0; yr < outH; ++yr) {
                const int rc = yr * sH - padTop;
                const int rmin = rc > 0 ? rc : 0;
                const int rmax = (kH + rc) < H ? (kH + rc) : H;
                for (int yc = 0; yc < outW; ++yc) {
                    const int cc = yc * sW - padLeft;
                    const int cmin = cc > 0 ? cc : 0;
                    const int cmax = (kW + cc) < W ? (kW + cc) : W;
                    float m = -INFINITY;
                    for (int r = rmin; r < rmax; ++r) {
                        for (int q = cmin; q < cmax; ++q) {
                            const float v = xp[(int64_t)r * W + q];
                            if (v > m) m = v;
                        }
                        if (m == -INFINITY) break;
                    }
                    yp[(int64_t)yr * outW + yc] = m;
                }
            }
        }
}

/* Reductions over the innermost `r` elements of each of `outer` rows, the
 * layout the reference reaches after moving the reduced axes innermost
 * (ArrayUtilities.GetAxesPermutationForReduction, ArrayUtilities.cs:357-373).
 *   op 0: ReduceSum  (TensorOps.cs:1610-1657) sequential float sum from 0.0f
 *   op 1: ReduceMax  (TensorOps.cs:1789-1839) running max that starts at 0.0f
 *         (reference defect: all-negative rows give 0)
 *   op 2: ReduceMean (TensorOps.cs:1735-1760) ReduceSum, then divide by (float)r */
ORACLE_API void oracle_reduce_inner(int op, const float *x, int64_t outer, int64_t r, float *y)
{
    for (int64_t i = 0; i < outer; ++i) {
        const float *p = x + i * r;
        float acc = 0.0f;
        if (op == 1) {
            for (int64_t j = 0; j < r; ++j)
                if (p[j] > acc) acc = p[j];
        } else {
            for (int64_t j = 0; j < r; ++j) acc = acc + p[j];
            if (op == 2) acc = acc / (float)r;
        }
        y[i] = acc;
    }
}

/* Tensor<float>.Softmax (src/Lokad.Onnx.Tensors/TensorOps.cs:1312-1330) over the
 * middle axis of an [outer, len, inner] view: ReduceMax (starting at 0.0f),
 * Subtract, Exp, ReduceSum (sequential), Divide -- each step rounded to float. */
ORACLE_API void oracle_softmax(const float *x, int64_t outer, int64_t len, int64_t inner, float *y)
{
    for (int64_t o = 0; o < outer; ++o)
        for (int64_t in = 0; in < inner; ++in) {
            const float *xp = x + o * len * inner + in;
            float *yp = y + o * len * inner + in;
            float m = 0.0f;
            for (int64_t j = 0; j < len; ++j)
                if (xp[j * inner] > m) m = xp[j * inner];
            float s = 0.0f;
            for (int64_t j = 0; j < len; ++j) {
                float d = xp[j * inner] - m;
                float e = expf(d);
                yp[j * inner] = e;
                s = s + e;
            }
            for (int64_t j = 0; j < len; ++j) yp[j * inner] = yp[j * inner] / s;
        }
}

/* MathOps.Erf(float) (src/Lokad.Onnx.Tensors/MathOps.cs:989-1010):
 * Abramowitz & Stegun formula 7.1.26 evaluated in float with expf. */
static float as_erf(float x)
{
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f;
    const float a4 = -1.453152027f, a5 = 1.061405429f, p = 0.3275911f;
    const int sign = x < 0 ? -1 : 1;
    x = fabsf(x);
    const float t = 1.0f / (1.0f + p * x);
    const float poly = ((((a5 * t + a4) * t) + a3) * t + a2) * t + a1;
    const float y = 1.0f - poly * t * expf(-x * x);
    return (float)sign * y;
}

/* Element-wise unary ops:
 *   0 Relu  (TensorOps.cs:1252: l > 0 ? l : 0)
 *   1 Sqrt  (TensorOps.cs:315, Vector.SquareRoot -> IEEE sqrt)
 *   2 Erf   (TensorOps.cs:1353 -> MathOps.Erf)
 *   3 Exp   (MathF.Exp, used inside Softmax) */
ORACLE_API void oracle_unary(int op, const float *x, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        switch (op) {
        case 0: y[i] = v > 0.0f ? v : 0.0f; break;
        case 1: y[i] = sqrtf(v); break;
        case 2: y[i] = as_erf(v); break;
        default: y[i] = expf(v); break;
        }
    }
}

/* Element-wise binary ops on operands the caller already broadcast to the
 * output shape (the reference densifies broadcasts before the math,
 * CPUExecutionProvider.cs:97-102):
 *   0 Add, 1 Sub, 2 Mul, 3 Div (TensorOps.cs:243-291), 4 Pow (MathF.Pow, :303) */
ORACLE_API void oracle_binary(int op, const float *a, const float *b, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) {
        const float l = a[i], r = b[i];
        switch (op) {
        case 0: y[i] = l + r; break;
        case 1: y[i] = l - r; break;
        case 2: y[i] = l * r; break;
        case 3: y[i] = l / r; break;
        default: y[i] = powf(l, r); break;
        }
    }
}
