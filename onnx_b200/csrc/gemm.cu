// GEMM / MatMul entry points, the fp32 FFMA fallback GEMM, direct
// convolution for small problems, and the GEMM dispatcher.
//
// Dispatch: a contraction with enough work and 16-byte aligned rows runs on
// the tcgen05 3xTF32 kernel (gemm_tc.cu); everything else runs on an fp32
// SIMT kernel whose per-output summation order (sequential over k, separate
// multiply and add) is exactly the reference's mm_unsafe_vectorized order
// (src/Lokad.Onnx.Tensors/MathOps.cs:380-410) -- bit-identical results on the
// small shapes where launch latency, not the tensor pipe, is the bound.
#include <vector>
#include <cstdio>

#include "lonnx_internal.cuh"

namespace {

constexpr int SB_M = 64, SB_N = 64, SB_K = 16;

// C[b] = alpha * A[b] . op(B[b]) (+ beta*bias) (+ residual) -> epilogue
template <bool TB>
__global__ void __launch_bounds__(256)
k_gemm_simt(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
            const float *__restrict__ res, float *__restrict__ C, int M, int N, int K, int64_t sA,
            int64_t sB, int64_t sC, float alpha, float beta, int epi) {
    __shared__ float As[SB_K][SB_M + 4];
    __shared__ float Bs[SB_K][SB_N + 4];
    const int b = blockIdx.z;
    A += b * sA;
    B += b * sB;
    C += b * sC;
    if (res) res += b * sC;
    const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += SB_K) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int e = threadIdx.x + 256 * t;  // 0..1023
            {
                const int kk = e & 15, mm = e >> 4;
                const int gm = m0 + mm, gk = k0 + kk;
                As[kk][mm] = (gm < M && gk < K) ? A[(int64_t)gm * K + gk] : 0.0f;
            }
            {
                int kk, nn;
                if (TB) { kk = e & 15; nn = e >> 4; } else { nn = e & 63; kk = e >> 6; }
                const int gn = n0 + nn, gk = k0 + kk;
                float v = 0.0f;
                if (gn < N && gk < K) v = TB ? B[(int64_t)gn * K + gk] : B[(int64_t)gk * N + gn];
                Bs[kk][nn] = v;
            }
        }
        __syncthreads();
        const int kmax = min(SB_K, K - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            float a[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], bv[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx + 16 * j;
            if (gn >= N) continue;
            float v = acc[i][j];
            if (alpha != 1.0f) v = __fmul_rn(v, alpha);
            if (bias) v = __fadd_rn(v, beta == 1.0f ? bias[gn] : __fmul_rn(beta, bias[gn]));
            if (res) v = __fadd_rn(v, res[(int64_t)gm * N + gn]);
            if (epi == LONNX_EPI_RELU) v = v > 0.0f ? v : 0.0f;
            else if (epi == LONNX_EPI_GELU_ERF) v = lonnx_gelu_chain(v);
            C[(int64_t)gm * N + gn] = v;
        }
    }
}

// Tiny outputs (e.g. the mnist-8 classifier, 1 x 256 . 256 x 10): one thread
// per output element, sequential over k with a separate multiply and add --
// the same order as k_gemm_simt, without its tile loop and block barriers,
// which make a one-block launch latency-bound.
template <bool TB>
__global__ void k_gemm_rowdot(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
                              const float *__restrict__ res, float *__restrict__ C, int M, int N, int K, int64_t sA,
                              int64_t sB, int64_t sC, int batch, float alpha, float beta, int epi) {
    const int64_t total = (int64_t)batch * M * N;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int n = (int)(t % N);
        const int m = (int)((t / N) % M);
        const int b = (int)(t / ((int64_t)N * M));
        const float *a = A + b * sA + (int64_t)m * K;
        const float *bb = B + b * sB;
        float acc = 0.0f;
#pragma unroll 8
        for (int k = 0; k < K; ++k) {
            const float bv = TB ? __ldg(bb + (int64_t)n * K + k) : __ldg(bb + (int64_t)k * N + n);
            acc = __fadd_rn(acc, __fmul_rn(__ldg(a + k), bv));
        }
        float v = acc;
        if (alpha != 1.0f) v = __fmul_rn(v, alpha);
        if (bias) v = __fadd_rn(v, beta == 1.0f ? bias[n] : __fmul_rn(beta, bias[n]));
        if (res) v = __fadd_rn(v, res[b * sC + (int64_t)m * N + n]);
        if (epi == LONNX_EPI_RELU) v = v > 0.0f ? v : 0.0f;
        else if (epi == LONNX_EPI_GELU_ERF) v = lonnx_gelu_chain(v);
        C[b * sC + (int64_t)m * N + n] = v;
    }
}

// The same sums for one small product (batch 1, A and B fit in 48 KB of
// shared memory): one block stages A [M, K] and B with coalesced loads, then
// each thread sums its output in the same order from shared memory.  The
// per-thread version waits on global loads inside its sequential sum.
template <bool TB>
__global__ void __launch_bounds__(256) k_gemm_rowdot_smem(const float *__restrict__ A, const float *__restrict__ B,
                                                          const float *__restrict__ bias, const float *__restrict__ res,
                                                          float *__restrict__ C, int M, int N, int K, float alpha,
                                                          float beta, int epi) {
    extern __shared__ float sh[];
    float *as = sh, *bs = sh + (int64_t)M * K;
    const int na = M * K, nb = K * N;
    for (int i = threadIdx.x; i < na; i += blockDim.x) as[i] = __ldg(A + i);
    for (int i = threadIdx.x; i < nb; i += blockDim.x) bs[i] = __ldg(B + i);
    __syncthreads();
    for (int t = threadIdx.x; t < M * N; t += blockDim.x) {
        const int m = t / N, n = t - m * N;
        const float *a = as + m * K;
        float acc = 0.0f;
#pragma unroll 8
        for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(a[k], TB ? bs[n * K + k] : bs[k * N + n]));
        float v = acc;
        if (alpha != 1.0f) v = __fmul_rn(v, alpha);
        if (bias) v = __fadd_rn(v, beta == 1.0f ? bias[n] : __fmul_rn(beta, bias[n]));
        if (res) v = __fadd_rn(v, res[t]);
        if (epi == LONNX_EPI_RELU) v = v > 0.0f ? v : 0.0f;
        else if (epi == LONNX_EPI_GELU_ERF) v = lonnx_gelu_chain(v);
        C[t] = v;
    }
}

// Direct NCHW convolution, one thread per output element, summing over
// (c, ky, kx) in the im2col row order of MathOps.Conv2D with a separate
// multiply and add (MathOps.cs:821-846), then the bias pass (:862-872) and
// an optional ReLU.  Padded taps are skipped (they add an exact zero).
__global__ void k_conv2d_direct(const float *__restrict__ x, const float *__restrict__ w,
                                const float *__restrict__ bias, float *__restrict__ y, int N, int C,
                                int H, int W, int M, int kh, int kw, int sh, int sw, int pt, int pl,
                                int dh, int dw, int group, int Ho, int Wo, int relu) {
    const int64_t total = (int64_t)N * M * Ho * Wo;
    const int cg = C / group, mg = M / group;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += stride) {
        const int ox = (int)(t % Wo);
        const int oy = (int)((t / Wo) % Ho);
        const int m = (int)((t / ((int64_t)Wo * Ho)) % M);
        const int n = (int)(t / ((int64_t)Wo * Ho * M));
        const int g = m / mg;
        const float *wp = w + (int64_t)m * cg * kh * kw;
        float acc = 0.0f;
        for (int c = 0; c < cg; ++c) {
            const float *xp = x + ((int64_t)n * C + g * cg + c) * H * W;
            for (int ky = 0; ky < kh; ++ky) {
                const int iy = oy * sh - pt + ky * dh;
                for (int kx = 0; kx < kw; ++kx) {
                    const int ix = ox * sw - pl + kx * dw;
                    if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
                    acc = __fadd_rn(acc, __fmul_rn(wp[(c * kh + ky) * kw + kx], xp[(int64_t)iy * W + ix]));
                }
            }
        }
        if (bias) acc = __fadd_rn(acc, bias[m]);
        if (relu) acc = acc > 0.0f ? acc : 0.0f;
        y[t] = acc;
    }
}

// weight [M, K] -> hi, lo [M, ldk] (tf32 split, zero padded)
__global__ void k_split_pad_rows(const float *__restrict__ w, float *__restrict__ hi, float *__restrict__ lo, int M,
                                 int K, int ldk) {
    const int64_t total = (int64_t)M * ldk;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += stride) {
        const int k = (int)(t % ldk);
        const int64_t m = t / ldk;
        const float v = k < K ? w[m * K + k] : 0.0f;
        const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
        hi[t] = h;
        lo[t] = __fsub_rn(v, h);
    }
}

// tap-major split: column tap * C + c of the output takes w[m][c * taps + tap]
__global__ void k_split_rows_tapmajor(const float *__restrict__ w, float *__restrict__ hi, float *__restrict__ lo,
                                      int M, int C, int taps) {
    const int64_t K = (int64_t)C * taps, total = (int64_t)M * K;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t m = t / K;
        const int k = (int)(t - m * K), tap = k / C, c = k - tap * C;
        const float v = w[m * K + (int64_t)c * taps + tap];
        const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
        hi[t] = h;
        lo[t] = __fsub_rn(v, h);
    }
}

// y = y + r (then ReLU): a Conv -> Add [-> Relu] chain off the tensor cores
__global__ void k_add_relu(float *__restrict__ y, const float *__restrict__ r, int64_t n, int relu) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += stride) {
        float v = __fadd_rn(y[t], r[t]);
        if (relu) v = v > 0.0f ? v : 0.0f;
        y[t] = v;
    }
}

inline int grid_for(lonnx_ctx *ctx, int64_t work, int threads = 256) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

inline bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

namespace lonnx {

int transpose_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, const int64_t *shape, int rank,
                     const int64_t *perm, void *y);

int gemm_simt(lonnx_ctx *ctx, const float *A, const float *B, const float *bias, float *C,
              int batch, int M, int N, int K, int64_t sA, int64_t sB, int64_t sC, int transB,
              float alpha, float beta, int epi, const float *residual) {
    if (batch == 1 && (int64_t)M * N <= 256 && ((int64_t)M * K + (int64_t)K * N) * 4 <= 48 * 1024) {
        const size_t smem = ((size_t)M * K + (size_t)K * N) * 4;
        if (transB)
            k_gemm_rowdot_smem<true><<<1, 256, smem, ctx->stream>>>(A, B, bias, residual, C, M, N, K, alpha, beta, epi);
        else
            k_gemm_rowdot_smem<false><<<1, 256, smem, ctx->stream>>>(A, B, bias, residual, C, M, N, K, alpha, beta, epi);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if ((int64_t)batch * M * N <= 16384) {
        const int64_t total = (int64_t)batch * M * N;
        const int blocks = (int)((total + 127) / 128);
        if (transB)
            k_gemm_rowdot<true><<<blocks, 128, 0, ctx->stream>>>(A, B, bias, residual, C, M, N, K, sA, sB, sC, batch,
                                                                 alpha, beta, epi);
        else
            k_gemm_rowdot<false><<<blocks, 128, 0, ctx->stream>>>(A, B, bias, residual, C, M, N, K, sA, sB, sC, batch,
                                                                  alpha, beta, epi);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    dim3 grid((N + SB_N - 1) / SB_N, (M + SB_M - 1) / SB_M, batch);
    if (grid.z > 65535) return set_error(LONNX_E_UNSUPPORTED, "gemm: batch %d too large", batch);
    if (transB)
        k_gemm_simt<true><<<grid, 256, 0, ctx->stream>>>(A, B, bias, residual, C, M, N, K, sA, sB, sC, alpha, beta, epi);
    else
        k_gemm_simt<false><<<grid, 256, 0, ctx->stream>>>(A, B, bias, residual, C, M, N, K, sA, sB, sC, alpha, beta, epi);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

// Minimum work (multiply-adds) before the tensor-core path pays off.
int64_t gemm_tc_min_work() {
    static int64_t v = [] {
        const char *e = getenv("LONNX_TC_MIN_WORK");
        return e ? atoll(e) : (int64_t)1 << 21;
    }();
    return v;
}

int gemm_dispatch(lonnx_ctx *ctx, const float *A, const float *B, const float *bias, float *C,
                  int batch, int M, int N, int K, int64_t sA, int64_t sB, int64_t sC, int transB,
                  float alpha, float beta, int epi, const float *residual, bool split_k) {
    if (M == 0 || N == 0 || batch == 0) return LONNX_OK;
    if (K == 0) {
        // empty contraction: C = beta*bias (+ epilogue); the SIMT kernel handles it
        return gemm_simt(ctx, A, B, bias, C, batch, M, N, K, sA, sB, sC, transB, alpha, beta, epi, residual);
    }
    // a shared weight with a dense batch of A folds into one tall GEMM
    if (batch > 1 && sB == 0 && sA == (int64_t)M * K && sC == (int64_t)M * N && (int64_t)batch * M < (1ll << 31)) {
        M *= batch;
        batch = 1;
    }
    const bool big = (int64_t)M * N * K >= gemm_tc_min_work();
    const bool aligned = (K % 4 == 0) && al16(A) && al16(B) && (sA % 4 == 0) && (sB % 4 == 0) &&
                         (transB || N % 4 == 0);
    static const bool tc_off = getenv("LONNX_DISABLE_TC") != nullptr;
    if (big && aligned && !residual && !tc_off) {
        // tensor-core operands: B[b] split into K-major tf32 high/low parts in scratch
        const int nb = sB == 0 ? 1 : batch;
        void *tmp = nullptr;
        int rc = ctx_scratch(ctx, (size_t)nb * 2 * K * N * sizeof(float), &tmp);
        if (rc) return rc;
        float *hi = (float *)tmp, *lo = hi + (size_t)nb * K * N;
        for (int b = 0; b < nb; ++b) {
            rc = split_tf32_nk(ctx, B + b * sB, hi + (int64_t)b * K * N, lo + (int64_t)b * K * N, K, N, transB);
            if (rc) return rc;
        }
        const int64_t sW = sB == 0 ? 0 : (int64_t)K * N;
        for (int b = 0; b < batch; ++b) {
            rc = gemm_tc(ctx, A + b * sA, hi + b * sW, lo + b * sW, bias, C + b * sC, M, N, K, K, K, N, alpha, beta,
                         epi, true, split_k && batch == 1);
            if (rc == LONNX_E_UNSUPPORTED && b == 0) break;  // fall through to SIMT
            if (rc) return rc;
            if (b == batch - 1) return LONNX_OK;
        }
    }
    return gemm_simt(ctx, A, B, bias, C, batch, M, N, K, sA, sB, sC, transB, alpha, beta, epi, residual);
}

}  // namespace lonnx

using namespace lonnx;

extern "C" {

LONNX_API int lonnx_gemm_f32(lonnx_ctx *ctx, const float *A, const float *B, const float *bias,
                             float *C, int batch, int M, int N, int K, int64_t strideA,
                             int64_t strideB, int64_t strideC, int transB, float alpha, float beta,
                             int epilogue) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!A || !B || !C || batch < 0 || M < 0 || N < 0 || K < 0 || epilogue < 0 || epilogue > 2)
        return set_error(LONNX_E_BADARG, "gemm: bad arguments");
    // the single-op entry point may split K when the output has few tiles
    return gemm_dispatch(ctx, A, B, bias, C, batch, M, N, K, strideA, strideB, strideC, transB, alpha,
                         beta, epilogue, nullptr, true);
}

LONNX_API int lonnx_matmul_f32(lonnx_ctx *ctx, const float *a, const int64_t *as, int ar,
                               const float *b, const int64_t *bs, int br, float *y) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!a || !b || !y || ar < 1 || br < 1 || ar > 8 || br > 8)
        return set_error(LONNX_E_BADARG, "The rank of each tensor in matrix multiplication must be greater than 1.");
    if (ar == 1 && br == 1) {
        if (as[0] != bs[0]) return set_error(LONNX_E_SHAPE, "MatMul: inner dimensions differ");
        return gemm_dispatch(ctx, a, b, nullptr, y, 1, 1, 1, (int)as[0], 0, 0, 0, 0, 1.0f, 0.0f, 0, nullptr);
    }
    if (ar < 2 || br < 2)
        return set_error(LONNX_E_UNSUPPORTED, "MatMul of a rank-1 and a rank>=2 tensor");
    const int64_t m = as[ar - 2], k = as[ar - 1], k2 = bs[br - 2], n = bs[br - 1];
    if (k != k2)
        return set_error(LONNX_E_SHAPE, "The number of columns in the first matrix (%lld) is not equal to the number of rows in the second matrix (%lld).",
                         (long long)k, (long long)k2);
    int64_t lead[8];
    int lr = 0;
    rc = lonnx_broadcast_shape(as, ar - 2, bs, br - 2, lead, &lr);
    if (rc) return set_error(LONNX_E_SHAPE, "The tensor shapes are not compatible for broadcasting.");
    int64_t nb = 1;
    for (int i = 0; i < lr; ++i) nb *= lead[i];
    if (nb == 0 || m == 0 || n == 0) return LONNX_OK;
    // per-dimension batch strides (0 where broadcast)
    int64_t sa[8], sb[8];
    {
        int64_t s1 = m * k, s2 = k * n;
        for (int d = lr - 1; d >= 0; --d) {
            const int ia = d - (lr - (ar - 2)), ib = d - (lr - (br - 2));
            const int64_t da = ia >= 0 ? as[ia] : 1, db = ib >= 0 ? bs[ib] : 1;
            sa[d] = (da == 1) ? 0 : s1;
            sb[d] = (db == 1) ? 0 : s2;
            s1 *= da;
            s2 *= db;
        }
    }
    // uniform strides over the flattened batch? (dense or fully broadcast operand)
    auto uniform = [&](const int64_t *s, int64_t unit) {
        bool all0 = true, dense = true;
        int64_t expect = unit;
        for (int d = lr - 1; d >= 0; --d) {
            all0 &= s[d] == 0;
            dense &= (s[d] == expect) || lead[d] == 1;
            expect *= lead[d];
        }
        return all0 ? 0 : (dense ? 1 : -1);
    };
    const int ua = uniform(sa, m * k), ub = uniform(sb, k * n);
    if (ua >= 0 && ub >= 0)
        return gemm_dispatch(ctx, a, b, nullptr, y, (int)nb, (int)m, (int)n, (int)k, ua ? m * k : 0,
                             ub ? k * n : 0, m * n, 0, 1.0f, 0.0f, 0, nullptr);
    // mixed broadcasting: one launch per batch index
    for (int64_t i = 0; i < nb; ++i) {
        int64_t rem = i, oa = 0, ob = 0;
        for (int d = lr - 1; d >= 0; --d) {
            const int64_t c = rem % lead[d];
            rem /= lead[d];
            oa += c * sa[d];
            ob += c * sb[d];
        }
        rc = gemm_dispatch(ctx, a + oa, b + ob, nullptr, y + i * m * n, 1, (int)m, (int)n, (int)k, 0, 0, 0, 0,
                           1.0f, 0.0f, 0, nullptr);
        if (rc) return rc;
    }
    return LONNX_OK;
}

LONNX_API int lonnx_conv2d_f32(lonnx_ctx *ctx, const float *x, const float *w, const float *bias,
                               float *y, int N, int C, int H, int W, int M, int kh, int kw, int sh,
                               int sw, int pt, int pl, int pb, int pr, int dh, int dw, int group,
                               int relu) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    return lonnx::conv2d(ctx, x, w, nullptr, nullptr, bias, nullptr, y, N, C, H, W, M, kh, kw, sh, sw, pt, pl, pb, pr,
                         dh, dw, group, relu);
}

}  // extern "C"

namespace lonnx {

int split_pad_rows(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int M, int K, int ldk) {
    k_split_pad_rows<<<grid_for(ctx, (int64_t)M * ldk), 256, 0, ctx->stream>>>(w, hi, lo, M, K, ldk);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

int split_rows_tapmajor(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int M, int C, int taps) {
    k_split_rows_tapmajor<<<grid_for(ctx, (int64_t)M * C * taps), 256, 0, ctx->stream>>>(w, hi, lo, M, C, taps);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

bool conv_nhwc_ok(int C, int kh, int kw, bool x_nhwc) {
    static const bool off = getenv("LONNX_CONV_NCHW_GATHER") != nullptr;
    return !off && C % 32 == 0 && (kh * kw > 1 || x_nhwc) && kh * kw <= 63;
}

// LONNX_CONV_TRACE=1: one stderr line per conv with its layouts and path
static bool conv_trace() {
    static const bool on = getenv("LONNX_CONV_TRACE") && getenv("LONNX_CONV_TRACE")[0] == '1';
    return on;
}

// [N, C, H, W] <-> [N, H, W, C] copy of a float tensor into scratch
static int relayout(lonnx_ctx *ctx, const float *x, int N, int C, int H, int W, bool to_nhwc, void **out) {
    int rc = ctx_alloc(ctx, (size_t)N * C * H * W * 4, out);
    if (rc) return rc;
    const int64_t nchw[4] = {N, C, H, W}, nhwc[4] = {N, H, W, C};
    const int64_t to[4] = {0, 2, 3, 1}, back[4] = {0, 3, 1, 2};
    rc = transpose_launch(ctx, x, 4, to_nhwc ? nchw : nhwc, 4, to_nhwc ? to : back, *out);
    if (rc) {
        ctx_free(ctx, *out);
        *out = nullptr;
    }
    return rc;
}

int conv2d(lonnx_ctx *ctx, const float *x, const float *w, const float *whi, const float *wlo, const float *bias,
           const float *res, float *y, int N, int C, int H, int W, int M, int kh, int kw, int sh, int sw, int pt,
           int pl, int pb, int pr, int dh, int dw, int group, int relu, int w_tapmajor, int x_nhwc, int res_nhwc,
           int *out_nhwc) {
    const bool want_out = out_nhwc && *out_nhwc;
    if (out_nhwc) *out_nhwc = 0;
    if (!x || !w || !y || N < 0 || C <= 0 || M <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
        dh <= 0 || dw <= 0 || group <= 0 || C % group || M % group)
        return set_error(LONNX_E_BADARG, "conv2d: bad arguments");
    const int Ho = (H + pt + pb - (dh * (kh - 1) + 1)) / sh + 1;
    const int Wo = (W + pl + pr - (dw * (kw - 1) + 1)) / sw + 1;
    if (Ho <= 0 || Wo <= 0) return set_error(LONNX_E_SHAPE, "conv2d: empty output");
    const int64_t total = (int64_t)N * M * Ho * Wo;
    if (total == 0) return LONNX_OK;
    const int K = C * kh * kw;
    const int64_t P = (int64_t)N * Ho * Wo;
    static const bool tc_off = getenv("LONNX_DISABLE_TC") != nullptr;
    if (!tc_off && group == 1 && total * K >= gemm_tc_min_work() && P < (1ll << 31) &&
        (int64_t)N * C * H * W < (1ll << 40)) {
        // implicit GEMM on the tensor cores: rows = output pixels (N*Ho*Wo),
        // columns = output channels, contraction over (c, ky, kx) in the
        // reference's im2col order; input gathered inside the kernel, bias,
        // residual and ReLU in the epilogue, NCHW (or NHWC) written directly.
        // NHWC gather: from the NHWC input as given, or from a transposed
        // copy in scratch, with the weights in tap-major column order
        // (prepared that way, or split so here)
        const bool nhwc = conv_nhwc_ok(C, kh, kw, x_nhwc) && (int64_t)C * H * W < (1ll << 31);
        const int ldk = (K + 3) & ~3;
        // an NHWC output of a residual conv reads its input NHWC (no tap
        // table); a tile shape that refuses the NHWC output runs once more
        // with an NCHW output rather than on the direct kernel
        const bool onhwc_first = want_out && (!res || nhwc);
        for (int attempt = 0; attempt < (onhwc_first ? 2 : 1); ++attempt) {
            const bool onhwc = onhwc_first && attempt == 0;
            const float *wh = whi, *wl = wlo;
            void *wt = nullptr, *xt = nullptr, *rt = nullptr;
            auto release = [&]() {
                if (wt) ctx_free(ctx, wt);
                if (xt) ctx_free(ctx, xt);
                if (rt) ctx_free(ctx, rt);
                wt = xt = rt = nullptr;
            };
            // one tap: tap-major and channel-major columns are the same order
            if (!wh || !wl || ((bool)w_tapmajor != nhwc && kh * kw > 1)) {
                int rc = ctx_alloc(ctx, (size_t)2 * M * ldk * 4, &wt);
                if (rc) return rc;
                wh = (const float *)wt;
                wl = wh + (size_t)M * ldk;
                rc = nhwc ? split_rows_tapmajor(ctx, w, (float *)wh, (float *)wl, M, C, kh * kw)
                          : split_pad_rows(ctx, w, (float *)wh, (float *)wl, M, K, ldk);
                if (rc) { release(); return rc; }
            }
            if (nhwc != (bool)x_nhwc) {
                const int rc = relayout(ctx, x, N, C, H, W, nhwc, &xt);
                if (rc) { release(); return rc; }
            }
            if (res && onhwc != (bool)res_nhwc) {
                const int rc = relayout(ctx, res, N, M, Ho, Wo, onhwc, &rt);
                if (rc) { release(); return rc; }
            }
            ConvArgs cv;
            cv.x = xt ? (const float *)xt : x;
            cv.nhwc = nhwc ? 1 : 0;
            cv.out_nhwc = onhwc ? 1 : 0;
            cv.C = C; cv.H = H; cv.W = W; cv.kh = kh; cv.kw = kw; cv.sh = sh; cv.sw = sw;
            cv.pt = pt; cv.pl = pl; cv.dh = dh; cv.dw = dw; cv.Ho = Ho; cv.Wo = Wo;
            cv.img_rows = Ho * Wo;
            cv.res = rt ? (const float *)rt : res;
            int rc = conv_tc(ctx, cv, wh, wl, ldk, bias, y, (int)P, M, K, relu ? LONNX_EPI_RELU : LONNX_EPI_NONE);
            release();
            if (conv_trace())
                fprintf(stderr,
                        "[lonnx conv] N%d C%d %dx%d M%d k%dx%d s%d x_nhwc %d gather %s out_nhwc %d res %d/%d: %s\n", N,
                        C, H, W, M, kh, kw, sh, x_nhwc, nhwc ? "nhwc" : "nchw", (int)onhwc,
                        res != nullptr, res_nhwc,
                        rc == LONNX_OK ? "tensor cores" : rc == LONNX_E_UNSUPPORTED ? "unsupported" : "error");
            if (rc == LONNX_OK && out_nhwc) *out_nhwc = onhwc ? 1 : 0;
            if (rc != LONNX_E_UNSUPPORTED) return rc;
        }
    }
    // direct conv: NCHW in and out
    if (conv_trace())
        fprintf(stderr, "[lonnx conv] N%d C%d %dx%d M%d k%dx%d s%d x_nhwc %d res %d/%d: direct\n", N, C, H, W, M, kh,
                kw, sh, x_nhwc, res != nullptr, res_nhwc);
    void *xt = nullptr, *rt = nullptr;
    if (x_nhwc) {
        const int rc = relayout(ctx, x, N, C, H, W, false, &xt);
        if (rc) return rc;
        x = (const float *)xt;
    }
    if (res && res_nhwc) {
        const int rc = relayout(ctx, res, N, M, Ho, Wo, false, &rt);
        if (rc) { if (xt) ctx_free(ctx, xt); return rc; }
        res = (const float *)rt;
    }
    k_conv2d_direct<<<grid_for(ctx, total), 256, 0, ctx->stream>>>(x, w, bias, y, N, C, H, W, M, kh, kw, sh, sw, pt,
                                                                     pl, dh, dw, group, Ho, Wo, res ? 0 : relu);
    ctx->launches++;
    cudaError_t e = cudaGetLastError();
    int rc = e == cudaSuccess ? LONNX_OK : cuda_error(e, "kernel launch");
    if (rc == LONNX_OK && res) {
        k_add_relu<<<grid_for(ctx, total), 256, 0, ctx->stream>>>(y, res, total, relu);
        ctx->launches++;
        e = cudaGetLastError();
        rc = e == cudaSuccess ? LONNX_OK : cuda_error(e, "kernel launch");
    }
    if (xt) ctx_free(ctx, xt);
    if (rt) ctx_free(ctx, rt);
    return rc;
}

}  // namespace lonnx
