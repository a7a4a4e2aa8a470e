// Internal declarations shared by the liblonnx_cuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/lonnx.h"

namespace lonnx {

// Device-side error flags, one int each, read and cleared by lonnx_sync().
enum DevFlag { FLAG_OOB = 0, FLAG_TIMEOUT = 1, FLAG_COUNT = 4 };

struct Allocator {
    // Caching allocator: freed blocks are kept per exact rounded size and
    // reused, so a graph that runs repeatedly reaches a steady state with no
    // cudaMalloc/cudaFree on the execute path.
    std::multimap<size_t, void *> free_blocks;
    std::unordered_map<void *, size_t> live;
    size_t bytes_reserved = 0;
    size_t limit = 0;  // 0 = none; LONNX_MEM_LIMIT (bytes) caps reservations
};

}  // namespace lonnx

struct lonnx_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int *dev_flags = nullptr;  // FLAG_COUNT ints
    int num_sms = 148;
    lonnx::Allocator alloc;
    int64_t launches = 0;
    // scratch used by ops that need a temporary (e.g. the split/transposed B
    // operand of a tensor-core GEMM); grown on demand, owned by the context
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    void *scratch2 = nullptr;
    size_t scratch2_bytes = 0;
    // while a graph is being captured, freed blocks are held (their addresses
    // are baked into the captured graph) instead of returning to the cache
    bool capturing = false;
    std::vector<void *> capture_hold;
};

namespace lonnx {

int set_error(int code, const char *fmt, ...);
int cuda_error(cudaError_t e, const char *what);
#define LONNX_CUDA(call)                                              \
    do {                                                              \
        cudaError_t e_ = (call);                                      \
        if (e_ != cudaSuccess) return ::lonnx::cuda_error(e_, #call); \
    } while (0)
#define LONNX_CHECK_LAUNCH(ctx)                                              \
    do {                                                                     \
        (ctx)->launches++;                                                   \
        cudaError_t e_ = cudaGetLastError();                                 \
        if (e_ != cudaSuccess) return ::lonnx::cuda_error(e_, "kernel launch"); \
    } while (0)

int ctx_alloc(lonnx_ctx *ctx, size_t bytes, void **out);
int ctx_free(lonnx_ctx *ctx, void *p);
int ctx_scratch(lonnx_ctx *ctx, size_t bytes, void **out);
// second, independent scratch slot (the GEMM's activation low parts)
int ctx_scratch2(lonnx_ctx *ctx, size_t bytes, void **out);
int device_guard(lonnx_ctx *ctx);

// kernels implemented in other translation units (device pointers, ctx stream)
int gemm_dispatch(lonnx_ctx *ctx, const float *A, const float *B, const float *bias, float *C,
                  int batch, int M, int N, int K, int64_t sA, int64_t sB, int64_t sC, int transB,
                  float alpha, float beta, int epi, const float *residual, bool split_k = false);
// Tensor-core GEMM: C = A . W^T with the weight pre-split into Whi, Wlo,
// both K-major ([N, K] row-major, see split_tf32_nk).  Returns
// LONNX_E_UNSUPPORTED when the operands do not fit its constraints.
// allow_scratch = false keeps the call free of device allocation (the
// activation split then happens inside the kernel).  split_k lets a call
// with too few output tiles split K across CTAs (workspace + fixed-order
// sum): deterministic for a shape, but the summation order then depends on
// M, so the graph executor (whose batch-sharded rows must not depend on the
// batch) never asks for it; the single-op Gemm entry point does.
int gemm_tc(lonnx_ctx *ctx, const float *A, const float *Whi, const float *Wlo, const float *bias,
            float *C, int M, int N, int K, int lda, int ldw, int ldc, float alpha, float beta,
            int epi, bool allow_scratch = true, bool split_k = false);
// Weight [K, N] (trans = 0) or [N, K] (trans = 1) -> hi, lo [N, K]:
// hi = w with the low 13 mantissa bits cleared, lo = w - hi (exact).
int split_tf32_nk(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int K, int N, int trans);
int64_t gemm_tc_min_work();
// Implicit-GEMM convolution geometry for the tensor-core kernel: x == nullptr
// selects the plain GEMM (A by TMA).  img_rows > 0 writes C as NCHW
// (row = image * img_rows + pixel, column = channel); res (same layout as
// C) is added after the bias and before the activation.
struct ConvArgs {
    const float *x = nullptr;
    int C = 0, H = 0, W = 0, kh = 0, kw = 0, sh = 1, sw = 1, pt = 0, pl = 0, dh = 1, dw = 1, Ho = 0, Wo = 0;
    int img_rows = 0;
    const float *res = nullptr;
    int tab = 0;  // set by conv_tc: the per-CTA tap table fits (see gemm_tc.cu)
    int nhwc = 0; // x is NHWC and the weights are tap-major: K order (ky, kx, c)
    // y (and res) NHWC: rows = output pixels, row-major [P, M] -- the GEMM
    // epilogue (TMA stores; the residual TMA-loaded into its staging blocks)
    int out_nhwc = 0;
};
// A small batch-1 network run as one launch on a cluster of CTAs (tiny.cu):
// a chain of layers; every CTA holds all weights and the current activation
// in shared memory (2 * max_elems + the weights <= TINY_MAX_SMEM_FLOATS).
enum { TINY_CONV = 0, TINY_MAXPOOL = 1, TINY_FC = 2, TINY_VIEW = 3 };
constexpr int TINY_MAX_LAYERS = 12;
constexpr int TINY_MAX_SMEM_FLOATS = 48 * 1024;
struct TinyLayer {
    int op;
    int C, H, W, M, kh, kw, sh, sw, pt, pl, dh, dw, Ho, Wo, relu;  // conv / pool (pool: C planes)
    int K, N;                                                      // fc
    const float *w, *bias;
    int woff;  // the weights' offset from the start of shared memory (floats), past both activation buffers
};
struct TinyProg {
    int n, in_elems, max_elems, smem_floats;
    TinyLayer L[TINY_MAX_LAYERS];
};
int tiny_chain(lonnx_ctx *ctx, const TinyProg &p, const float *x, float *y);
// Convs gathered from an NHWC copy of their input (one tap's 32 consecutive
// channels per K stage, 16-byte copies) with tap-major weights: C a multiple
// of 32 and a kernel of 2..63 taps.  x_nhwc: the input is already NHWC, so a
// 1x1 kernel gathers from it too (no transpose to pay for).
bool conv_nhwc_ok(int C, int kh, int kw, bool x_nhwc = false);
// MaxPool and the H x W reduction (global average pool) over NHWC tensors
int maxpool2d_nhwc(lonnx_ctx *ctx, const float *x, float *y, int N, int C, int H, int W, int kh, int kw, int sh,
                   int sw, int pt, int pl, int Ho, int Wo);
int reduce_hw_nhwc(lonnx_ctx *ctx, int op, const float *x, float *y, int N, int HW, int C);
// y[N, M, Ho, Wo] = conv(x, W) + bias (+ res) (ReLU if epi); W pre-split
// into Whi, Wlo [M, ldw] (K = C*kh*kw columns used).  P = N*Ho*Wo.
int conv_tc(lonnx_ctx *ctx, const ConvArgs &cv, const float *Whi, const float *Wlo, int ldw, const float *bias,
            float *y, int P, int M, int K, int epi);
// weight [M, K] -> hi, lo [M, ldk] (tf32 split, zero padded)
int split_pad_rows(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int M, int K, int ldk);
// the same split with the columns reordered from (c, tap) to (tap, c):
// hi[m][tap * C + c] = tf32(w[m][c * taps + tap]) (K = C * taps = ldk)
int split_rows_tapmajor(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int M, int C, int taps);
// Conv with optional pre-split weights (whi/wlo [M, ldk], ldk = (K+3)&~3, or
// nullptr) and an optional residual added before the ReLU.
// Layouts: x_nhwc / res_nhwc say how x and res are stored; want_out_nhwc
// asks for an NHWC y, which the tensor-core path gives (*out_nhwc says which
// layout y got; nullptr: NCHW is required).
int conv2d(lonnx_ctx *ctx, const float *x, const float *w, const float *whi, const float *wlo, const float *bias,
           const float *res, float *y, int N, int C, int H, int W, int M, int kh, int kw, int sh, int sw, int pt,
           int pl, int pb, int pr, int dh, int dw, int group, int relu, int w_tapmajor = 0, int x_nhwc = 0,
           int res_nhwc = 0, int *out_nhwc = nullptr);
// Fused attention on tensor cores (dh = 32, S <= 128); LONNX_E_UNSUPPORTED otherwise.
int attention_tc(lonnx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld, const float *mask,
                 float *out, int B, int S, int heads, int dh, float scale);
int gemm_simt(lonnx_ctx *ctx, const float *A, const float *B, const float *bias, float *C,
              int batch, int M, int N, int K, int64_t sA, int64_t sB, int64_t sC, int transB,
              float alpha, float beta, int epi, const float *residual);

// Programmatic dependent launch (sm_90+).  A kernel launched by launch_pdl
// may start while the previous kernel on the stream is still running: its
// CTAs do their set-up (barrier init, TMEM allocation, tensor-map prefetch)
// and then pdl_wait(), which returns once the previous kernel has completed
// and its memory is visible.  No global memory may be read or written
// before pdl_wait(): the buffers this kernel reads are being produced, and
// the ones it writes may still be read by the previous kernel.
// pdl_trigger() lets the next kernel be scheduled once every CTA of this one
// has started (or exited); without it that happens at this kernel's end.
// Kernels launched without the attribute see pdl_wait() return at once.
// LONNX_PDL=0 turns the attribute off (every launch fully serialised).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
int launch_pdl(lonnx_ctx *ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_error(e, "kernel launch");
    const cudaError_t e2 = cudaGetLastError();
    if (e2 != cudaSuccess) return cuda_error(e2, "kernel launch");
    return LONNX_OK;
}

}  // namespace lonnx

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Numerics shared by kernels -------------------------------------------------

// Abramowitz & Stegun 7.1.26 (the reference's MathOps.Erf,
// src/Lokad.Onnx.Tensors/MathOps.cs:989-1010), evaluated in float with expf.
__device__ __forceinline__ float lonnx_erf_as(float x) {
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f;
    const float a4 = -1.453152027f, a5 = 1.061405429f, p = 0.3275911f;
    const unsigned neg = x < 0.0f ? 0x80000000u : 0u;  // s * y with s = -1 is an exact negation
    x = fabsf(x);
    const float t = __frcp_rn(__fadd_rn(1.0f, __fmul_rn(p, x)));  // == RN(1 / d), as 1.0f / d
    float poly = __fadd_rn(__fmul_rn(a5, t), a4);
    poly = __fadd_rn(__fmul_rn(poly, t), a3);
    poly = __fadd_rn(__fmul_rn(poly, t), a2);
    poly = __fadd_rn(__fmul_rn(poly, t), a1);
    const float e = expf(__fmul_rn(-x, x));
    const float y = __fsub_rn(1.0f, __fmul_rn(__fmul_rn(poly, t), e));
    return __uint_as_float(__float_as_uint(y) ^ neg);
}

// GELU as the exported node chain computes it: Div(x, sqrt 2) -> Erf ->
// Add(1) -> Mul(x) -> Mul(0.5), each step rounded to float.
// x / fl(sqrt 2) correctly rounded.  For 2^-100 < |x| < inf one Markstein
// correction step of q0 = x * RN(1/c) gives the correctly rounded quotient
// (P. Markstein, "IA-64 and elementary functions", 2000: the remainder
// x - q0*c is exact in an FMA, then q = q0 + rem * RN(1/c)); this was
// checked against IEEE float division for every finite float.  Tiny,
// subnormal and non-finite x take the ordinary division.
__device__ __forceinline__ float lonnx_div_sqrt2(float x) {
    const float c = 1.41421353816986083984375f;
    const float r = 0.707106769084930419921875f;  // RN(1 / c)
    const float ax = fabsf(x);
    if (!(ax > 0x1p-100f && ax < INFINITY)) return __fdiv_rn(x, c);
    const float q0 = __fmul_rn(x, r);
    const float rem = __fmaf_rn(-q0, c, x);
    return __fmaf_rn(rem, r, q0);
}

__device__ __forceinline__ float lonnx_gelu_chain(float x) {
    const float a = lonnx_div_sqrt2(x);
    const float e = lonnx_erf_as(a);
    const float c = __fadd_rn(e, 1.0f);
    return __fmul_rn(__fmul_rn(x, c), 0.5f);
}

// The same GELU (A&S 7.1.26 erf of x / sqrt 2) for the fused GEMM epilogue,
// where it costs ~13 instructions instead of ~55: x times RN(1/sqrt 2)
// instead of the division, the hardware's approximate reciprocal for t and
// base-2 exponential for exp(-a^2) (flush-to-zero forms: one MUFU operation
// each; exp(-a^2) is subnormal only where erf is +-1 in float), the
// polynomial in FMAs and 0.5 x (1 + erf) as one FMA.  Each step is within a
// few ulp of the chain above, so the result is well inside the GEMM's own
// tolerance (|err| <= 1e-4 + 1e-4 |ref|); inf and NaN behave as in the chain.
__device__ __forceinline__ float lonnx_gelu_fast(float x) {
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f;
    const float a4 = -1.453152027f, a5 = 1.061405429f, p = 0.3275911f;
    const float ax = fabsf(x) * 0.707106769084930419921875f;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(p, ax, 1.0f)));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"((ax * ax) * -1.44269502162933349609375f));
    const float poly = fmaf(fmaf(fmaf(fmaf(a5, t, a4), t, a3), t, a2), t, a1);
    const float y = fmaf(-poly * t, e, 1.0f);
    const float h = 0.5f * x;
    return fmaf(h, copysignf(y, x), h);
}
