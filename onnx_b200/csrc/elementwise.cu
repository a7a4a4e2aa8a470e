// Element-wise kernels: broadcast binary ops, unary ops, int64 -> float cast.
//
// All of these are HBM-bound: one read of each operand element and one write
// of the result.  The fast paths move 16-byte vectors with a grid-stride loop
// sized to a multiple of the SM count; the general broadcast path computes
// per-element source offsets from up to 8 output coordinates (stride 0 on
// broadcast dimensions), which is how the reference's BroadcastedTensor views
// index (src/Lokad.Onnx.Tensors/BroadcastedTensor.cs:11-53) without
// materialising the broadcast operand.
#include "lonnx_internal.cuh"

namespace {

constexpr int kMaxRank = 8;

struct BcastParams {
    int rank;
    int64_t dims[kMaxRank];
    int64_t sa[kMaxRank];
    int64_t sb[kMaxRank];
};

template <int OP>
__device__ __forceinline__ float binop(float l, float r) {
    if (OP == LONNX_ADD) return __fadd_rn(l, r);
    if (OP == LONNX_SUB) return __fsub_rn(l, r);
    if (OP == LONNX_MUL) return __fmul_rn(l, r);
    if (OP == LONNX_DIV) return __fdiv_rn(l, r);
    // Pow: x^2 is exactly x*x rounded once, which is what a correctly rounded
    // pow returns; other exponents use powf.
    if (r == 2.0f) return __fmul_rn(l, l);
    return powf(l, r);
}

template <int OP>
__global__ void k_binary_same(const float *__restrict__ a, const float *__restrict__ b,
                              float *__restrict__ y, int64_t n) {
    const int64_t n4 = n / 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const float4 *a4 = reinterpret_cast<const float4 *>(a);
    const float4 *b4 = reinterpret_cast<const float4 *>(b);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 u = __ldg(a4 + i), v = __ldg(b4 + i);
        y4[i] = make_float4(binop<OP>(u.x, v.x), binop<OP>(u.y, v.y), binop<OP>(u.z, v.z),
                            binop<OP>(u.w, v.w));
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = binop<OP>(a[i], b[i]);
}

// b (or a, when SWAP) repeats with period `inner` along the flat output:
// [.., inner] op [inner] (bias add, LayerNorm gamma/beta).
template <int OP, bool SWAP>
__global__ void k_binary_rowbcast(const float *__restrict__ full, const float *__restrict__ row,
                                  float *__restrict__ y, int64_t n, int64_t inner) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if ((inner & 3) == 0) {
        const int64_t n4 = n / 4, in4 = inner / 4;
        const float4 *f4 = reinterpret_cast<const float4 *>(full);
        const float4 *r4 = reinterpret_cast<const float4 *>(row);
        float4 *y4 = reinterpret_cast<float4 *>(y);
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
            float4 u = __ldg(f4 + i), v = __ldg(r4 + (i % in4));
            if (SWAP) { float4 t = u; u = v; v = t; }
            y4[i] = make_float4(binop<OP>(u.x, v.x), binop<OP>(u.y, v.y), binop<OP>(u.z, v.z),
                                binop<OP>(u.w, v.w));
        }
        return;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        float u = full[i], v = row[i % inner];
        y[i] = SWAP ? binop<OP>(v, u) : binop<OP>(u, v);
    }
}

// b (or a, when SWAP) is constant along the trailing `inner` elements of
// the flat output: [.., R, inner] op [.., R, 1..1] (masked mean pooling,
// unfused LayerNorm Sub/Div by the row statistics).
template <int OP, bool SWAP>
__global__ void k_binary_colbcast(const float *__restrict__ full, const float *__restrict__ col,
                                  float *__restrict__ y, int64_t n, int64_t inner, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {  // inner % 4 == 0, full and y 16-byte aligned
        const int64_t n4 = n / 4, in4 = inner / 4;
        const float4 *f4 = reinterpret_cast<const float4 *>(full);
        float4 *y4 = reinterpret_cast<float4 *>(y);
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
            const float4 u = __ldg(f4 + i);
            const float v = __ldg(col + i / in4);
            y4[i] = SWAP ? make_float4(binop<OP>(v, u.x), binop<OP>(v, u.y), binop<OP>(v, u.z), binop<OP>(v, u.w))
                         : make_float4(binop<OP>(u.x, v), binop<OP>(u.y, v), binop<OP>(u.z, v), binop<OP>(u.w, v));
        }
        return;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        const float u = full[i], v = col[i / inner];
        y[i] = SWAP ? binop<OP>(v, u) : binop<OP>(u, v);
    }
}

// scalar operand: a op s (or s op a when SWAP)
template <int OP, bool SWAP>
__global__ void k_binary_scalar(const float *__restrict__ full, const float *__restrict__ s,
                                float *__restrict__ y, int64_t n) {
    const float v = __ldg(s);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        float u = full[i];
        y[i] = SWAP ? binop<OP>(v, u) : binop<OP>(u, v);
    }
}

template <int OP>
__global__ void k_binary_general(const float *__restrict__ a, const float *__restrict__ b,
                                 float *__restrict__ y, int64_t n, BcastParams p) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        int64_t rem = i, oa = 0, ob = 0;
        for (int d = p.rank - 1; d >= 0; --d) {
            const int64_t c = rem % p.dims[d];
            rem /= p.dims[d];
            oa += c * p.sa[d];
            ob += c * p.sb[d];
        }
        y[i] = binop<OP>(a[oa], b[ob]);
    }
}

template <int OP>
__device__ __forceinline__ float unop(float x) {
    if (OP == LONNX_RELU) return x > 0.0f ? x : 0.0f;
    if (OP == LONNX_SQRT) return __fsqrt_rn(x);
    if (OP == LONNX_ERF) return lonnx_erf_as(x);
    if (OP == LONNX_EXP) return expf(x);
    // the fused GELU op (no single reference node): the fast evaluation of
    // the same A&S formula, within a few ulp of the exported node chain
    return lonnx_gelu_fast(x);
}

template <int OP>
__global__ void k_unary(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
    const int64_t n4 = n / 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 u = __ldg(x4 + i);
        y4[i] = make_float4(unop<OP>(u.x), unop<OP>(u.y), unop<OP>(u.z), unop<OP>(u.w));
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = unop<OP>(x[i]);
}

template <int OP>
__global__ void k_unary_scalar(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = unop<OP>(x[i]);
}

__global__ void k_cast_i64_f32(const int64_t *__restrict__ x, float *__restrict__ y, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = (float)x[i];
}

// Inference BatchNormalization over axis 1 of an [outer, C, inner] view, in
// the ONNX formula's operation order with every step rounded once:
// y = (x - mean) / sqrt(var + eps) * scale + B.  One CTA per (outer, c)
// plane (grid-stride), threads across the plane, float4 when it is aligned.
__global__ void k_batchnorm(const float *__restrict__ x, const float *__restrict__ scale,
                            const float *__restrict__ bias, const float *__restrict__ mean,
                            const float *__restrict__ var, float eps, float *__restrict__ y, int64_t planes,
                            int64_t C, int64_t inner, bool vec4) {
    for (int64_t p = blockIdx.x; p < planes; p += gridDim.x) {
        const int64_t c = p % C;
        const float m = mean[c], sc = scale[c], b = bias[c];
        const float den = __fsqrt_rn(__fadd_rn(var[c], eps));
        const float *xp = x + p * inner;
        float *yp = y + p * inner;
        auto f = [&](float v) { return __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(v, m), den), sc), b); };
        if (vec4) {
            const float4 *x4 = reinterpret_cast<const float4 *>(xp);
            float4 *y4 = reinterpret_cast<float4 *>(yp);
            for (int64_t i = threadIdx.x; i < inner / 4; i += blockDim.x) {
                float4 u = __ldg(x4 + i);
                y4[i] = make_float4(f(u.x), f(u.y), f(u.z), f(u.w));
            }
        } else {
            for (int64_t i = threadIdx.x; i < inner; i += blockDim.x) yp[i] = f(xp[i]);
        }
    }
}

inline int grid_for(lonnx_ctx *ctx, int64_t work, int threads = 256) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

template <int OP>
int launch_binary(lonnx_ctx *ctx, const float *a, const int64_t *as, int ar, const float *b,
                  const int64_t *bs, int br, float *y, const int64_t *os, int orank, int64_t n) {
    const int T = 256;
    cudaStream_t st = ctx->stream;
    int64_t na = 1, nb = 1;
    for (int i = 0; i < ar; ++i) na *= as[i];
    for (int i = 0; i < br; ++i) nb *= bs[i];
    if (na == n && nb == n) {
        const bool vec = aligned16(a) && aligned16(b) && aligned16(y);
        if (vec) k_binary_same<OP><<<grid_for(ctx, n / 4 + 1, T), T, 0, st>>>(a, b, y, n);
        else k_binary_general<OP><<<grid_for(ctx, n, T), T, 0, st>>>(a, b, y, n, BcastParams{1, {n}, {1}, {1}});
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if (nb == 1 && na == n) {
        k_binary_scalar<OP, false><<<grid_for(ctx, n, T), T, 0, st>>>(a, b, y, n);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if (na == 1 && nb == n) {
        k_binary_scalar<OP, true><<<grid_for(ctx, n, T), T, 0, st>>>(b, a, y, n);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    // row broadcast: the small operand's shape equals the output's trailing dims
    auto trailing = [&](const int64_t *s, int r, int64_t cnt) {
        if (cnt == n) return false;
        int k = r;
        while (k > 0 && s[r - k] == 1) --k;  // strip leading 1s
        if (k > orank) return false;
        for (int i = 0; i < k; ++i)
            if (s[r - k + i] != os[orank - k + i]) return false;
        return true;
    };
    const bool vecok = aligned16(a) && aligned16(b) && aligned16(y);
    if (na == n && trailing(bs, br, nb) && vecok) {
        k_binary_rowbcast<OP, false><<<grid_for(ctx, n / 4 + 1, T), T, 0, st>>>(a, b, y, n, nb);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if (nb == n && trailing(as, ar, na) && vecok) {
        k_binary_rowbcast<OP, true><<<grid_for(ctx, n / 4 + 1, T), T, 0, st>>>(b, a, y, n, na);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    // column broadcast: the small operand's shape is the output's leading
    // dims followed by 1s; returns the run length it is constant over
    auto leading = [&](const int64_t *s, int r, int64_t cnt) -> int64_t {
        if (cnt == n || cnt <= 1 || r > orank) return 0;
        int last = -1;
        for (int d = 0; d < orank; ++d) {
            const int i = d - (orank - r);
            const int64_t sd = i >= 0 ? s[i] : 1;
            if (sd != 1) {
                if (sd != os[d]) return 0;
                last = d;
            }
        }
        for (int d = 0; d <= last; ++d) {
            const int i = d - (orank - r);
            if ((i >= 0 ? s[i] : 1) != os[d]) return 0;
        }
        int64_t inner = 1;
        for (int d = last + 1; d < orank; ++d) inner *= os[d];
        return inner > 1 && cnt * inner == n ? inner : 0;
    };
    if (int64_t inner = na == n ? leading(bs, br, nb) : 0) {
        const int vec = (inner & 3) == 0 && aligned16(a) && aligned16(y);
        k_binary_colbcast<OP, false><<<grid_for(ctx, (vec ? n / 4 : n) + 1, T), T, 0, st>>>(a, b, y, n, inner, vec);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if (int64_t inner = nb == n ? leading(as, ar, na) : 0) {
        const int vec = (inner & 3) == 0 && aligned16(b) && aligned16(y);
        k_binary_colbcast<OP, true><<<grid_for(ctx, (vec ? n / 4 : n) + 1, T), T, 0, st>>>(b, a, y, n, inner, vec);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    BcastParams p{};
    p.rank = orank;
    int64_t sa = 1, sb = 1;
    for (int d = orank - 1; d >= 0; --d) {
        const int ia = d - (orank - ar), ib = d - (orank - br);
        const int64_t da = ia >= 0 ? as[ia] : 1, db = ib >= 0 ? bs[ib] : 1;
        p.dims[d] = os[d];
        p.sa[d] = (da == 1 && os[d] != 1) ? 0 : sa;
        p.sb[d] = (db == 1 && os[d] != 1) ? 0 : sb;
        sa *= da;
        sb *= db;
    }
    k_binary_general<OP><<<grid_for(ctx, n, T), T, 0, st>>>(a, b, y, n, p);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // namespace

using namespace lonnx;

extern "C" {

LONNX_API int lonnx_broadcast_shape(const int64_t *a, int ar, const int64_t *b, int br,
                                    int64_t *out, int *orank) {
    if (ar < 0 || br < 0 || ar > kMaxRank || br > kMaxRank || !orank)
        return set_error(LONNX_E_BADARG, "broadcast: rank out of range");
    const int r = ar > br ? ar : br;
    for (int i = 0; i < r; ++i) {
        const int ia = i - (r - ar), ib = i - (r - br);
        const int64_t da = ia >= 0 ? a[ia] : 1, db = ib >= 0 ? b[ib] : 1;
        if (da == db || db == 1) out[i] = da;
        else if (da == 1) out[i] = db;
        else return set_error(LONNX_E_SHAPE, "The tensors are not compatible for broadcasting (dim %d: %lld vs %lld).",
                              i, (long long)da, (long long)db);
    }
    *orank = r;
    return LONNX_OK;
}

LONNX_API int lonnx_binary_f32(lonnx_ctx *ctx, int op, const float *a, const int64_t *as, int ar,
                               const float *b, const int64_t *bs, int br, float *y) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!a || !b || !y) return set_error(LONNX_E_BADARG, "binary: null tensor");
    int64_t os[kMaxRank];
    int orank = 0;
    rc = lonnx_broadcast_shape(as, ar, bs, br, os, &orank);
    if (rc) return rc;
    int64_t n = 1;
    for (int i = 0; i < orank; ++i) n *= os[i];
    if (n == 0) return LONNX_OK;
    switch (op) {
    case LONNX_ADD: return launch_binary<LONNX_ADD>(ctx, a, as, ar, b, bs, br, y, os, orank, n);
    case LONNX_SUB: return launch_binary<LONNX_SUB>(ctx, a, as, ar, b, bs, br, y, os, orank, n);
    case LONNX_MUL: return launch_binary<LONNX_MUL>(ctx, a, as, ar, b, bs, br, y, os, orank, n);
    case LONNX_DIV: return launch_binary<LONNX_DIV>(ctx, a, as, ar, b, bs, br, y, os, orank, n);
    case LONNX_POW: return launch_binary<LONNX_POW>(ctx, a, as, ar, b, bs, br, y, os, orank, n);
    default: return set_error(LONNX_E_BADARG, "binary: unknown op %d", op);
    }
}

LONNX_API int lonnx_unary_f32(lonnx_ctx *ctx, int op, const float *x, float *y, int64_t n) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (n == 0) return LONNX_OK;
    if (!x || !y || n < 0) return set_error(LONNX_E_BADARG, "unary: bad arguments");
    const int T = 256;
    // the float4 path needs 16-byte alignment; unaligned views take the scalar kernel
    const bool vec = aligned16(x) && aligned16(y);
    const int g = grid_for(ctx, (vec ? n / 4 : n) + 1, T);
    cudaStream_t st = ctx->stream;
    if (!vec) {
        switch (op) {
        case LONNX_RELU: k_unary_scalar<LONNX_RELU><<<g, T, 0, st>>>(x, y, n); break;
        case LONNX_SQRT: k_unary_scalar<LONNX_SQRT><<<g, T, 0, st>>>(x, y, n); break;
        case LONNX_ERF: k_unary_scalar<LONNX_ERF><<<g, T, 0, st>>>(x, y, n); break;
        case LONNX_EXP: k_unary_scalar<LONNX_EXP><<<g, T, 0, st>>>(x, y, n); break;
        case LONNX_GELU_ERF: k_unary_scalar<LONNX_GELU_ERF><<<g, T, 0, st>>>(x, y, n); break;
        default: return set_error(LONNX_E_BADARG, "unary: unknown op %d", op);
        }
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    switch (op) {
    case LONNX_RELU: k_unary<LONNX_RELU><<<g, T, 0, st>>>(x, y, n); break;
    case LONNX_SQRT: k_unary<LONNX_SQRT><<<g, T, 0, st>>>(x, y, n); break;
    case LONNX_ERF: k_unary<LONNX_ERF><<<g, T, 0, st>>>(x, y, n); break;
    case LONNX_EXP: k_unary<LONNX_EXP><<<g, T, 0, st>>>(x, y, n); break;
    case LONNX_GELU_ERF: k_unary<LONNX_GELU_ERF><<<g, T, 0, st>>>(x, y, n); break;
    default: return set_error(LONNX_E_BADARG, "unary: unknown op %d", op);
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

LONNX_API int lonnx_batchnorm_f32(lonnx_ctx *ctx, const float *x, const float *scale, const float *bias,
                                  const float *mean, const float *var, float eps, float *y, int64_t outer,
                                  int64_t channels, int64_t inner) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (outer < 0 || channels < 0 || inner < 0) return set_error(LONNX_E_BADARG, "batchnorm: negative size");
    const int64_t planes = outer * channels;
    if (planes == 0 || inner == 0) return LONNX_OK;
    if (!x || !scale || !bias || !mean || !var || !y) return set_error(LONNX_E_BADARG, "batchnorm: null tensor");
    const bool vec4 = inner % 4 == 0 && aligned16(x) && aligned16(y);
    const int threads = inner >= 1024 ? 256 : 128;
    const int64_t cap = (int64_t)ctx->num_sms * 16;
    k_batchnorm<<<(int)(planes < cap ? planes : cap), threads, 0, ctx->stream>>>(x, scale, bias, mean, var, eps, y,
                                                                                 planes, channels, inner, vec4);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

LONNX_API int lonnx_cast_i64_f32(lonnx_ctx *ctx, const int64_t *x, float *y, int64_t n) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (n == 0) return LONNX_OK;
    k_cast_i64_f32<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(x, y, n);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // extern "C"
