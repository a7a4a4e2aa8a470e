// Row kernels: softmax, LayerNorm, reductions, MaxPool.
//
// All HBM-bound.  A row of the innermost axis is owned by one warp and kept in
// registers between passes, so each element is read from HBM once and written
// once (the reference makes 6 full passes for Softmax, TensorOps.cs:1312-1330,
// and 9 node passes for a LayerNorm).  Reductions over a middle axis use one
// thread per output column so that the loads stay coalesced.
#include <float.h>

#include <algorithm>

#include "lonnx_internal.cuh"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

inline int grid_for(lonnx_ctx *ctx, int64_t work, int threads = 256) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

// ---------------------------------------------------------------------------
// Softmax along the innermost axis: one warp per row, row cached in registers
// (VPT values per lane, len <= 32*VPT).  The running max starts at 0.0f like
// the reference's ReduceMax (TensorOps.cs:1820); softmax is shift-invariant so
// this only matters when every logit is very negative.
template <int VPT>
__global__ void k_softmax_lastdim(const float *__restrict__ x, float *__restrict__ y,
                                  int64_t rows, int len) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float *xr = x + r * len;
        float v[VPT];
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            v[i] = c < len ? xr[c] : -INFINITY;
            m = fmaxf(m, v[i]);
        }
        m = warp_max(m);
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            v[i] = c < len ? expf(__fsub_rn(v[i], m)) : 0.0f;
            s = __fadd_rn(s, v[i]);
        }
        s = warp_sum(s);
        float *yr = y + r * len;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            if (c < len) yr[c] = __fdiv_rn(v[i], s);
        }
    }
}

// Softmax along a strided axis ([outer, len, inner], inner > 1) or a long
// innermost axis: one thread per (outer, inner) column, three passes.
__global__ void k_softmax_strided(const float *__restrict__ x, float *__restrict__ y,
                                  int64_t outer, int64_t len, int64_t inner) {
    const int64_t cols = outer * inner;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < cols; t += stride) {
        const int64_t o = t / inner, in = t % inner;
        const float *xp = x + o * len * inner + in;
        float *yp = y + o * len * inner + in;
        float m = 0.0f;
        for (int64_t j = 0; j < len; ++j) m = fmaxf(m, xp[j * inner]);
        float s = 0.0f;
        for (int64_t j = 0; j < len; ++j) {
            const float e = expf(__fsub_rn(xp[j * inner], m));
            yp[j * inner] = e;
            s = __fadd_rn(s, e);
        }
        for (int64_t j = 0; j < len; ++j) yp[j * inner] = __fdiv_rn(yp[j * inner], s);
    }
}

// ---------------------------------------------------------------------------
// LayerNorm over the last axis, following the exported node chain step by
// step in float: mean = sum(x)/n; d = x - mean; var = sum(d*d)/n;
// y = d / sqrt(var + eps) * gamma + beta.  With `res`, x = a + res first (the
// residual Add node that feeds the LayerNorm).
template <int VPT>
__global__ void k_layernorm(const float *__restrict__ x, const float *__restrict__ res,
                            const float *__restrict__ gamma, const float *__restrict__ beta,
                            float eps, float *__restrict__ y, int64_t rows, int cols) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const float fn = (float)cols;
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float *xr = x + r * cols;
        const float *rr = res ? res + r * cols : nullptr;
        float v[VPT];
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            float t = 0.0f;
            if (c < cols) {
                t = xr[c];
                if (rr) t = __fadd_rn(t, rr[c]);
            }
            v[i] = t;
            s = __fadd_rn(s, t);
        }
        const float mean = __fdiv_rn(warp_sum(s), fn);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            v[i] = __fsub_rn(v[i], mean);
            if (c < cols) q = __fadd_rn(q, __fmul_rn(v[i], v[i]));
        }
        const float var = __fdiv_rn(warp_sum(q), fn);
        const float sd = __fsqrt_rn(__fadd_rn(var, eps));
        float *yr = y + r * cols;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = lane + 32 * i;
            if (c < cols) yr[c] = __fadd_rn(__fmul_rn(__fdiv_rn(v[i], sd), gamma[c]), beta[c]);
        }
    }
}

// Generic LayerNorm for long rows: one block per row, values re-read from HBM.
__global__ void k_layernorm_block(const float *__restrict__ x, const float *__restrict__ res,
                                  const float *__restrict__ gamma, const float *__restrict__ beta,
                                  float eps, float *__restrict__ y, int64_t rows, int cols) {
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const float *xr = x + r * cols;
    const float *rr = res ? res + r * cols : nullptr;
    auto val = [&](int c) { return rr ? __fadd_rn(xr[c], rr[c]) : xr[c]; };
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        if (threadIdx.x < 32) t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
        __syncthreads();
        t = red[0];
        __syncthreads();
        return t;
    };
    float s = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, val(c));
    const float mean = __fdiv_rn(block_sum(s), (float)cols);
    float q = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = __fsub_rn(val(c), mean);
        q = __fadd_rn(q, __fmul_rn(d, d));
    }
    const float sd = __fsqrt_rn(__fadd_rn(__fdiv_rn(block_sum(q), (float)cols), eps));
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = __fsub_rn(val(c), mean);
        y[r * cols + c] = __fadd_rn(__fmul_rn(__fdiv_rn(d, sd), gamma[c]), beta[c]);
    }
}

// ---------------------------------------------------------------------------
// Reductions.  op: 0 sum, 1 max (running max from 0.0f, as the reference's
// ReduceMax, TensorOps.cs:1820), 2 mean (sum, then divide by the count).
__device__ __forceinline__ float reduce_finish(int op, float acc, int64_t r) {
    return op == LONNX_REDUCE_MEAN ? __fdiv_rn(acc, (float)r) : acc;
}

// [outer, r] -> [outer], one warp per row
__global__ void k_reduce_rows(int op, const float *__restrict__ x, float *__restrict__ y,
                              int64_t outer, int64_t r) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t o = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); o < outer; o += warps) {
        const float *xr = x + o * r;
        float acc = 0.0f;
        if (op == LONNX_REDUCE_MAX) {
            for (int64_t j = lane; j < r; j += 32) acc = fmaxf(acc, xr[j]);
            acc = warp_max(acc);
        } else {
            for (int64_t j = lane; j < r; j += 32) acc = __fadd_rn(acc, xr[j]);
            acc = warp_sum(acc);
        }
        if (lane == 0) y[o] = reduce_finish(op, acc, r);
    }
}

// [outer, r, inner] -> [outer, inner], one thread per output, sequential in r
__global__ void k_reduce_mid(int op, const float *__restrict__ x, float *__restrict__ y,
                             int64_t outer, int64_t r, int64_t inner) {
    const int64_t n = outer * inner;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += stride) {
        const int64_t o = t / inner, in = t % inner;
        const float *xp = x + o * r * inner + in;
        float acc = 0.0f;
        if (op == LONNX_REDUCE_MAX)
            for (int64_t j = 0; j < r; ++j) acc = fmaxf(acc, xp[j * inner]);
        else
            for (int64_t j = 0; j < r; ++j) acc = __fadd_rn(acc, xp[j * inner]);
        y[t] = reduce_finish(op, acc, r);
    }
}

// ---------------------------------------------------------------------------
// MaxPool2D (TensorOps.cs:1025-1099): window clipped to the input, max from
// -inf; the window ignores dilation as the reference's does.  blockIdx.y
// walks the (n, c) planes and x the output pixels of a plane, so the index
// arithmetic is one 32-bit division per output (a flat 64-bit index with
// three 64-bit divisions made this kernel instruction-bound at 29% of HBM).
// KH = KW = 0: runtime window; otherwise the window is unrolled and all its
// loads are issued before the max (predicated on the clipped window), so a
// thread has KH*KW loads in flight instead of one.
template <int KH, int KW>
__global__ void k_maxpool2d(const float *__restrict__ x, float *__restrict__ y, int64_t planes, int H,
                            int W, int kh, int kw, int sh, int sw, int pt, int pl, int Ho, int Wo) {
    if (KH > 0) { kh = KH; kw = KW; }
    const int per_plane = Ho * Wo;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= per_plane) return;
    const int oy = t / Wo, ox = t - oy * Wo;
    const int r0 = oy * sh - pt, c0 = ox * sw - pl;
    const int rmin = max(r0, 0), rmax = min(r0 + kh, H);
    const int cmin = max(c0, 0), cmax = min(c0 + kw, W);
    if (KH > 0) {
        // two planes per iteration: 2 * KH * KW independent loads in flight
        constexpr int T = KH * KW > 0 ? KH * KW : 1;
        int off[T];
        bool ok[T];
#pragma unroll
        for (int i = 0; i < KH; ++i)
#pragma unroll
            for (int j = 0; j < KW; ++j) {
                const int r = r0 + i, c = c0 + j;
                ok[i * KW + j] = r >= 0 && r < H && c >= 0 && c < W;
                off[i * KW + j] = r * W + c;
            }
        const int64_t step = (int64_t)gridDim.y;
        for (int64_t nc = blockIdx.y; nc < planes; nc += 2 * step) {
            const bool two = nc + step < planes;
            const float *xa = x + nc * H * W, *xb = x + (two ? nc + step : nc) * H * W;
            float va[T], vb[T];
#pragma unroll
            for (int i = 0; i < T; ++i) {
                va[i] = ok[i] ? __ldg(xa + off[i]) : -INFINITY;
                vb[i] = ok[i] ? __ldg(xb + off[i]) : -INFINITY;
            }
            float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
            for (int i = 0; i < T; ++i) {
                ma = fmaxf(ma, va[i]);
                mb = fmaxf(mb, vb[i]);
            }
            y[nc * per_plane + t] = ma;
            if (two) y[(nc + step) * per_plane + t] = mb;
        }
        return;
    }
    for (int64_t nc = blockIdx.y; nc < planes; nc += gridDim.y) {
        const float *xp = x + nc * H * W;
        float m = -INFINITY;
        {
            for (int r = rmin; r < rmax; ++r)
                for (int c = cmin; c < cmax; ++c) m = fmaxf(m, __ldg(xp + r * W + c));
        }
        y[nc * per_plane + t] = m;
    }
}

// MaxPool 3x3 / stride 2 / pad (1, 1) with W % 4 == 0 and Wo == W / 2 (the
// ResNet stem's pool).  A thread computes two adjacent outputs (columns 2j,
// 2j + 1) for RS consecutive output rows: input row r contributes the
// float4 x[r][4j .. 4j + 3] plus column 4j - 1, the left neighbour lane's .w
// through a shuffle (an explicit load on lane 0; -inf at j = 0, the pad).
// Each input row of the strip is loaded once, as 16 bytes, and all 2 RS + 1
// loads are issued before the first max.  The per-output scalar kernel
// issues 9 four-byte loads per output, each warp access spanning three
// 128-byte lines: L1-wavefront bound at ~69% of HBM.  Same maxima, so the
// same bits (fmaxf from -inf over the clipped window, any order).
template <int RS>
__global__ void __launch_bounds__(256) k_maxpool3s2(const float *__restrict__ x, float *__restrict__ y,
                                                    int64_t total, int H, int W, int Ho, int Wo, int strips) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = g < total;
    const int P = W >> 2;                                 // column pairs per output row
    const int64_t per_plane = (int64_t)P * strips;
    const int64_t plane = active ? g / per_plane : 0;
    const int t = active ? (int)(g - plane * per_plane) : 0;
    const int s = t / P, j = t - s * P, lane = threadIdx.x & 31;
    const int oy0 = s * RS, rin0 = 2 * oy0 - 1;
    const float *xp = x + plane * H * W + 4 * j;
    constexpr int NR = 2 * RS + 1;
    float4 v[NR];
    float h[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        const int r = rin0 + i;
        const bool in = active && r >= 0 && r < H;
        v[i] = in ? __ldg(reinterpret_cast<const float4 *>(xp + (int64_t)r * W))
                  : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        h[i] = in && j > 0 && lane == 0 ? __ldg(xp + (int64_t)r * W - 1) : -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        const float w = __shfl_up_sync(0xffffffffu, v[i].w, 1);
        if (j > 0 && lane > 0) h[i] = w;  // lane - 1 holds column pair j - 1 of the same strip
    }
    float a[NR], b[NR];  // row maxima for output columns 2j and 2j + 1
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        a[i] = fmaxf(fmaxf(h[i], v[i].x), v[i].y);
        b[i] = fmaxf(fmaxf(v[i].y, v[i].z), v[i].w);
    }
    if (!active) return;
    float *yp = y + plane * Ho * Wo + 2 * j;
#pragma unroll
    for (int o = 0; o < RS; ++o) {
        const int oy = oy0 + o;
        if (oy >= Ho) break;
        const float2 r2 = make_float2(fmaxf(fmaxf(a[2 * o], a[2 * o + 1]), a[2 * o + 2]),
                                      fmaxf(fmaxf(b[2 * o], b[2 * o + 1]), b[2 * o + 2]));
        *reinterpret_cast<float2 *>(yp + (int64_t)oy * Wo) = r2;
    }
}

// MaxPool over an NHWC tensor (the conv chain's internal layout, see
// graph.cpp): blockIdx.y walks the output rows (n, oy), blockIdx.x x
// threads the row's (ox, 4-channel group) pairs, so the per-thread index
// math is 32-bit and done once (float4 loads coalesced along C; C % 4 != 0
// falls back to one channel per thread).  Window clipped to the input, max
// from -inf: the same maxima as the NCHW kernels.
template <int V>
__global__ void k_maxpool2d_nhwc(const float *__restrict__ x, float *__restrict__ y, int N, int C, int H, int W,
                                 int kh, int kw, int sh, int sw, int pt, int pl, int Ho, int Wo) {
    const int CV = C / V, per_row = Wo * CV;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= per_row) return;
    const int cv = i % CV, ox = i / CV;
    const int c0 = ox * sw - pl, cmin = max(c0, 0), cmax = min(c0 + kw, W);
    for (int row = blockIdx.y; row < N * Ho; row += gridDim.y) {
        const int n = row / Ho, oy = row - n * Ho;
        const int r0 = oy * sh - pt, rmin = max(r0, 0), rmax = min(r0 + kh, H);
        const float *xn = x + (int64_t)n * H * W * C;
        float *yr = y + (int64_t)row * Wo * C;
        if constexpr (V == 4) {
            float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            for (int r = rmin; r < rmax; ++r)
                for (int c = cmin; c < cmax; ++c) {
                    const float4 v = __ldg(reinterpret_cast<const float4 *>(xn + ((int64_t)r * W + c) * C) + cv);
                    m = make_float4(fmaxf(m.x, v.x), fmaxf(m.y, v.y), fmaxf(m.z, v.z), fmaxf(m.w, v.w));
                }
            reinterpret_cast<float4 *>(yr)[i] = m;
        } else {
            float m = -INFINITY;
            for (int r = rmin; r < rmax; ++r)
                for (int c = cmin; c < cmax; ++c) m = fmaxf(m, __ldg(xn + ((int64_t)r * W + c) * C + cv));
            yr[i] = m;
        }
    }
}

// Sum / max / mean over the H x W pixels of an NHWC tensor [N, HW, C] ->
// [N, C], one thread per (n, c) (coalesced along C), in k_reduce_rows'
// order: 32 partial sums (element j goes to partial j % 32, each partial
// sequential in j), then the butterfly of warp_sum over the partials.  The
// result is bit-identical to reducing the same tensor in NCHW layout.
__global__ void k_reduce_hw_nhwc(int op, const float *__restrict__ x, float *__restrict__ y, int N, int HW, int C) {
    const int64_t total = (int64_t)N * C;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = t / C, c = t % C;
        const float *xp = x + n * HW * C + c;
        float a[32];
#pragma unroll
        for (int l = 0; l < 32; ++l) a[l] = 0.0f;
        for (int base = 0; base < HW; base += 32) {
#pragma unroll
            for (int l = 0; l < 32; ++l) {
                if (base + l < HW) {
                    const float v = __ldg(xp + (int64_t)(base + l) * C);
                    a[l] = op == LONNX_REDUCE_MAX ? fmaxf(a[l], v) : __fadd_rn(a[l], v);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int l = 0; l < o; ++l) a[l] = op == LONNX_REDUCE_MAX ? fmaxf(a[l], a[l + o]) : __fadd_rn(a[l], a[l + o]);
        y[t] = reduce_finish(op, a[0], HW);
    }
}

}  // namespace

using namespace lonnx;

namespace lonnx {
// Reduction of a dense [outer, r, inner] view (no allocation).
int reduce_view(lonnx_ctx *ctx, int op, const float *x, int64_t outer, int64_t r, int64_t inner,
                float *y) {
    if (inner == 1) {
        k_reduce_rows<<<grid_for(ctx, outer * 32), 256, 0, ctx->stream>>>(op, x, y, outer, r);
    } else {
        k_reduce_mid<<<grid_for(ctx, outer * inner), 256, 0, ctx->stream>>>(op, x, y, outer, r, inner);
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}
int transpose_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, const int64_t *shape, int rank,
                     const int64_t *perm, void *y);

int maxpool2d_nhwc(lonnx_ctx *ctx, const float *x, float *y, int N, int C, int H, int W, int kh, int kw, int sh,
                   int sw, int pt, int pl, int Ho, int Wo) {
    const bool v4 = C % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0;
    const int64_t per_row = (int64_t)Wo * (v4 ? C / 4 : C), rows = (int64_t)N * Ho;
    if (per_row <= 0 || rows <= 0) return LONNX_OK;
    if (per_row >= (1ll << 31) || rows >= (1ll << 31))
        return set_error(LONNX_E_UNSUPPORTED, "maxpool2d_nhwc: more than 2^31 outputs per row or rows");
    const int threads = per_row >= 256 ? 256 : 128;
    const dim3 grid((unsigned)((per_row + threads - 1) / threads), (unsigned)std::min<int64_t>(rows, 65535));
    if (v4)
        k_maxpool2d_nhwc<4><<<grid, threads, 0, ctx->stream>>>(x, y, N, C, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo);
    else
        k_maxpool2d_nhwc<1><<<grid, threads, 0, ctx->stream>>>(x, y, N, C, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

int reduce_hw_nhwc(lonnx_ctx *ctx, int op, const float *x, float *y, int N, int HW, int C) {
    const int64_t total = (int64_t)N * C;
    if (total <= 0) return LONNX_OK;
    if (HW <= 0) return set_error(LONNX_E_BADARG, "reduce: empty reduction");
    const int64_t blocks = std::min<int64_t>((total + 127) / 128, (int64_t)ctx->num_sms * 16);
    k_reduce_hw_nhwc<<<(unsigned)blocks, 128, 0, ctx->stream>>>(op, x, y, N, HW, C);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}
}  // namespace lonnx

extern "C" {

LONNX_API int lonnx_softmax_f32(lonnx_ctx *ctx, const float *x, float *y, int64_t outer,
                                int64_t len, int64_t inner) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!x || !y || outer < 0 || len < 0 || inner < 0) return set_error(LONNX_E_BADARG, "softmax: bad arguments");
    if (outer * len * inner == 0) return LONNX_OK;
    cudaStream_t st = ctx->stream;
    if (inner == 1 && len <= 1024) {
        const int64_t rows = outer;
        const int g = grid_for(ctx, rows * 32);
        if (len <= 128) k_softmax_lastdim<4><<<g, 256, 0, st>>>(x, y, rows, (int)len);
        else if (len <= 512) k_softmax_lastdim<16><<<g, 256, 0, st>>>(x, y, rows, (int)len);
        else k_softmax_lastdim<32><<<g, 256, 0, st>>>(x, y, rows, (int)len);
    } else {
        k_softmax_strided<<<grid_for(ctx, outer * inner), 256, 0, st>>>(x, y, outer, len, inner);
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

LONNX_API int lonnx_layernorm_f32(lonnx_ctx *ctx, const float *x, const float *res,
                                  const float *gamma, const float *beta, float eps, float *y,
                                  int64_t rows, int cols) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!x || !gamma || !beta || !y || rows < 0 || cols <= 0) return set_error(LONNX_E_BADARG, "layernorm: bad arguments");
    if (rows == 0) return LONNX_OK;
    const int g = grid_for(ctx, rows * 32);
    if (cols <= 128) return launch_pdl(ctx, k_layernorm<4>, dim3(g), dim3(256), 0, x, res, gamma, beta, eps, y, rows, cols);
    if (cols <= 384) return launch_pdl(ctx, k_layernorm<12>, dim3(g), dim3(256), 0, x, res, gamma, beta, eps, y, rows, cols);
    if (cols <= 1024) return launch_pdl(ctx, k_layernorm<32>, dim3(g), dim3(256), 0, x, res, gamma, beta, eps, y, rows, cols);
    return launch_pdl(ctx, k_layernorm_block, dim3((unsigned)rows), dim3(256), 0, x, res, gamma, beta, eps, y, rows, cols);
}

LONNX_API int lonnx_reduce_f32(lonnx_ctx *ctx, int op, const float *x, const int64_t *shape,
                               int rank, const int64_t *axes, int naxes, float *y) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!x || !y || rank < 0 || rank > 8 || naxes < 0 || naxes > rank || op < 0 || op > 2)
        return set_error(LONNX_E_BADARG, "reduce: bad arguments");
    bool red[8] = {false};
    int ax[8];
    int na = 0;
    if (naxes == 0) {
        for (int d = 0; d < rank; ++d) ax[na++] = d;
    } else {
        for (int i = 0; i < naxes; ++i) {
            int a = (int)axes[i];
            if (a < 0) a += rank;
            if (a < 0 || a >= rank) return set_error(LONNX_E_BADARG, "reduce: axis %lld out of range", (long long)axes[i]);
            if (red[a]) return set_error(LONNX_E_BADARG, "axes contains a repeated dimension.");
            ax[na++] = a;
        }
    }
    for (int i = 0; i < na; ++i) red[ax[i]] = true;
    int64_t total = 1;
    for (int d = 0; d < rank; ++d) total *= shape[d];
    if (total == 0) return LONNX_OK;
    // contiguous reduced block [lo, hi)?
    int lo = rank, hi = -1;
    for (int d = 0; d < rank; ++d)
        if (red[d]) { lo = d < lo ? d : lo; hi = d > hi ? d : hi; }
    bool contiguous = true;
    for (int d = lo; d <= hi; ++d) contiguous &= red[d];
    if (contiguous) {
        int64_t outer = 1, r = 1, inner = 1;
        for (int d = 0; d < lo; ++d) outer *= shape[d];
        for (int d = lo; d <= hi; ++d) r *= shape[d];
        for (int d = hi + 1; d < rank; ++d) inner *= shape[d];
        return reduce_view(ctx, op, x, outer, r, inner, y);
    }
    // general: move the reduced axes innermost (in the given order, as
    // ArrayUtilities.GetAxesPermutationForReduction does) into scratch
    int64_t perm[8];
    int np = 0;
    int64_t outer = 1, r = 1;
    for (int d = 0; d < rank; ++d)
        if (!red[d]) { perm[np++] = d; outer *= shape[d]; }
    for (int i = 0; i < na; ++i) { perm[np++] = ax[i]; r *= shape[ax[i]]; }
    void *tmp = nullptr;
    rc = ctx_scratch(ctx, (size_t)total * sizeof(float), &tmp);
    if (rc) return rc;
    rc = transpose_launch(ctx, x, 4, shape, rank, perm, tmp);
    if (rc) return rc;
    return reduce_view(ctx, op, (const float *)tmp, outer, r, 1, y);
}

LONNX_API int lonnx_maxpool2d_f32(lonnx_ctx *ctx, const float *x, float *y, int N, int C, int H,
                                  int W, int kh, int kw, int sh, int sw, int pt, int pl, int Ho,
                                  int Wo) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!x || !y || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0) return set_error(LONNX_E_BADARG, "maxpool: bad arguments");
    const int64_t total = (int64_t)N * C * Ho * Wo;
    if (total <= 0) return LONNX_OK;
    if ((int64_t)H * W >= ((int64_t)1 << 31) || (int64_t)Ho * Wo >= ((int64_t)1 << 31))
        return set_error(LONNX_E_UNSUPPORTED, "maxpool: plane of more than 2^31 elements");
    const int64_t planes = (int64_t)N * C;
    if (kh == 3 && kw == 3 && sh == 2 && sw == 2 && pt == 1 && pl == 1 && W % 4 == 0 && Wo == W / 2 &&
        Ho <= (H + 2) / 2 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 7) == 0) {
        constexpr int RS = 4;
        const int strips = (Ho + RS - 1) / RS;
        const int64_t tot = planes * (W / 4) * strips;
        k_maxpool3s2<RS><<<(unsigned)((tot + 255) / 256), 256, 0, ctx->stream>>>(x, y, tot, H, W, Ho, Wo, strips);
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    const int per_plane = Ho * Wo;
    // about 16 blocks per SM in all; each thread then walks several planes
    const int64_t bx = (per_plane + 255) / 256;
    const int64_t by = std::max<int64_t>(1, std::min<int64_t>({planes, 65535, ((int64_t)ctx->num_sms * 16 + bx - 1) / bx}));
    const dim3 grid((unsigned)bx, (unsigned)by);
    if (kh == 3 && kw == 3)
        k_maxpool2d<3, 3><<<grid, 256, 0, ctx->stream>>>(x, y, planes, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo);
    else if (kh == 2 && kw == 2)
        k_maxpool2d<2, 2><<<grid, 256, 0, ctx->stream>>>(x, y, planes, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo);
    else
        k_maxpool2d<0, 0><<<grid, 256, 0, ctx->stream>>>(x, y, planes, H, W, kh, kw, sh, sw, pt, pl, Ho, Wo);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // extern "C"
