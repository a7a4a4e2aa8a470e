// Data movement: Gather (embedding row gather) and Transpose.
//
// Both are pure copies and bit-exact.  Gather moves whole rows of `inner`
// elements with 16-byte vectors when the row is 16-byte aligned, one warp per
// output row -- the embedding lookup of an encoder reads T rows of the
// [vocab, hidden] table and writes [T, hidden] once.
#include "lonnx_internal.cuh"

namespace {

template <typename V>
__global__ void k_gather_rows(const V *__restrict__ data, int64_t outer, int64_t dim,
                              int64_t inner_v, const int64_t *__restrict__ idx, int64_t n_idx,
                              V *__restrict__ y, int *__restrict__ flags) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t rows = outer * n_idx;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int64_t o = r / n_idx, j = r % n_idx;
        int64_t k = __ldg(idx + j);
        if (k < 0) k += dim;  // ArrayUtilities.HandleNegativeAxisOrIndex
        V *dst = y + r * inner_v;
        if (k < 0 || k >= dim) {
            if (lane == 0) atomicExch(flags + lonnx::FLAG_OOB, 1);
            for (int64_t c = lane; c < inner_v; c += 32) dst[c] = V{};
            continue;
        }
        const V *src = data + (o * dim + k) * inner_v;
        // four loads in flight per lane before the stores (a 384-float row is
        // 96 16-byte vectors: one batch of three per lane)
        for (int64_t c0 = lane; c0 < inner_v; c0 += 128) {
            V t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + 32 * u < inner_v) t[u] = __ldg(src + c0 + 32 * u);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + 32 * u < inner_v) dst[c0 + 32 * u] = t[u];
        }
    }
}

struct TransposeParams {
    int rank;
    int64_t out_dims[8];
    int64_t in_strides_perm[8];  // input stride of the dimension that output dim d reads
};

template <typename T>
__global__ void k_transpose(const T *__restrict__ x, T *__restrict__ y, int64_t n, TransposeParams p) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        int64_t rem = i, off = 0;
        for (int d = p.rank - 1; d >= 0; --d) {
            const int64_t c = rem % p.out_dims[d];
            rem /= p.out_dims[d];
            off += c * p.in_strides_perm[d];
        }
        y[i] = x[off];
    }
}

// Division of 32-bit unsigned n by a runtime-invariant d via multiply-high
// and shift (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, round-up method with N = 32): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, q = (umulhi(m, n) + n) >> l, exact for
// every n < 2^32 (the add is done in 64 bits).
struct FastDiv {
    uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0, 0};
    while ((1ull << f.l) < d) ++f.l;
    f.m = (uint32_t)((((1ull << f.l) - d) << 32) / d + 1);
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
    return (uint32_t)(((uint64_t)__umulhi(f.m, n) + n) >> f.l);
}

// Canonical transpose: size-1 dimensions dropped and input dimensions that
// stay adjacent in the output merged, so (0,2,1,3) of [B,S,12,32] stays
// rank 4 but e.g. (0,1,3,2) of [1,B,S,H] becomes rank 3.
struct TransposeRuns {
    int rank;          // dimensions of the output except the innermost run
    FastDiv out_dims[7];
    uint32_t in_strides_perm[7];  // in units of V
    uint32_t run_v;    // length of the innermost contiguous run, in V
    FastDiv run;
};

// Innermost axis kept: the output is runs of run_v contiguous V-sized
// vectors, each a contiguous run of the input.  One thread per vector.
template <typename V>
__global__ void k_transpose_runs(const V *__restrict__ x, V *__restrict__ y, uint32_t n_v, TransposeRuns p) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_v; i += stride) {
        uint32_t r = fdiv(i, p.run);
        const uint32_t j = i - r * p.run_v;
        uint32_t off = j;
        for (int d = p.rank - 1; d >= 0; --d) {
            const uint32_t q = fdiv(r, p.out_dims[d]);
            off += (r - q * p.out_dims[d].d) * p.in_strides_perm[d];
            r = q;
        }
        y[i] = __ldg(x + off);
    }
}

// Innermost axis moved: input dim `a` becomes the output's innermost and the
// input's innermost lands at output dim `b`.  A 32 x 32 tile of (a, last) is
// read along the input's innermost axis and written along the output's, via
// shared memory; the other dimensions form the tile's batch index.
struct TransposeTiles {
    int nb;                 // batch dimensions
    FastDiv bdims[6];
    uint32_t b_in[6], b_out[6];
    uint32_t len_a, len_l;  // extents of input dim a and of the input's innermost dim
    uint32_t in_stride_a, out_stride_l;
    FastDiv tiles_a, tiles_l;
    uint32_t n_tiles;
};

template <typename T>
__global__ void __launch_bounds__(256) k_transpose_tiles(const T *__restrict__ x, T *__restrict__ y, TransposeTiles p) {
    __shared__ T tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (uint32_t t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
        uint32_t rest = fdiv(t, p.tiles_l);
        const uint32_t l0 = (t - rest * p.tiles_l.d) * 32;
        uint32_t bi = fdiv(rest, p.tiles_a);
        const uint32_t a0 = (rest - bi * p.tiles_a.d) * 32;
        uint32_t in_base = 0, out_base = 0;
        for (int d = p.nb - 1; d >= 0; --d) {
            const uint32_t q = fdiv(bi, p.bdims[d]);
            const uint32_t c = bi - q * p.bdims[d].d;
            in_base += c * p.b_in[d];
            out_base += c * p.b_out[d];
            bi = q;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
            const uint32_t a = a0 + ty + k, l = l0 + tx;
            if (a < p.len_a && l < p.len_l) tile[ty + k][tx] = __ldg(x + in_base + a * p.in_stride_a + l);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
            const uint32_t l = l0 + ty + k, a = a0 + tx;
            if (a < p.len_a && l < p.len_l) y[out_base + l * p.out_stride_l + a] = tile[tx][ty + k];
        }
    }
}

struct StridedParams {
    int rank;
    int64_t out_dims[8];
    int64_t in_strides[8];
    int64_t out_strides[8];
};

// y[sum c_d * out_strides[d]] = x[in_offset + sum c_d * in_strides[d]] (Slice, Concat)
template <typename T>
__global__ void k_strided_copy(const T *__restrict__ x, T *__restrict__ y, int64_t n, int64_t in_offset,
                               StridedParams p) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        int64_t rem = i, ioff = in_offset, ooff = 0;
        for (int d = p.rank - 1; d >= 0; --d) {
            const int64_t c = rem % p.out_dims[d];
            rem /= p.out_dims[d];
            ioff += c * p.in_strides[d];
            ooff += c * p.out_strides[d];
        }
        y[ooff] = x[ioff];
    }
}

inline int grid_for(lonnx_ctx *ctx, int64_t work, int threads = 256) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

}  // namespace

namespace lonnx {

// Canonicalise and launch the run-copy or tiled transpose; returns 1 when
// the shape needs the generic per-element kernel (more than 6 batch dims).
int transpose_fast(lonnx_ctx *ctx, const void *x, int eb, const int64_t *shape, int rank,
                   const int64_t *perm, void *y, int64_t n) {
    // input dims of size > 1, renumbered; output order of those dims
    int64_t dims[8];
    int map[8], np = 0, nd = 0;
    for (int d = 0; d < rank; ++d) map[d] = shape[d] > 1 ? nd++ : -1;
    for (int d = 0; d < rank; ++d)
        if (shape[d] > 1) dims[map[d]] = shape[d];
    int order[8];
    for (int d = 0; d < rank; ++d) {
        const int64_t pd = perm[d] < 0 ? perm[d] + rank : perm[d];
        if (map[pd] >= 0) order[np++] = map[pd];
    }
    // merge input dims i, i+1 that are consecutive in the output
    int64_t mdims[8];
    int gid[8], mo[8], nm = 0;  // gid: input dim -> merged dim; mo: output order of merged dims
    {
        int next_in[8];
        for (int i = 0; i < nd; ++i) next_in[i] = -1;
        for (int k = 0; k + 1 < np; ++k)
            if (order[k + 1] == order[k] + 1) next_in[order[k]] = order[k + 1];
        for (int i = 0; i < nd; ++i) {
            if (i > 0 && next_in[i - 1] == i) {
                gid[i] = gid[i - 1];
                mdims[gid[i]] *= dims[i];
            } else {
                gid[i] = nm;
                mdims[nm++] = dims[i];
            }
        }
        int k2 = 0;
        for (int k = 0; k < np; ++k)
            if (k == 0 || gid[order[k]] != gid[order[k - 1]]) mo[k2++] = gid[order[k]];
    }
    cudaStream_t st = ctx->stream;
    if (nm <= 1) {  // a plain copy
        cudaError_t e = cudaMemcpyAsync(y, x, (size_t)(n * eb), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return set_error(LONNX_E_CUDA, "Transpose copy: %s", cudaGetErrorString(e));
        return LONNX_OK;
    }
    int64_t istr[8];
    {
        int64_t s = 1;
        for (int d = nm - 1; d >= 0; --d) { istr[d] = s; s *= mdims[d]; }
    }
    if (mo[nm - 1] == nm - 1) {
        // innermost run kept; pick the widest vector that divides the run
        const int64_t run_bytes = mdims[nm - 1] * eb;
        int vb = eb;
        for (int c = 16; c > eb; c >>= 1)
            if (run_bytes % c == 0 && (uintptr_t)x % c == 0 && (uintptr_t)y % c == 0) { vb = c; break; }
        const int64_t rv = run_bytes / vb, scale = mdims[nm - 1] * eb / vb;
        TransposeRuns p{};
        p.rank = nm - 1;
        for (int d = 0; d < nm - 1; ++d) {
            p.out_dims[d] = make_fastdiv((uint32_t)mdims[mo[d]]);
            p.in_strides_perm[d] = (uint32_t)(istr[mo[d]] / mdims[nm - 1] * scale);
        }
        p.run_v = (uint32_t)rv;
        p.run = make_fastdiv((uint32_t)rv);
        const uint32_t nv = (uint32_t)(n * eb / vb);
        const int g = grid_for(ctx, nv);
        switch (vb) {
        case 16: k_transpose_runs<uint4><<<g, 256, 0, st>>>((const uint4 *)x, (uint4 *)y, nv, p); break;
        case 8: k_transpose_runs<uint2><<<g, 256, 0, st>>>((const uint2 *)x, (uint2 *)y, nv, p); break;
        case 4: k_transpose_runs<uint32_t><<<g, 256, 0, st>>>((const uint32_t *)x, (uint32_t *)y, nv, p); break;
        case 2: k_transpose_runs<uint16_t><<<g, 256, 0, st>>>((const uint16_t *)x, (uint16_t *)y, nv, p); break;
        default: k_transpose_runs<uint8_t><<<g, 256, 0, st>>>((const uint8_t *)x, (uint8_t *)y, nv, p); break;
        }
        LONNX_CHECK_LAUNCH(ctx);
        return LONNX_OK;
    }
    if (nm - 2 > 6) return 1;
    const int a = mo[nm - 1], L = nm - 1;
    int b = 0;
    while (mo[b] != L) ++b;
    int64_t ostr[8];
    {
        int64_t s = 1;
        for (int k = nm - 1; k >= 0; --k) { ostr[k] = s; s *= mdims[mo[k]]; }
    }
    TransposeTiles p{};
    for (int k = 0; k < nm; ++k) {
        if (k == b || k == nm - 1) continue;
        p.bdims[p.nb] = make_fastdiv((uint32_t)mdims[mo[k]]);
        p.b_in[p.nb] = (uint32_t)istr[mo[k]];
        p.b_out[p.nb] = (uint32_t)ostr[k];
        ++p.nb;
    }
    p.len_a = (uint32_t)mdims[a];
    p.len_l = (uint32_t)mdims[L];
    p.in_stride_a = (uint32_t)istr[a];
    p.out_stride_l = (uint32_t)ostr[b];
    const uint32_t ta = (p.len_a + 31) / 32, tl = (p.len_l + 31) / 32;
    p.tiles_a = make_fastdiv(ta);
    p.tiles_l = make_fastdiv(tl);
    const int64_t nt = (int64_t)(n / ((int64_t)p.len_a * p.len_l)) * ta * tl;
    if (nt >= ((int64_t)1 << 32)) return 1;
    p.n_tiles = (uint32_t)nt;
    const int g = (int)std::min<int64_t>(nt, (int64_t)ctx->num_sms * 32);
    switch (eb) {
    case 1: k_transpose_tiles<uint8_t><<<g, 256, 0, st>>>((const uint8_t *)x, (uint8_t *)y, p); break;
    case 2: k_transpose_tiles<uint16_t><<<g, 256, 0, st>>>((const uint16_t *)x, (uint16_t *)y, p); break;
    case 4: k_transpose_tiles<uint32_t><<<g, 256, 0, st>>>((const uint32_t *)x, (uint32_t *)y, p); break;
    default: k_transpose_tiles<uint64_t><<<g, 256, 0, st>>>((const uint64_t *)x, (uint64_t *)y, p); break;
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

int transpose_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, const int64_t *shape, int rank,
                     const int64_t *perm, void *y) {
    TransposeParams p{};
    p.rank = rank;
    int64_t in_strides[8];
    int64_t s = 1;
    for (int d = rank - 1; d >= 0; --d) {
        in_strides[d] = s;
        s *= shape[d];
    }
    const int64_t n = s;
    bool seen[8] = {false};
    for (int d = 0; d < rank; ++d) {
        int64_t pd = perm[d] < 0 ? perm[d] + rank : perm[d];
        if (pd < 0 || pd >= rank || seen[pd])
            return set_error(LONNX_E_BADARG, "Transpose: invalid permutation");
        seen[pd] = true;
        p.out_dims[d] = shape[pd];
        p.in_strides_perm[d] = in_strides[pd];
    }
    if (n == 0) return LONNX_OK;
    if (n * elem_bytes < (int64_t)1 << 32 && (elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 ||
                                               elem_bytes == 8)) {
        const int rc = transpose_fast(ctx, x, elem_bytes, shape, rank, perm, y, n);
        if (rc != 1) return rc;
    }
    const int g = grid_for(ctx, n);
    switch (elem_bytes) {
    case 1: k_transpose<uint8_t><<<g, 256, 0, ctx->stream>>>((const uint8_t *)x, (uint8_t *)y, n, p); break;
    case 2: k_transpose<uint16_t><<<g, 256, 0, ctx->stream>>>((const uint16_t *)x, (uint16_t *)y, n, p); break;
    case 4: k_transpose<uint32_t><<<g, 256, 0, ctx->stream>>>((const uint32_t *)x, (uint32_t *)y, n, p); break;
    case 8: k_transpose<uint64_t><<<g, 256, 0, ctx->stream>>>((const uint64_t *)x, (uint64_t *)y, n, p); break;
    default: return set_error(LONNX_E_UNSUPPORTED, "Transpose: element size %d", elem_bytes);
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

int strided_copy_launch(lonnx_ctx *ctx, const void *x, int elem_bytes, int rank, const int64_t *out_dims,
                        const int64_t *in_strides, int64_t in_offset, void *y, const int64_t *out_strides) {
    if (rank < 0 || rank > 8) return set_error(LONNX_E_BADARG, "strided copy: rank out of range");
    StridedParams p{};
    p.rank = rank;
    int64_t n = 1;
    for (int d = 0; d < rank; ++d) {
        p.out_dims[d] = out_dims[d];
        p.in_strides[d] = in_strides[d];
        p.out_strides[d] = out_strides[d];
        n *= out_dims[d];
    }
    if (n == 0) return LONNX_OK;
    const int g = grid_for(ctx, n);
    switch (elem_bytes) {
    case 1: k_strided_copy<uint8_t><<<g, 256, 0, ctx->stream>>>((const uint8_t *)x, (uint8_t *)y, n, in_offset, p); break;
    case 4: k_strided_copy<uint32_t><<<g, 256, 0, ctx->stream>>>((const uint32_t *)x, (uint32_t *)y, n, in_offset, p); break;
    case 8: k_strided_copy<uint64_t><<<g, 256, 0, ctx->stream>>>((const uint64_t *)x, (uint64_t *)y, n, in_offset, p); break;
    default: return set_error(LONNX_E_UNSUPPORTED, "strided copy: element size %d", elem_bytes);
    }
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // namespace lonnx

using namespace lonnx;

extern "C" {

LONNX_API int lonnx_gather(lonnx_ctx *ctx, const void *data, int elem_bytes, int64_t outer,
                           int64_t dim, int64_t inner, const int64_t *idx, int64_t n_idx, void *y) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!data || !idx || !y || outer < 0 || dim <= 0 || inner < 0 || n_idx < 0)
        return set_error(LONNX_E_BADARG, "gather: bad arguments");
    if (outer * n_idx * inner == 0) return LONNX_OK;
    const int64_t row_bytes = inner * elem_bytes;
    const int64_t rows = outer * n_idx;
    const int g = grid_for(ctx, rows * 32);
    auto al = [](const void *p, int a) { return ((uintptr_t)p % a) == 0; };
    if (row_bytes % 16 == 0 && al(data, 16) && al(y, 16))
        return launch_pdl(ctx, k_gather_rows<uint4>, dim3(g), dim3(256), 0, (const uint4 *)data, outer, dim,
                          row_bytes / 16, idx, n_idx, (uint4 *)y, ctx->dev_flags);
    if (row_bytes % 4 == 0 && al(data, 4) && al(y, 4))
        return launch_pdl(ctx, k_gather_rows<uint32_t>, dim3(g), dim3(256), 0, (const uint32_t *)data, outer, dim,
                          row_bytes / 4, idx, n_idx, (uint32_t *)y, ctx->dev_flags);
    return launch_pdl(ctx, k_gather_rows<uint8_t>, dim3(g), dim3(256), 0, (const uint8_t *)data, outer, dim, row_bytes,
                      idx, n_idx, (uint8_t *)y, ctx->dev_flags);
}

LONNX_API int lonnx_transpose(lonnx_ctx *ctx, const void *x, int elem_bytes, const int64_t *shape,
                              int rank, const int64_t *perm, void *y) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!x || !y || !shape || rank < 0 || rank > 8) return set_error(LONNX_E_BADARG, "transpose: bad arguments");
    int64_t defperm[8];
    if (!perm) {
        for (int d = 0; d < rank; ++d) defperm[d] = rank - 1 - d;
        perm = defperm;
    }
    return transpose_launch(ctx, x, elem_bytes, shape, rank, perm, y);
}

}  // extern "C"
