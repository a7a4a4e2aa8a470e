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
        for (int64_t c = lane; c < inner_v; c += 32) dst[c] = __ldg(src + c);
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
    cudaStream_t st = ctx->stream;
    auto al = [](const void *p, int a) { return ((uintptr_t)p % a) == 0; };
    if (row_bytes % 16 == 0 && al(data, 16) && al(y, 16))
        k_gather_rows<uint4><<<g, 256, 0, st>>>((const uint4 *)data, outer, dim, row_bytes / 16, idx, n_idx, (uint4 *)y, ctx->dev_flags);
    else if (row_bytes % 4 == 0 && al(data, 4) && al(y, 4))
        k_gather_rows<uint32_t><<<g, 256, 0, st>>>((const uint32_t *)data, outer, dim, row_bytes / 4, idx, n_idx, (uint32_t *)y, ctx->dev_flags);
    else
        k_gather_rows<uint8_t><<<g, 256, 0, st>>>((const uint8_t *)data, outer, dim, row_bytes, idx, n_idx, (uint8_t *)y, ctx->dev_flags);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
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
