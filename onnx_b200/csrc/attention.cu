// Fused scaled-dot-product attention of a BERT layer (fp32, SIMT).
//
// Replaces the node chain MatMul(Q, K^T) -> Div(sqrt dh) -> Add(mask) ->
// Softmax -> MatMul(P, V) and the Reshape/Transpose nodes around it
// (src/Lokad.Onnx.Tensors/TensorOps.cs:600-704,1312-1330,1358-1407): Q, K and
// V are read in place from the [B, S, ld] projection output (head h at column
// h*dh) and the context is written straight into [B, S, heads*dh], so the
// [B, heads, S, S] score tensor never reaches HBM.
//
// One CTA per (batch, head, 128-query tile), one thread per query row.  K and
// V of the head are staged in shared memory; each thread keeps its scores in
// a padded shared-memory row.  Every step follows the node chain's float
// rounding: score = (q.k) / scale + mask; softmax with the running max
// starting at 0 (the reference ReduceMax, TensorOps.cs:1820); sequential
// sums over keys, as the reference's i-j-k matmul accumulates.
#include <stdlib.h>

#include "lonnx_internal.cuh"

namespace {

constexpr int QT = 128;  // query rows per CTA

template <int DH>
__global__ void __launch_bounds__(QT)
k_attention(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
            int64_t ld, const float *__restrict__ maskadd, float *__restrict__ out, int S, int heads,
            float scale) {
    extern __shared__ float sm[];
    float *Ks = sm;                      // [S][DH]
    float *Vs = Ks + (size_t)S * DH;     // [S][DH]
    float *P = Vs + (size_t)S * DH;      // [QT][S+1]
    const int bh = blockIdx.y;
    const int b = bh / heads, h = bh % heads;
    const int i0 = blockIdx.x * QT;
    const int tid = threadIdx.x;
    const int64_t base = (int64_t)b * S * ld + (int64_t)h * DH;
    // stage K and V (float4 when DH % 4 == 0)
    for (int e = tid; e < S * DH / 4; e += QT) {
        const int r = e / (DH / 4), c = (e % (DH / 4)) * 4;
        const float4 kv = *reinterpret_cast<const float4 *>(k + base + (int64_t)r * ld + c);
        const float4 vv = *reinterpret_cast<const float4 *>(v + base + (int64_t)r * ld + c);
        *reinterpret_cast<float4 *>(Ks + r * DH + c) = kv;
        *reinterpret_cast<float4 *>(Vs + r * DH + c) = vv;
    }
    __syncthreads();
    const int i = i0 + tid;
    if (i >= S) return;
    float qr[DH];
    const float *qp = q + base + (int64_t)i * ld;
#pragma unroll
    for (int d = 0; d < DH; d += 4) {
        const float4 t = *reinterpret_cast<const float4 *>(qp + d);
        qr[d] = t.x; qr[d + 1] = t.y; qr[d + 2] = t.z; qr[d + 3] = t.w;
    }
    float *pr = P + (size_t)tid * (S + 1);
    const float *mrow = maskadd ? maskadd + (int64_t)b * S : nullptr;
    float mx = 0.0f;
    for (int j = 0; j < S; ++j) {
        const float *kr = Ks + j * DH;
        float dot = 0.0f;
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
            const float4 kk = *reinterpret_cast<const float4 *>(kr + d);
            dot = __fadd_rn(dot, __fmul_rn(qr[d], kk.x));
            dot = __fadd_rn(dot, __fmul_rn(qr[d + 1], kk.y));
            dot = __fadd_rn(dot, __fmul_rn(qr[d + 2], kk.z));
            dot = __fadd_rn(dot, __fmul_rn(qr[d + 3], kk.w));
        }
        float s = __fdiv_rn(dot, scale);
        if (mrow) s = __fadd_rn(s, mrow[j]);
        pr[j] = s;
        mx = fmaxf(mx, s);
    }
    float sum = 0.0f;
    for (int j = 0; j < S; ++j) {
        const float e = expf(__fsub_rn(pr[j], mx));
        pr[j] = e;
        sum = __fadd_rn(sum, e);
    }
    float acc[DH];
#pragma unroll
    for (int d = 0; d < DH; ++d) acc[d] = 0.0f;
    for (int j = 0; j < S; ++j) {
        const float p = __fdiv_rn(pr[j], sum);
        const float *vr = Vs + j * DH;
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
            const float4 vv = *reinterpret_cast<const float4 *>(vr + d);
            acc[d] = __fadd_rn(acc[d], __fmul_rn(p, vv.x));
            acc[d + 1] = __fadd_rn(acc[d + 1], __fmul_rn(p, vv.y));
            acc[d + 2] = __fadd_rn(acc[d + 2], __fmul_rn(p, vv.z));
            acc[d + 3] = __fadd_rn(acc[d + 3], __fmul_rn(p, vv.w));
        }
    }
    float *op = out + ((int64_t)b * S + i) * ((int64_t)heads * DH) + (int64_t)h * DH;
#pragma unroll
    for (int d = 0; d < DH; d += 4) *reinterpret_cast<float4 *>(op + d) = make_float4(acc[d], acc[d + 1], acc[d + 2], acc[d + 3]);
}

// Online-softmax variant: scores stay in registers, 32 keys at a time; the
// running max starts at 0 like the reference's ReduceMax (shift-invariant),
// exp-sums and the P.V accumulation are rescaled when the max grows, and the
// division by the row sum happens once at the end.  FMA contractions; the
// result matches the node chain within fp32 rounding.
template <int DH>
__global__ void __launch_bounds__(QT)
k_attention_online(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                   int64_t ld, const float *__restrict__ maskadd, float *__restrict__ out, int S, int heads,
                   float scale) {
    extern __shared__ float sm[];
    float *Ks = sm;                   // [S][DH]
    float *Vs = Ks + (size_t)S * DH;  // [S][DH]
    float *Ms = Vs + (size_t)S * DH;  // [S] additive mask
    const int bh = blockIdx.y;
    const int b = bh / heads, h = bh % heads;
    const int tid = threadIdx.x;
    const int64_t base = (int64_t)b * S * ld + (int64_t)h * DH;
    for (int e = tid; e < S * DH / 4; e += QT) {
        const int r = e / (DH / 4), c = (e % (DH / 4)) * 4;
        *reinterpret_cast<float4 *>(Ks + r * DH + c) = __ldg(reinterpret_cast<const float4 *>(k + base + (int64_t)r * ld + c));
        *reinterpret_cast<float4 *>(Vs + r * DH + c) = __ldg(reinterpret_cast<const float4 *>(v + base + (int64_t)r * ld + c));
    }
    for (int j = tid; j < S; j += QT) Ms[j] = maskadd ? maskadd[(int64_t)b * S + j] : 0.0f;
    __syncthreads();
    const int i = blockIdx.x * QT + tid;
    if (i >= S) return;
    const float inv_scale = 1.0f / scale;
    float qr[DH];
    const float *qp = q + base + (int64_t)i * ld;
#pragma unroll
    for (int d = 0; d < DH; d += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(qp + d));
        qr[d] = t.x * inv_scale; qr[d + 1] = t.y * inv_scale; qr[d + 2] = t.z * inv_scale; qr[d + 3] = t.w * inv_scale;
    }
    float acc[DH];
#pragma unroll
    for (int d = 0; d < DH; ++d) acc[d] = 0.0f;
    float m = 0.0f, l = 0.0f;
    constexpr int KC = 32;
    for (int j0 = 0; j0 < S; j0 += KC) {
        float sc[KC];
        float cmax = m;
#pragma unroll
        for (int jj = 0; jj < KC; ++jj) {
            const int j = j0 + jj;
            float dot = -INFINITY;
            if (j < S) {
                const float *kr = Ks + j * DH;
                dot = 0.0f;
#pragma unroll
                for (int d = 0; d < DH; d += 4) {
                    const float4 kk = *reinterpret_cast<const float4 *>(kr + d);
                    dot = fmaf(qr[d], kk.x, dot);
                    dot = fmaf(qr[d + 1], kk.y, dot);
                    dot = fmaf(qr[d + 2], kk.z, dot);
                    dot = fmaf(qr[d + 3], kk.w, dot);
                }
                dot += Ms[j];
            }
            sc[jj] = dot;
            cmax = fmaxf(cmax, dot);
        }
        const float corr = expf(m - cmax);
        m = cmax;
        l *= corr;
#pragma unroll
        for (int d = 0; d < DH; ++d) acc[d] *= corr;
#pragma unroll
        for (int jj = 0; jj < KC; ++jj) {
            const int j = j0 + jj;
            if (j >= S) break;
            const float p = expf(sc[jj] - m);
            l += p;
            const float *vr = Vs + j * DH;
#pragma unroll
            for (int d = 0; d < DH; d += 4) {
                const float4 vv = *reinterpret_cast<const float4 *>(vr + d);
                acc[d] = fmaf(p, vv.x, acc[d]);
                acc[d + 1] = fmaf(p, vv.y, acc[d + 1]);
                acc[d + 2] = fmaf(p, vv.z, acc[d + 2]);
                acc[d + 3] = fmaf(p, vv.w, acc[d + 3]);
            }
        }
    }
    const float inv_l = 1.0f / l;
    float *op = out + ((int64_t)b * S + i) * ((int64_t)heads * DH) + (int64_t)h * DH;
#pragma unroll
    for (int d = 0; d < DH; d += 4)
        *reinterpret_cast<float4 *>(op + d) = make_float4(acc[d] * inv_l, acc[d + 1] * inv_l, acc[d + 2] * inv_l, acc[d + 3] * inv_l);
}

template <int DH>
int launch_attn(lonnx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld,
                const float *mask, float *out, int B, int S, int heads, float scale) {
    static const bool exact = getenv("LONNX_ATTN_EXACT") != nullptr;
    static const bool simt = getenv("LONNX_ATTN_SIMT") != nullptr || getenv("LONNX_DISABLE_TC") != nullptr;
    if (!exact && !simt) {
        const int rc = lonnx::attention_tc(ctx, q, k, v, ld, mask, out, B, S, heads, DH, scale);
        if (rc != LONNX_E_UNSUPPORTED) return rc;
    }
    dim3 grid((S + QT - 1) / QT, B * heads);
    if (!exact) {
        const size_t smem = ((size_t)2 * S * DH + S) * sizeof(float);
        if (smem <= 227 * 1024) {
            LONNX_CUDA(cudaFuncSetAttribute(k_attention_online<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k_attention_online<DH><<<grid, QT, smem, ctx->stream>>>(q, k, v, ld, mask, out, S, heads, scale);
            LONNX_CHECK_LAUNCH(ctx);
            return LONNX_OK;
        }
    }
    const size_t smem = ((size_t)2 * S * DH + (size_t)QT * (S + 1)) * sizeof(float);
    if (smem > 227 * 1024)
        return lonnx::set_error(LONNX_E_UNSUPPORTED, "attention: sequence length %d too long for the fused kernel", S);
    LONNX_CUDA(cudaFuncSetAttribute(k_attention<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_attention<DH><<<grid, QT, smem, ctx->stream>>>(q, k, v, ld, mask, out, S, heads, scale);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // namespace

using namespace lonnx;

extern "C" LONNX_API int lonnx_attention_f32(lonnx_ctx *ctx, const float *q, const float *k,
                                             const float *v, int64_t ld, const float *maskadd,
                                             float *out, int B, int S, int heads, int dh,
                                             float scale) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!q || !k || !v || !out || B < 0 || S < 0 || heads <= 0 || ld % 4 || (uintptr_t)q % 16 ||
        (uintptr_t)k % 16 || (uintptr_t)v % 16 || (uintptr_t)out % 16)
        return set_error(LONNX_E_BADARG, "attention: bad arguments (rows must be 16-byte aligned)");
    if (B == 0 || S == 0) return LONNX_OK;
    switch (dh) {
    case 16: return launch_attn<16>(ctx, q, k, v, ld, maskadd, out, B, S, heads, scale);
    case 32: return launch_attn<32>(ctx, q, k, v, ld, maskadd, out, B, S, heads, scale);
    case 64: return launch_attn<64>(ctx, q, k, v, ld, maskadd, out, B, S, heads, scale);
    default: return set_error(LONNX_E_UNSUPPORTED, "attention: head size %d", dh);
    }
}
