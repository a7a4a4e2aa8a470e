// fp32 GEMM on sm_100a tensor cores: tcgen05.mma kind::tf32 with a 3xTF32
// split, TMEM accumulators, TMA-fed shared-memory ring.
//
//   C[M, N] = alpha * A[M, K] . W[N, K]^T + beta * bias[N]   (+ epilogue)
//
// Both operands are K-major (row-major A; the weight stored as [N, K]).  Each
// operand element x is split into hi = x with the low 13 mantissa bits
// cleared (exactly representable in tf32) and lo = x - hi (exact in fp32),
// and the tile product accumulates hi.hi + hi.lo + lo.hi in fp32 TMEM -- the
// published 3xTF32 scheme, which keeps fp32-level accuracy (the dropped
// lo.lo term is ~2^-22 relative).  The split is done in shared memory right
// after the TMA load, so HBM traffic is that of a plain fp32 GEMM.
//
// CTA = 8 warps, one 128 x BN output tile:
//   warp 0      TMA producer (one lane): A and W tiles of 32 K-columns
//               (128 bytes = one 128B-swizzle row) per stage
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 K-steps of 8 x
//               3 products per stage, tcgen05.commit frees the stage
//   warps 4..7  split the stage into hi/lo (128 threads), then run the
//               epilogue: tcgen05.ld of their 32 TMEM lanes, bias and
//               activation, fp32 stores
// Every mbarrier wait is bounded (~2 s); on expiry the CTA raises an abort
// flag, records LONNX_E_TIMEOUT in the context's device flags, drains and
// frees its TMEM, and returns.
//
// Replaces MathOps.mm_unsafe_vectorized (src/Lokad.Onnx.Tensors/MathOps.cs:380-410).
#include <cuda.h>
#include <stdio.h>

#include <mutex>

#include "lonnx_internal.cuh"
#include "tc_common.cuh"

namespace {

using namespace lonnx::tc;

constexpr int BM = 128;
constexpr int BK = 32;                  // fp32 elements per 128-byte row
constexpr int A_TILE = BM * BK * 4;     // 16 KB
constexpr int kThreads = 256;

template <int BN>
struct Cfg {
    static constexpr int W_TILE = BN * BK * 4;
    static constexpr int STAGE = 2 * A_TILE + 2 * W_TILE;  // A, A_lo, W, W_lo
    static constexpr int STAGES = (BN == 256) ? 2 : 3;
    static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};

__device__ __forceinline__ void split_tf32(float4 v, float4 &hi, float4 &lo) {
    auto h = [](float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
    hi = make_float4(h(v.x), h(v.y), h(v.z), h(v.w));
    lo = make_float4(__fsub_rn(v.x, hi.x), __fsub_rn(v.y, hi.y), __fsub_rn(v.z, hi.z), __fsub_rn(v.w, hi.w));
}

// in place: buf <- hi(buf), lo_buf <- lo(buf); `bytes` multiple of 16*128
__device__ __forceinline__ void split_tile(uint8_t *buf, uint8_t *lo_buf, int bytes, int tid) {
    for (int off = tid * 16; off < bytes; off += 128 * 16) {
        float4 v = *reinterpret_cast<float4 *>(buf + off);
        float4 h, l;
        split_tf32(v, h, l);
        *reinterpret_cast<float4 *>(buf + off) = h;
        *reinterpret_cast<float4 *>(lo_buf + off) = l;
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
              const float *__restrict__ bias, float *__restrict__ C, int M, int N, int K, int ldc,
              float alpha, float beta, int epi, int *dev_flags) {
    using G = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::STAGES * G::STAGE);
    // bars[0..S): full (TMA landed), [S..2S): split done, [2S..3S): empty (MMA done),
    // [3S]: accumulator ready, [3S+1]: drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * G::STAGES + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nk = (K + BK - 1) / BK;

    auto full = [&](int s) { return smem_u32(bars + s); };
    auto conv = [&](int s) { return smem_u32(bars + G::STAGES + s); };
    auto empty = [&](int s) { return smem_u32(bars + 2 * G::STAGES + s); };
    const uint32_t accbar = smem_u32(bars + 3 * G::STAGES);
    const uint32_t drainbar = smem_u32(bars + 3 * G::STAGES + 1);
    int issued = 0;  // TMA stage loads issued (producer lane)
    auto stageA = [&](int s) { return smem + s * G::STAGE; };
    auto stageAlo = [&](int s) { return smem + s * G::STAGE + A_TILE; };
    auto stageW = [&](int s) { return smem + s * G::STAGE + 2 * A_TILE; };
    auto stageWlo = [&](int s) { return smem + s * G::STAGE + 2 * A_TILE + G::W_TILE; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(conv(s), 4);  // one arrive per splitting warp
            mbar_init(empty(s), 1);
        }
        mbar_init(accbar, 1);
        mbar_init(drainbar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % G::STAGES;
                const uint32_t ph = (i / G::STAGES) & 1;
                if (!mbar_wait(empty(s), ph ^ 1, abort_flag)) { ok = false; break; }
                mbar_arrive_expect_tx(full(s), A_TILE + G::W_TILE);
                tma_load_2d(smem_u32(stageA(s)), &tmA, full(s), i * BK, m0);
                tma_load_2d(smem_u32(stageW(s)), &tmW, full(s), i * BK, n0);
                issued = i + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % G::STAGES;
                const uint32_t ph = (i / G::STAGES) & 1;
                if (!mbar_wait(conv(s), ph, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a = smem_u32(stageA(s)), alo = smem_u32(stageAlo(s));
                const uint32_t w = smem_u32(stageW(s)), wlo = smem_u32(stageWlo(s));
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint32_t ko = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
                    const uint64_t da = smem_desc_sw128(a + ko), dal = smem_desc_sw128(alo + ko);
                    const uint64_t dw = smem_desc_sw128(w + ko), dwl = smem_desc_sw128(wlo + ko);
                    mma_tf32(tmem, dal, dw, idesc, (i | kk) != 0);
                    mma_tf32(tmem, da, dwl, idesc, 1);
                    mma_tf32(tmem, da, dw, idesc, 1);
                }
                mma_commit(empty(s));
            }
            if (ok) mma_commit(accbar);
        }
    } else if (warp >= 4) {
        const int tid = threadIdx.x - 128;
        for (int i = 0; i < nk && ok; ++i) {
            const int s = i % G::STAGES;
            const uint32_t ph = (i / G::STAGES) & 1;
            if (!mbar_wait(full(s), ph, abort_flag)) { ok = false; break; }
            split_tile(stageA(s), stageAlo(s), A_TILE, tid);
            split_tile(stageW(s), stageWlo(s), G::W_TILE, tid);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(conv(s));
        }
        // epilogue: warp (w % 4) owns TMEM lanes 32*(w%4) .. +31 = tile rows
        if (ok && mbar_wait(accbar, 0, abort_flag)) {
            tc_fence_after();
            const int q = warp & 3;
            const int row = m0 + q * 32 + lane;
            float *crow = C + (int64_t)row * ldc;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c0, r);
                tmem_ld_wait();
                if (row < M) {
                    const int nb = n0 + c0;
                    float out[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float v = __uint_as_float(r[j]);
                        if (alpha != 1.0f) v = __fmul_rn(v, alpha);
                        const int col = nb + j;
                        if (bias && col < N) v = __fadd_rn(v, beta == 1.0f ? bias[col] : __fmul_rn(beta, bias[col]));
                        if (epi == LONNX_EPI_RELU) v = v > 0.0f ? v : 0.0f;
                        else if (epi == LONNX_EPI_GELU_ERF) v = lonnx_gelu_chain(v);
                        out[j] = v;
                    }
                    if (nb + 32 <= N && (ldc & 3) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(crow + nb + j) = make_float4(out[j], out[j + 1], out[j + 2], out[j + 3]);
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < N) crow[nb + j] = out[j];
                    }
                }
            }
        } else {
            ok = false;
        }
    }

    if (!ok) {
        *abort_flag = 1;
        atomicExch(dev_flags + lonnx::FLAG_TIMEOUT, 1);
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        // drain before releasing TMEM / exiting: MMAs already issued, and TMA
        // loads that may still land in this CTA's shared memory (bounded waits)
        if (warp == 1 && lane == 0) {
            mma_commit(drainbar);
            mbar_wait(drainbar, 0, nullptr, 200000000ull);
        }
        if (warp == 0 && lane == 0) {
            for (int j = issued - G::STAGES < 0 ? 0 : issued - G::STAGES; j < issued; ++j)
                mbar_wait(full(j % G::STAGES), (j / G::STAGES) & 1, nullptr, 200000000ull);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

// ---- host side ----------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        cudaGetLastError();
    });
    return fn;
}

// row-major [rows, cols] fp32 with leading dimension ld; box = box_rows x 32
int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return lonnx::set_error(LONNX_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return lonnx::set_error(LONNX_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LONNX_OK;
}

template <int BN>
int launch_tc(lonnx_ctx *ctx, const CUtensorMap &ma, const CUtensorMap &mw, const float *bias,
              float *C, int M, int N, int K, int ldc, float alpha, float beta, int epi) {
    using G = Cfg<BN>;
    static bool attr_set[64] = {false};
    if (!attr_set[ctx->device & 63]) {
        LONNX_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_set[ctx->device & 63] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    k_gemm_tf32x3<BN><<<grid, kThreads, G::SMEM, ctx->stream>>>(ma, mw, bias, C, M, N, K, ldc, alpha, beta, epi,
                                                                ctx->dev_flags);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // namespace

namespace lonnx {

int gemm_tc(lonnx_ctx *ctx, const float *A, const float *W, const float *bias,
            const float *residual, float *C, int M, int N, int K, int lda, int ldw, int ldc,
            float alpha, float beta, int epi) {
    if (residual) return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: residual epilogue not supported");
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (M <= 0 || N <= 0 || K <= 0 || (lda & 3) || (ldw & 3) || !al16(A) || !al16(W))
        return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: operands not 16-byte aligned");
    CUtensorMap ma, mw;
    int rc = make_map(&ma, A, M, K, lda, BM);
    if (rc) return rc;
    // Tile width: 128 columns unless N is large and a multiple of 256.
    if (N >= 1024 && N % 256 == 0 && (int64_t)M * N >= (int64_t)148 * BM * 256) {
        rc = make_map(&mw, W, N, K, ldw, 256);
        if (rc) return rc;
        return launch_tc<256>(ctx, ma, mw, bias, C, M, N, K, ldc, alpha, beta, epi);
    }
    rc = make_map(&mw, W, N, K, ldw, 128);
    if (rc) return rc;
    return launch_tc<128>(ctx, ma, mw, bias, C, M, N, K, ldc, alpha, beta, epi);
}

}  // namespace lonnx
