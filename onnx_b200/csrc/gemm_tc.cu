// fp32 GEMM on sm_100a tensor cores: tcgen05.mma kind::tf32 with a 3xTF32
// split, TMEM accumulators, TMA-fed shared-memory ring.
//
//   C[M, N] = alpha * A[M, K] . W[N, K]^T + beta * bias[N]   (+ epilogue)
//
// Both operands are K-major (row-major A; the weight stored as [N, K]).  Each
// operand element x is split into hi = x with the low 13 mantissa bits
// cleared (exactly representable in tf32) and lo = x - hi (exact in fp32);
// the tile product accumulates hi.hi + hi.lo + lo.hi -- the published 3xTF32
// scheme, which keeps fp32-level accuracy (the dropped lo.lo term is ~2^-22
// relative).  The weight is split once, ahead of time (split_tf32_nk); the
// activation tile is split in shared memory right after its TMA load, so HBM
// traffic for A is that of a plain fp32 GEMM.
//
// CTA = 12 warps, one 128 x BN output tile (BN = 128 or 192):
//   warp 0      TMA producer (one lane): A, W_hi, W_lo tiles of 32 K-columns
//               (128 bytes = one 128B-swizzle row) per stage, 3-4 stages
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 K-steps x 3
//               products per stage into one of two TMEM chunk accumulators
//   warps 2-3   write A_lo of each stage into a 2-buffer ring
//   warps 4-11  drain each chunk accumulator into fp32 registers (round to
//               nearest), then run the epilogue: bias, activation, stores
// Every mbarrier wait is bounded (~2 s); on expiry the CTA raises an abort
// flag, records LONNX_E_TIMEOUT in the context's device flags, drains its
// in-flight copies and MMAs, frees its TMEM, and returns.
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
constexpr int kThreads = 384;           // 12 warps
// warp roles: 0 TMA, 1 MMA + TMEM owner, 2-3 split A, 4-11 accumulate/epilogue
constexpr int W_TMA = 0, W_MMA = 1, W_SPLIT0 = 2, N_SPLIT = 2, W_ACC0 = 4, N_ACC = 8;

template <int BN, bool ALO>
struct Cfg {
    static constexpr int W_TILE = BN * BK * 4;
    // TMA ring: A, W_hi, W_lo (+ A_lo when it comes from HBM)
    static constexpr int STAGE = (ALO ? 2 : 1) * A_TILE + 2 * W_TILE;
    static constexpr int LO = ALO ? 0 : 2 * A_TILE;    // in-kernel A_lo ring: 2 buffers
    static constexpr int STAGES = (4 * STAGE + LO + 1280 <= 227 * 1024) ? 4
                                  : (3 * STAGE + LO + 1280 <= 227 * 1024) ? 3 : 2;
    static constexpr int SMEM = STAGES * STAGE + LO + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;  // two chunk accumulators
    static constexpr int COLS_PER_ACC = BN / 2;                  // per accumulator thread
};

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// lo_buf <- x - tf32(x).  The tensor core reads an fp32 operand as its tf32
// truncation (tests/test_gemm_gpu.py::test_tf32_operand_truncation), so the
// raw tile already serves as the high part.
__device__ __forceinline__ void split_lo(const uint8_t *buf, uint8_t *lo_buf, int bytes, int tid, int nthreads) {
#pragma unroll 4
    for (int off = tid * 16; off < bytes; off += nthreads * 16) {
        const float4 v = *reinterpret_cast<const float4 *>(buf + off);
        float4 l;
        l.x = __fsub_rn(v.x, tf32_hi(v.x));
        l.y = __fsub_rn(v.y, tf32_hi(v.y));
        l.z = __fsub_rn(v.z, tf32_hi(v.z));
        l.w = __fsub_rn(v.w, tf32_hi(v.w));
        *reinterpret_cast<float4 *>(lo_buf + off) = l;
    }
}

// Accumulation: each K stage is accumulated by the tensor core into a fresh
// TMEM buffer (two buffers, ping-pong) and the stage sums are added into fp32
// registers with round-to-nearest by the accumulator warps.  The tensor
// core's accumulator rounds toward zero, so one TMEM accumulator over all of
// K builds an error that grows linearly with K (measured ~10x the
// sequential fp32 sum at K = 1536); 32-wide chunks keep it at fp32 level.
//
// Shared-memory bandwidth is the binding resource of a 3xTF32 tile (operand
// reads of three MMAs + TMA writes + the split), which is why the weight is
// split once ahead of time and A_lo has its own 2-buffer ring (so the TMA
// ring can be 3-4 stages deep).
template <int BN, bool ALO>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmAlo,
              const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmWlo,
              const float *__restrict__ bias, float *__restrict__ C, int M, int N, int K, int ldc, float alpha,
              float beta, int epi, int *dev_flags) {
    using G = Cfg<BN, ALO>;
    constexpr int S = G::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * G::STAGE + G::LO);
    // [0,S) full  [S,2S) split done  [2S,3S) stage free  [3S,3S+2) chunk ready
    // [3S+2,3S+4) chunk drained  [3S+4] abort drain  [3S+5,3S+7) A_lo buffer free
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 7);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nk = (K + BK - 1) / BK;

    auto full = [&](int s) { return smem_u32(bars + s); };
    auto conv = [&](int s) { return smem_u32(bars + S + s); };
    auto empty = [&](int s) { return smem_u32(bars + 2 * S + s); };
    auto tfull = [&](int b) { return smem_u32(bars + 3 * S + b); };
    auto tdrain = [&](int b) { return smem_u32(bars + 3 * S + 2 + b); };
    const uint32_t drainbar = smem_u32(bars + 3 * S + 4);
    auto lofree = [&](int b) { return smem_u32(bars + 3 * S + 5 + b); };
    auto stageA = [&](int s) { return smem + s * G::STAGE; };
    auto stageW = [&](int s) { return smem + s * G::STAGE + A_TILE; };
    auto stageWlo = [&](int s) { return smem + s * G::STAGE + A_TILE + G::W_TILE; };
    auto stageAlo = [&](int s) { return smem + s * G::STAGE + A_TILE + 2 * G::W_TILE; };
    auto bufAlo = [&](int b) { return smem + S * G::STAGE + b * A_TILE; };
    int issued = 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(conv(s), ALO ? 1 : N_SPLIT + N_ACC);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull(b), 1);
            mbar_init(tdrain(b), N_ACC);
            mbar_init(lofree(b), 1);
        }
        mbar_init(drainbar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmWlo);
        if (ALO) prefetch_tmap(&tmAlo);
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_u32(tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == W_TMA) {
        if (lane == 0) {
            constexpr uint32_t bytes = G::STAGE;
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % S;
                if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, abort_flag)) { ok = false; break; }
                mbar_arrive_expect_tx(full(s), bytes);
                tma_load_2d(smem_u32(stageA(s)), &tmA, full(s), i * BK, m0);
                tma_load_2d(smem_u32(stageW(s)), &tmW, full(s), i * BK, n0);
                tma_load_2d(smem_u32(stageWlo(s)), &tmWlo, full(s), i * BK, n0);
                if (ALO) tma_load_2d(smem_u32(stageAlo(s)), &tmAlo, full(s), i * BK, m0);
                issued = i + 1;
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % S, b = i & 1;
                if (!mbar_wait(ALO ? full(s) : conv(s), (i / S) & 1, abort_flag)) { ok = false; break; }
                if (!mbar_wait(tdrain(b), ((i >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + b * BN;
                const uint32_t a = smem_u32(stageA(s)), alo = smem_u32(ALO ? stageAlo(s) : bufAlo(b));
                const uint32_t w = smem_u32(stageW(s)), wlo = smem_u32(stageWlo(s));
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint32_t ko = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
                    const uint64_t da = smem_desc_sw128(a + ko), dal = smem_desc_sw128(alo + ko);
                    const uint64_t dw = smem_desc_sw128(w + ko), dwl = smem_desc_sw128(wlo + ko);
                    mma_tf32(acc, dal, dw, idesc, kk != 0);
                    mma_tf32(acc, da, dwl, idesc, 1);
                    mma_tf32(acc, da, dw, idesc, 1);
                }
                mma_commit(empty(s));
                mma_commit(lofree(b));
                mma_commit(tfull(b));
            }
        }
    } else if (warp < W_ACC0) {
        if (ALO) goto done_roles;
        const int tid = threadIdx.x - W_SPLIT0 * 32;
        for (int i = 0; i < nk && ok; ++i) {
            const int s = i % S, b = i & 1;
            if (!mbar_wait(full(s), (i / S) & 1, abort_flag)) { ok = false; break; }
            if (!mbar_wait(lofree(b), ((i >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
            split_lo(stageA(s), bufAlo(b), A_TILE, tid, (N_SPLIT + N_ACC) * 32);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(conv(s));
        }
    } else {
        // accumulator / epilogue warps: warp w owns TMEM lanes 32*(w%4)..+31
        // (tile rows) and one half of the tile's columns
        constexpr int CPA = G::COLS_PER_ACC;
        const int q = warp & 3, half = (warp - W_ACC0) >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + half * CPA;
        float acc[CPA];
#pragma unroll
        for (int j = 0; j < CPA; ++j) acc[j] = 0.0f;
        // per iteration: help split stage i (unless A_lo comes from HBM), then
        // drain chunk i-1 -- the drain of a chunk never waits on a split the
        // same warps still have to do
        const int stid = N_SPLIT * 32 + (threadIdx.x - W_ACC0 * 32);
        auto drain = [&](int i) {
            const int b = i & 1;
            if (!mbar_wait(tfull(b), (i >> 1) & 1, abort_flag)) return false;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < CPA / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(lane_base + b * BN + c * 32, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[c * 32 + j] = __fadd_rn(acc[c * 32 + j], __uint_as_float(r[j]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tdrain(b));
            return true;
        };
        for (int i = 0; i <= nk && ok; ++i) {
            if (!ALO && i < nk) {
                const int s = i % S, b = i & 1;
                if (!mbar_wait(full(s), (i / S) & 1, abort_flag) ||
                    !mbar_wait(lofree(b), ((i >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                split_lo(stageA(s), bufAlo(b), A_TILE, stid, (N_SPLIT + N_ACC) * 32);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(conv(s));
            }
            if (i > 0 && !drain(i - 1)) { ok = false; break; }
        }
        // epilogue: raw sums staged row-major in the (now idle) stage buffers,
        // then one pass that applies alpha, bias and the activation and writes
        // coalesced 16-byte stores.  The activation code appears once (a
        // per-element unrolled epilogue with Erf-GELU inlined overflows the
        // instruction cache).
        constexpr int PITCH = BN + 4;  // floats; keeps the per-row writes conflict-free
        static_assert(BM * PITCH * 4 <= G::STAGES * G::STAGE, "C tile must fit in the stage ring");
        float *ctile = reinterpret_cast<float *>(smem);
        float *sbias = ctile + BM * PITCH;  // BN floats
        static_assert(BM * PITCH * 4 + BN * 4 <= G::STAGES * G::STAGE, "C tile + bias must fit in the stage ring");
        const int rloc = q * 32 + lane;
        {
            const int t = threadIdx.x - W_ACC0 * 32;
            for (int c = t; c < BN; c += N_ACC * 32) {
                const int col = n0 + c;
                float bv = 0.0f;
                if (bias && col < N) bv = beta == 1.0f ? __ldg(bias + col) : __fmul_rn(beta, __ldg(bias + col));
                sbias[c] = bv;
            }
        }
        if (ok) {
#pragma unroll
            for (int j = 0; j < CPA; j += 4)
                *reinterpret_cast<float4 *>(ctile + rloc * PITCH + half * CPA + j) =
                    make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(N_ACC * 32) : "memory");
        if (ok) {
            const int t = threadIdx.x - W_ACC0 * 32;
            constexpr int V4 = BN / 4;  // float4 per tile row
            const bool vec = (ldc & 3) == 0 && n0 + BN <= N;
#pragma unroll 1
            for (int e = t; e < BM * V4; e += N_ACC * 32) {
                const int r = e / V4, c4 = e % V4;
                const int grow = m0 + r;
                if (grow >= M) continue;
                const float4 raw = *reinterpret_cast<const float4 *>(ctile + r * PITCH + c4 * 4);
                float v[4] = {raw.x, raw.y, raw.z, raw.w};
                const int col0 = n0 + c4 * 4;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float x = v[u];
                    if (alpha != 1.0f) x = __fmul_rn(x, alpha);
                    if (bias) x = __fadd_rn(x, sbias[c4 * 4 + u]);
                    if (epi == LONNX_EPI_RELU) x = x > 0.0f ? x : 0.0f;
                    else if (epi == LONNX_EPI_GELU_ERF) x = lonnx_gelu_chain(x);
                    v[u] = x;
                }
                float *dst = C + (int64_t)grow * ldc + col0;
                if (vec) {
                    *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
                    for (int u = 0; u < 4; ++u)
                        if (col0 + u < N) dst[u] = v[u];
                }
            }
        }
    }

done_roles:
    if (!ok) {
        *abort_flag = 1;
        atomicExch(dev_flags + lonnx::FLAG_TIMEOUT, 1);
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        // drain before releasing TMEM / exiting: MMAs already issued, and TMA
        // loads that may still land in this CTA's shared memory (bounded waits)
        if (warp == W_MMA && lane == 0) {
            mma_commit(drainbar);
            mbar_wait(drainbar, 0, nullptr, 400000000ll);
        }
        if (warp == W_TMA && lane == 0) {
            for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
                mbar_wait(full(j % S), (j / S) & 1, nullptr, 400000000ll);
        }
        __syncthreads();
    }
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

// Activation low parts: lo = a - tf32(a), row-major like a (fp32 streaming).
__global__ void k_split_lo(const float4 *__restrict__ a, float4 *__restrict__ lo, int64_t n4) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = __ldg(a + i);
        lo[i] = make_float4(__fsub_rn(v.x, tf32_hi(v.x)), __fsub_rn(v.y, tf32_hi(v.y)), __fsub_rn(v.z, tf32_hi(v.z)),
                            __fsub_rn(v.w, tf32_hi(v.w)));
    }
}

// Weight preparation: W given as [K, N] (trans = 0) or [N, K] (trans = 1)
// -> hi, lo as [N, K] with hi = tf32(w) (low 13 mantissa bits cleared) and
// lo = w - hi (exact).  Run once per weight; O(N K).
__global__ void k_split_tf32_nk(const float *__restrict__ w, float *__restrict__ hi, float *__restrict__ lo,
                                int K, int N, int trans) {
    const int64_t n_el = (int64_t)N * K;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_el; i += stride) {
        const int64_t nn = i / K, kk = i % K;
        const float v = trans ? w[i] : w[kk * N + nn];
        const float h = tf32_hi(v);
        hi[i] = h;
        lo[i] = __fsub_rn(v, h);
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

template <int BN, bool ALO>
int launch_tc(lonnx_ctx *ctx, const CUtensorMap &ma, const CUtensorMap &malo, const CUtensorMap &mw,
              const CUtensorMap &mwlo, const float *bias, float *C, int M, int N, int K, int ldc, float alpha,
              float beta, int epi) {
    using G = Cfg<BN, ALO>;
    static bool attr_set[64] = {false};
    if (!attr_set[ctx->device & 63]) {
        LONNX_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<BN, ALO>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_set[ctx->device & 63] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    k_gemm_tf32x3<BN, ALO><<<grid, kThreads, G::SMEM, ctx->stream>>>(ma, malo, mw, mwlo, bias, C, M, N, K, ldc, alpha,
                                                                     beta, epi, ctx->dev_flags);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

// Tile width for N: 192 or 128, whichever divides N, else the one with the
// least padding.
int pick_bn(int N) {
    if (N % 192 == 0) return 192;
    if (N % 128 == 0) return 128;
    return ((N + 191) / 192 * 192 - N) < ((N + 127) / 128 * 128 - N) ? 192 : 128;
}

}  // namespace

namespace lonnx {

int gemm_tc(lonnx_ctx *ctx, const float *A, const float *Whi, const float *Wlo, const float *bias, float *C, int M,
            int N, int K, int lda, int ldw, int ldc, float alpha, float beta, int epi, bool allow_scratch) {
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (!Wlo) return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: weight must be pre-split");
    if (M <= 0 || N <= 0 || K <= 0 || (lda & 3) || (ldw & 3) || !al16(A) || !al16(Whi) || !al16(Wlo))
        return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: operands not 16-byte aligned");
    const int bn = pick_bn(N);
    CUtensorMap ma, mw, mwlo;
    int rc = make_map(&ma, A, M, K, lda, BM);
    if (rc) return rc;
    rc = make_map(&mw, Whi, N, K, ldw, bn);
    if (rc) return rc;
    rc = make_map(&mwlo, Wlo, N, K, ldw, bn);
    if (rc) return rc;
    // A's low parts: split inside the kernel per tile (default; measured
    // faster on every BASELINE shape), or streamed once into scratch and
    // TMA-loaded beside A (LONNX_GEMM_ALO=1).
    static const int mode = [] {
        const char *e = getenv("LONNX_GEMM_ALO");
        return e ? atoi(e) : -1;
    }();
    const bool alo = mode > 0;
    if (alo && allow_scratch) {
        // A_lo streamed into scratch, then TMA-loaded beside A
        void *tmp = nullptr;
        rc = ctx_scratch2(ctx, (size_t)M * lda * 4, &tmp);
        if (rc) return rc;
        const int64_t n4 = (int64_t)M * lda / 4;
        int64_t blocks = (n4 + 255) / 256;
        if (blocks > (int64_t)ctx->num_sms * 16) blocks = (int64_t)ctx->num_sms * 16;
        k_split_lo<<<(int)blocks, 256, 0, ctx->stream>>>((const float4 *)A, (float4 *)tmp, n4);
        LONNX_CHECK_LAUNCH(ctx);
        CUtensorMap malo;
        rc = make_map(&malo, (const float *)tmp, M, K, lda, BM);
        if (rc) return rc;
        if (bn == 192) return launch_tc<192, true>(ctx, ma, malo, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi);
        return launch_tc<128, true>(ctx, ma, malo, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi);
    }
    if (bn == 192) return launch_tc<192, false>(ctx, ma, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi);
    return launch_tc<128, false>(ctx, ma, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi);
}

int split_tf32_nk(lonnx_ctx *ctx, const float *w, float *hi, float *lo, int K, int N, int trans) {
    const int64_t n = (int64_t)N * K;
    if (n <= 0) return LONNX_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)ctx->num_sms * 16) blocks = (int64_t)ctx->num_sms * 16;
    k_split_tf32_nk<<<(int)blocks, 256, 0, ctx->stream>>>(w, hi, lo, K, N, trans);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // namespace lonnx
