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
// activation tile is split on chip right after its TMA load, so HBM traffic
// for A is that of a plain fp32 GEMM.
//
// CTA = 20 warps, one 128 x BN output tile (BN = 128 or 192):
//   warp 0      TMA producer (one lane): A, W_hi, W_lo tiles of 32 K-columns
//               (128 bytes = one 128B-swizzle row) per stage, 3-4 stages
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 K-steps x 3
//               products per stage, A from TMEM, W from shared memory, into
//               one of two TMEM chunk accumulators
//   warps 4-7   move each stage's A rows into TMEM as tf32 hi and lo parts
//   warps 8-19  drain each chunk accumulator into fp32 registers (round to
//               nearest), 64 columns per warp, then run the epilogue
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
constexpr int kThreads = 640;           // 20 warps
// warp roles: 0 TMA, 1 MMA + TMEM owner, 4-7 A -> TMEM, 8-19 accumulate/epilogue
constexpr int W_TMA = 0, W_MMA = 1, W_A0 = 4, W_ACC0 = 8;

template <int BN>
struct Cfg {
    static constexpr int W_TILE = BN * BK * 4;
    static constexpr int STAGE = A_TILE + 2 * W_TILE;  // TMA ring: A, W_hi, W_lo
    static constexpr int STAGES = (4 * STAGE + 1280 <= 227 * 1024) ? 4 : 3;
    static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int GROUPS = BN / 64;              // accumulator column groups of 64
    static constexpr int ACC_COL = 0;                   // TMEM: 2 chunk accumulators [0, 2 BN)
    static constexpr int A_COL = 2 * BN;                // then NAB A buffers of 64 (hi 32 | lo 32)
    static constexpr int NAB = 2 * BN + 3 * 64 <= 512 ? 3 : 2;
    static constexpr int TMEM_COLS = 2 * BN + NAB * 64 <= 256 ? 256 : 512;
};

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// C[M,N] = alpha * A . W^T + beta * bias, epilogue.
//   A [M,K] fp32 (tmA); W_hi, W_lo [N,K] (tmW, tmWlo): the weight pre-split
//   into its tf32 part and the exact fp32 remainder.
// Per 32-wide K stage: 4 K-steps x {A_lo.W_hi, A_hi.W_lo, A_hi.W_hi}, with
// A_hi and A_lo in TMEM (written by the A warps) and W_hi / W_lo in shared
// memory (TMA).
//
// Why A lives in TMEM: shared-memory bandwidth binds a 3xTF32 tile.  With
// both operands in shared memory one 32-wide stage moved ~216 KB through it
// (TMA writes, the split, three MMAs re-reading A and W); with A in TMEM it
// is ~152 KB, about the MMA time of the stage.
//
// Accumulation: each K stage is accumulated by the tensor core into a fresh
// TMEM buffer (two buffers, ping-pong) and the stage sums are added into fp32
// registers with round-to-nearest by the accumulator warps.  The tensor
// core's accumulator rounds toward zero, so one TMEM accumulator over all of
// K builds an error that grows linearly with K (measured ~10x the
// sequential fp32 sum at K = 1536); 32-wide chunks keep it at fp32 level.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
              const __grid_constant__ CUtensorMap tmWlo, const float *__restrict__ bias, float *__restrict__ C,
              int M, int N, int K, int ldc, float alpha, float beta, int epi, int *dev_flags,
              const lonnx::ConvArgs cv) {
    using G = Cfg<BN>;
    constexpr int S = G::STAGES;
    constexpr int NACC = 4 * G::GROUPS;  // accumulator warps in use
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * G::STAGE);
    // [0,S) full  [S,2S) A in TMEM  [2S,3S) stage free  [3S,3S+2) chunk ready
    // [3S+2,3S+4) chunk drained  [3S+4] abort drain  [3S+5,3S+5+NAB) TMEM A buffer free
    constexpr int NAB = G::NAB;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 5 + NAB);
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
    auto afree = [&](int b) { return smem_u32(bars + 3 * S + 5 + b); };
    auto stageA = [&](int s) { return smem + s * G::STAGE; };
    auto stageW = [&](int s) { return smem + s * G::STAGE + A_TILE; };
    auto stageWlo = [&](int s) { return smem + s * G::STAGE + A_TILE + G::W_TILE; };
    int issued = 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(conv(s), 4);  // one arrive per A warp
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull(b), 1);
            mbar_init(tdrain(b), NACC);
        }
        for (int b = 0; b < NAB; ++b) mbar_init(afree(b), 1);
        mbar_init(drainbar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmWlo);
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
            const uint32_t bytes = cv.x ? 2 * G::W_TILE : G::STAGE;
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % S;
                if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, abort_flag)) { ok = false; break; }
                mbar_arrive_expect_tx(full(s), bytes);
                if (!cv.x) tma_load_2d(smem_u32(stageA(s)), &tmA, full(s), i * BK, m0);
                tma_load_2d(smem_u32(stageW(s)), &tmW, full(s), i * BK, n0);
                tma_load_2d(smem_u32(stageWlo(s)), &tmWlo, full(s), i * BK, n0);
                issued = i + 1;
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % S, b = i & 1;
                if (!mbar_wait(conv(s), (i / S) & 1, abort_flag)) { ok = false; break; }
                // implicit conv: the A warps do not wait for the W tiles, so the MMA does
                if (cv.x && !mbar_wait(full(s), (i / S) & 1, abort_flag)) { ok = false; break; }
                if (!mbar_wait(tdrain(b), ((i >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + G::ACC_COL + b * BN;
                const int ab = i % NAB;
                const uint32_t ahi = tmem + G::A_COL + ab * 64, alo = ahi + 32;
                const uint32_t w = smem_u32(stageW(s)), wlo = smem_u32(stageWlo(s));
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint64_t dw = smem_desc_sw128(w + kk * 32), dwl = smem_desc_sw128(wlo + kk * 32);
                    mma_tf32_ts(acc, alo + kk * 8, dw, idesc, kk != 0);
                    mma_tf32_ts(acc, ahi + kk * 8, dwl, idesc, 1);
                    mma_tf32_ts(acc, ahi + kk * 8, dw, idesc, 1);
                }
                mma_commit(empty(s));
                mma_commit(afree(ab));
                mma_commit(tfull(b));
            }
        }
    } else if (warp >= W_A0 && warp < W_A0 + 4) {
        // A warps: warp (w % 4) owns TMEM lanes = tile rows 32*(w%4)..+31;
        // each thread moves its row of the stage's A tile into TMEM as
        // hi = tf32(a) and lo = a - hi
        const int q = warp & 3, r = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::A_COL;
        if (cv.x) {
            // implicit-GEMM conv: row r is output pixel m0 + r, column k is
            // (c, ky, kx).  Each thread gathers its pixel's 32 taps of a
            // stage straight from the NCHW input with 4-byte cp.async into
            // its own row of the stage's (otherwise unused) A slot, S - 1
            // stages ahead; lanes are consecutive pixels, so each tap is one
            // coalesced warp access; taps outside the image or past K are
            // zero-filled.  Rows are rotated by r words so the 32 lanes hit
            // 32 banks.
            constexpr int D = S - 1;
            int iy0 = -(1 << 20), ix0 = 0;
            const float *xr = cv.x;
            const int p = m0 + r;
            if (p < M) {
                const int hw = cv.Ho * cv.Wo, n = p / hw, rem = p - n * hw;
                const int oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
                iy0 = oy * cv.sh - cv.pt;
                ix0 = ox * cv.sw - cv.pl;
                xr = cv.x + (int64_t)n * cv.C * cv.H * cv.W + (int64_t)iy0 * cv.W + ix0;
            }
            const int khw = cv.kh * cv.kw, HW = cv.H * cv.W;
            auto gather = [&](int i) {
                const uint32_t row = smem_u32(stageA(i % S)) + r * 128;
                const int k = i * BK + lane;
                int off = 0, dy = -(1 << 20), dx = 0;  // taps past K read as zero
                if (k < K) {
                    const int c = k / khw, rr = k - c * khw, ky = rr / cv.kw, kx = rr - ky * cv.kw;
                    dy = ky * cv.dh;
                    dx = kx * cv.dw;
                    off = c * HW + dy * cv.W + dx;
                }
#pragma unroll 4
                for (int u = 0; u < BK; ++u) {
                    const int o = __shfl_sync(0xffffffffu, off, u);
                    const int yy = iy0 + __shfl_sync(0xffffffffu, dy, u);
                    const int xx = ix0 + __shfl_sync(0xffffffffu, dx, u);
                    const bool in = (unsigned)yy < (unsigned)cv.H && (unsigned)xx < (unsigned)cv.W;
                    cp_async4(row + (((u + r) & 31) << 2), in ? xr + o : cv.x, in ? 4u : 0u);
                }
            };
            for (int j = 0; j < D; ++j) {
                if (j < nk) gather(j);
                cp_async_commit();
            }
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % S, b = i % NAB;
                if (i + D < nk) gather(i + D);
                cp_async_commit();
                cp_async_wait<D>();  // this thread's taps of stage i have landed
                const float *row = reinterpret_cast<const float *>(stageA(s) + r * 128);
                if (!mbar_wait(afree(b), ((i / NAB) & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float x = row[(hf * 16 + j + r) & 31], h = tf32_hi(x);
                        hi[j] = __float_as_uint(h);
                        lo[j] = __float_as_uint(__fsub_rn(x, h));
                    }
                    tmem_st_32x32b_x16(lane_base + b * 64 + hf * 16, hi);
                    tmem_st_32x32b_x16(lane_base + b * 64 + 32 + hf * 16, lo);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(conv(s));
            }
            cp_async_wait<0>();
        }
        for (int i = 0; i < nk && ok && !cv.x; ++i) {
            const int s = i % S, b = i % NAB;
            if (!mbar_wait(full(s), (i / S) & 1, abort_flag)) { ok = false; break; }
            if (!mbar_wait(afree(b), ((i / NAB) & 1) ^ 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint8_t *row = stageA(s) + r * 128;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    const int c = hf * 4 + c4;
                    const float4 v = *reinterpret_cast<const float4 *>(row + (((c ^ (r & 7))) << 4));
                    const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float h = tf32_hi(x[u]);
                        hi[c4 * 4 + u] = __float_as_uint(h);
                        lo[c4 * 4 + u] = __float_as_uint(__fsub_rn(x[u], h));
                    }
                }
                tmem_st_32x32b_x16(lane_base + b * 64 + hf * 16, hi);
                tmem_st_32x32b_x16(lane_base + b * 64 + 32 + hf * 16, lo);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(conv(s));
        }
    } else if (warp >= W_ACC0 && warp < W_ACC0 + NACC) {
        // accumulator / epilogue warps: warp w owns TMEM lanes 32*(w%4)..+31
        // (tile rows) and one 64-column group of the tile
        const int q = warp & 3, grp = (warp - W_ACC0) >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::ACC_COL + grp * 64;
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
        for (int i = 0; i < nk && ok; ++i) {
            const int b = i & 1;
            if (!mbar_wait(tfull(b), (i >> 1) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t rr[16];
                tmem_ld_32x32b_x16(lane_base + b * BN + c * 16, rr);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[c * 16 + j] = __fadd_rn(acc[c * 16 + j], __uint_as_float(rr[j]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tdrain(b));
        }
        // epilogue: raw sums staged row-major in the (now idle) stage buffers,
        // then one pass that applies alpha, bias and the activation and writes
        // coalesced 16-byte stores.  The activation code appears once (a
        // per-element unrolled epilogue with Erf-GELU inlined overflows the
        // instruction cache).
        constexpr int PITCH = BN + 4;  // floats; keeps the per-row writes conflict-free
        static_assert(BM * PITCH * 4 + BN * 4 <= G::STAGES * G::STAGE, "C tile + bias must fit in the stage ring");
        float *ctile = reinterpret_cast<float *>(smem);
        float *sbias = ctile + BM * PITCH;
        const int t = threadIdx.x - W_ACC0 * 32;
        for (int c = t; c < BN; c += NACC * 32) {
            const int col = n0 + c;
            float bv = 0.0f;
            if (bias && col < N) bv = beta == 1.0f ? __ldg(bias + col) : __fmul_rn(beta, __ldg(bias + col));
            sbias[c] = bv;
        }
        const int rloc = q * 32 + lane;
        if (cv.img_rows > 0) {
            // NCHW output: row = (image, pixel), column = channel; a warp's
            // lanes hold consecutive pixels, so each column store coalesces.
            // Optional residual (same layout) added after the bias, before
            // the activation, as a following Add node would.
            asm volatile("bar.sync 1, %0;" ::"n"(NACC * 32) : "memory");
            const int grow = m0 + rloc;
            if (ok && grow < M) {
                const int img = grow / cv.img_rows, pix = grow - img * cv.img_rows;
                const int64_t o = (int64_t)img * N * cv.img_rows + pix;
                float *dst = C + o;
                const float *rs = cv.res ? cv.res + o : nullptr;
                const int cs = cv.img_rows;  // N * img_rows (one image's output) < 2^31
#pragma unroll
                for (int j0 = 0; j0 < 64; j0 += 8) {
                    // residual loads for 8 columns first (all in flight at once)
                    float rv[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int col = min(n0 + grp * 64 + j0 + j, N - 1);
                        rv[j] = rs ? __ldg(rs + col * cs) : 0.0f;
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int cl = grp * 64 + j0 + j, col = n0 + cl;
                        if (col < N) {
                            float x = acc[j0 + j];
                            if (alpha != 1.0f) x = __fmul_rn(x, alpha);
                            if (bias) x = __fadd_rn(x, sbias[cl]);
                            if (rs) x = __fadd_rn(x, rv[j]);
                            if (epi == LONNX_EPI_RELU) x = x > 0.0f ? x : 0.0f;
                            dst[col * cs] = x;
                        }
                    }
                }
            }
        } else {
        if (ok) {
#pragma unroll
            for (int j = 0; j < 64; j += 4)
                *reinterpret_cast<float4 *>(ctile + rloc * PITCH + grp * 64 + j) =
                    make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NACC * 32) : "memory");
        if (ok) {
            constexpr int V4 = BN / 4;  // float4 per tile row
            const bool vec = (ldc & 3) == 0 && n0 + BN <= N;
#pragma unroll 1
            for (int e = t; e < BM * V4; e += NACC * 32) {
                const int rr = e / V4, c4 = e % V4;
                const int grow = m0 + rr;
                if (grow >= M) continue;
                const float4 raw = *reinterpret_cast<const float4 *>(ctile + rr * PITCH + c4 * 4);
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

template <int BN>
int launch_tc(lonnx_ctx *ctx, const CUtensorMap &ma, const CUtensorMap &mw, const CUtensorMap &mwlo,
              const float *bias, float *C, int M, int N, int K, int ldc, float alpha, float beta, int epi,
              const lonnx::ConvArgs &cv) {
    using G = Cfg<BN>;
    static bool attr_set[64] = {false};
    if (!attr_set[ctx->device & 63]) {
        LONNX_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_set[ctx->device & 63] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    k_gemm_tf32x3<BN><<<grid, kThreads, G::SMEM, ctx->stream>>>(ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi,
                                                                ctx->dev_flags, cv);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

// Tile width for N: 192 or 128, whichever divides N, else the one with the
// least padding.
int pick_bn(int N) {
    static const int forced = [] {
        const char *e = getenv("LONNX_GEMM_BN");
        return e ? atoi(e) : 0;
    }();
    if (forced == 128 || forced == 192) return forced;
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
    (void)allow_scratch;  // this path allocates nothing
    const ConvArgs none{};
    if (bn == 192) return launch_tc<192>(ctx, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi, none);
    return launch_tc<128>(ctx, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi, none);
}

int conv_tc(lonnx_ctx *ctx, const ConvArgs &cv, const float *Whi, const float *Wlo, int ldw, const float *bias,
            float *y, int P, int M, int K, int epi) {
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (P <= 0 || M <= 0 || K <= 0 || (ldw & 3) || !al16(Whi) || !al16(Wlo) || !cv.x || cv.img_rows <= 0 ||
        (epi != LONNX_EPI_NONE && epi != LONNX_EPI_RELU) || (int64_t)M * cv.img_rows >= (1ll << 31) ||
        (int64_t)cv.C * cv.H * cv.W >= (1ll << 31))
        return set_error(LONNX_E_UNSUPPORTED, "conv_tc: unsupported operands");
    const int bn = pick_bn(M);
    CUtensorMap mw, mwlo;
    int rc = make_map(&mw, Whi, M, K, ldw, bn);
    if (rc) return rc;
    rc = make_map(&mwlo, Wlo, M, K, ldw, bn);
    if (rc) return rc;
    // the A map is unused in implicit mode (the kernel gathers A itself)
    if (bn == 192) return launch_tc<192>(ctx, mw, mw, mwlo, bias, y, P, M, K, 0, 1.0f, 1.0f, epi, cv);
    return launch_tc<128>(ctx, mw, mw, mwlo, bias, y, P, M, K, 0, 1.0f, 1.0f, epi, cv);
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
