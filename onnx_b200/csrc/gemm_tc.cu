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
//   warps 1, 2  MMA issuers (one lane each, even / odd stages; warp 1 also
//               owns TMEM): 4 K-steps x 3 products per stage, A from TMEM, W
//               from shared memory, into one of two TMEM chunk accumulators
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

#include <algorithm>
#include <type_traits>
#include <mutex>

#include "lonnx_internal.cuh"
#include "tc_common.cuh"

namespace {

using namespace lonnx::tc;

constexpr int BM = 128;
constexpr int BK = 32;                  // fp32 elements per 128-byte row
constexpr int A_TILE = BM * BK * 4;     // 16 KB
constexpr int kThreads = 640;           // 20 warps
// warp roles: 0 TMA, 1-2 MMA (1 owns TMEM), 4-7 A -> TMEM, 8-19 accumulate/epilogue
constexpr int W_TMA = 0, W_MMA = 1, W_MMA2 = 2, W_A0 = 4, W_ACC0 = 8;
// kernel modes: plain GEMM (A by TMA, row-major C); implicit conv (A
// gathered, NCHW C); implicit conv + residual; the two conv modes with an
// NHWC output (row-major C = [pixels, channels], the GEMM epilogue)
constexpr int MODE_GEMM = 0, MODE_CONV = 1, MODE_CONV_RES = 2, MODE_CONV_NHWC = 3, MODE_CONV_RES_NHWC = 4;
// K stages per accumulator chunk.  The tensor core accumulates a chunk
// (CH x 32 K-columns) into TMEM, rounding toward zero; the accumulator warps
// add chunk sums into fp32 registers with round-to-nearest.  Two 32-wide
// stages per chunk halve the drains and give the MMAs four stages of slack
// over an epilogue (two chunk buffers), at a truncation error of a 64-term
// sum per chunk -- still below the reference's own sequential-fp32 error at
// the encoder's K.
//
// Barrier-phase invariant: the two issuers alternate chunks, so when an
// issuer starts a chunk at stage j its last wait on a ring slot was for
// stage j - CH - 1 (or none, for the first chunk of issuer 1 at j = CH).
// Its wait on conv(j % S) with parity (j / S) & 1 is only meaningful once
// the slot's previous phase (stage j - S) has completed: a parity wait on a
// barrier still in that previous phase returns at once (the phase before it
// has the other parity).  The A warps complete stages in order, so the
// previous phase is complete whenever j - S <= j - CH - 1, i.e. S >= CH + 1.
// (CH = 4 with a 3-stage ring broke this and faulted.)
constexpr int CH = 2;
// Drain groups (chunk_group_pos): GRP chunks of one TMEM buffer are summed
// by the tensor core before a drain, a truncating sum of GRP * CH * BK = 192
// terms at most; the issuers' alternation, and so the invariant above, is
// unchanged.  Groups are what lets the next tile's MMAs run under an
// epilogue: with one drain per chunk they stopped two chunks into it.
constexpr int GRP = 3;

// Role timeline of CTA 0 (clock64), compiled only into a diagnostic build
// (-DLONNX_GEMM_TIMELINE); read back with lonnx_debug_gemm_timeline.
// [0, 256): issuer start of chunk c, [256, 512): issuer commit of chunk c,
// [512, 768): accumulator warp 8 past tfull of chunk c, [768, 1024): its
// tdrain arrive, [1024, 1040): epilogue start of tile t, [1040, 1056): end,
// [1056, 1184): 8 marks inside the epilogue of tile t (t < 16), [1184]:
// kernel entry, [1185]: past the dependency wait.
#ifdef LONNX_GEMM_TIMELINE
__device__ long long g_gemm_tl[1192];
#define GTL(off, idx)                                                                      \
    do {                                                                                   \
        if (blockIdx.x == 0 && (idx) < ((off) >= 1184 ? 8 : (off) >= 1056 ? 128 : (off) >= 1024 ? 16 : 256)) \
            g_gemm_tl[(off) + (idx)] = clock64();                                          \
    } while (0)
#else
#define GTL(off, idx) \
    do {              \
    } while (0)
#endif

// RES: the conv epilogue adds a residual tile, prefetched into shared memory
// (BM x BN fp32) while the tile's mainloop runs; it costs one ring stage.
template <int BN, bool RES = false>
struct Cfg {
    static constexpr int W_TILE = BN * BK * 4;
    static constexpr int STAGE = A_TILE + 2 * W_TILE;  // ring slot: A, W_hi, W_lo
    static constexpr int SMEM = 227 * 1024;
    static constexpr int RES_BYTES = RES ? BM * BN * 4 : 0;
    static constexpr int FIT = (SMEM - 1024 - 256 - 2 * BN * 4 - RES_BYTES - (RES ? 4096 : 0)) / STAGE;
    static constexpr int STAGES = FIT > 6 ? 6 : FIT;
    static_assert(STAGES >= 2, "ring too shallow");
    static constexpr int RES_OFF = STAGES * STAGE + 256 + 2 * BN * 4;  // after ring, barriers, bias
    static constexpr int TAB_OFF = RES_OFF + RES_BYTES;  // the rest holds the conv tap table
    static constexpr int TAB_MAX = (SMEM - 1024 - TAB_OFF) / 4;  // tap-table entries
    // accumulator column groups: 64 columns per warp, or 32 when BN is not a
    // multiple of 64 (the 96-wide tile for N = 384 at small M)
    static constexpr int GW = BN % 64 == 0 ? 64 : 32;
    static constexpr int GROUPS = BN / GW;
    static constexpr int NACC = 4 * GROUPS;             // accumulator warps 8 .. 8 + NACC - 1
    // GEMM epilogue: one dense 32 x 16 staging block per accumulator warp
    // (2 KB, 1024-aligned), its 16-byte chunks swizzled as TMA's 64-byte
    // swizzle lays them out: chunk c of row r at c ^ ((r >> 1) & 3), so the
    // block is both a TMA store source and conflict-free for float4 access
    static constexpr int STG_OFF = (TAB_OFF + 1023) & ~1023;
    static constexpr int GEMM_SMEM = STG_OFF + NACC * 2048 + 1024;
    // A warpgroups: warps 4-7, plus warps 8 + NACC .. +3 when the
    // accumulators leave four warps idle (BN <= 128); each group then moves
    // 16 of a stage's 32 K-columns
    static constexpr int NAG = (20 - W_ACC0 - NACC) >= 4 ? 2 : 1;
    static constexpr int W_A1 = W_ACC0 + NACC;
    static constexpr int ACC_COL = 0;                   // TMEM: 2 chunk accumulators [0, 2 BN)
    static constexpr int A_COL = 2 * BN;                // then NAB A buffers of 64 (hi 32 | lo 32)
    static constexpr int NAB = 2 * BN + 3 * 64 <= 512 ? 3 : 2;
    static constexpr int TMEM_COLS = 2 * BN + NAB * 64 <= 256 ? 256 : 512;
    static_assert(3 * STAGES + 5 + NAB <= 30, "barrier area");
    // RES with an NHWC output: the residual tile held as the epilogue's
    // 32 x 16 staging blocks (accumulator warp w, column block ch at block
    // w * GW / 16 + ch), TMA-loaded, finished in place and TMA-stored; one
    // mbarrier per accumulator warp after the TMEM slot
    static constexpr int RESB_OFF = (RES_OFF + 1023) & ~1023;
    static constexpr int RBAR = 3 * STAGES + 6 + NAB;
    static_assert(!RES || RESB_OFF + RES_BYTES <= SMEM - 1024, "residual blocks must fit");
    static_assert(!RES || RBAR + NACC <= 32, "barrier area");
    static_assert(RES || GEMM_SMEM <= SMEM, "GEMM epilogue staging must fit beside the ring");
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
//
// Tiles: tile t = (t / ntn) row block, (t % ntn) column block; CTA b takes
// tiles b, b + gridDim.x, ...  Every role walks one global sequence of
// (tile, stage) steps, so ring slots and barrier phases carry across tiles
// and the accumulator warps' epilogue of one tile overlaps the next tile's
// loads and MMAs.  The row-major epilogue stages C through the ring, so it
// needs one tile per CTA (grid = tiles); the NCHW epilogue (conv) stores from
// registers and runs persistent (grid = SMs).
//
// Implicit-GEMM conv (cv.x != nullptr): no A tensor map; row r of a tile is
// output pixel m0 + r, column k is (c, ky, kx), and the A warps gather the
// taps from the NCHW input themselves (cp.async into the ring's A slots).
template <int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
              const __grid_constant__ CUtensorMap tmWlo, const __grid_constant__ CUtensorMap tmC,
              const float *__restrict__ bias, float *__restrict__ C, int M, int N, int K, int ldc, float alpha,
              float beta, int epi, int *dev_flags, const lonnx::ConvArgs cv, int ksplit, int64_t split_stride,
              int cstore) {
    constexpr bool CONV = MODE != MODE_GEMM, RES = MODE == MODE_CONV_RES || MODE == MODE_CONV_RES_NHWC;
    constexpr bool OUTN = MODE == MODE_CONV_NHWC || MODE == MODE_CONV_RES_NHWC;  // conv with NHWC output
    using G = Cfg<BN, RES>;
    constexpr int S = G::STAGES;
    constexpr int NACC = G::NACC, NAG = G::NAG, NAB = G::NAB;
    static_assert(S >= CH + 1, "a chunk's first conv(s) wait would alias a ring phase (see CH)");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * G::STAGE);
    // [0,S) full  [S,2S) A in TMEM  [2S,3S) stage free  [3S,3S+2) chunk ready
    // [3S+2,3S+4) chunk drained  [3S+4] abort drain  [3S+5,3S+5+NAB) TMEM A buffer free
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 5 + NAB);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *ebias = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + 256);  // [2][BN], NCHW epilogue
    uint32_t *tab = reinterpret_cast<uint32_t *>(smem + G::TAB_OFF);                      // conv tap table
    float *sres = reinterpret_cast<float *>(smem + G::RES_OFF);  // [BN][BM] residual tile (RES)
    float *sresb = reinterpret_cast<float *>(smem + G::RESB_OFF);  // residual blocks (RES, NHWC output)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk_all = (K + BK - 1) / BK;
    const int ntn = (N + BN - 1) / BN, ntiles = ntn * ((M + BM - 1) / BM);
    // GEMM split-K: CTA b takes tile b / ksplit and that tile's K stages
    // [ks * chunk, ks * chunk + nk); its raw sums go to C + ks * split_stride
    const int ks = CONV ? 0 : (int)blockIdx.x % ksplit;
    const int t0 = CONV || ksplit == 1 ? (int)blockIdx.x : (int)blockIdx.x / ksplit;
    const int chunk = (nk_all + ksplit - 1) / ksplit;
    const int nk = CONV ? nk_all : min(chunk, nk_all - ks * chunk);
    const int kofs = ks * chunk * BK;
    if (!CONV && ksplit > 1) C += ks * split_stride;
    // persistent (CTA b takes tiles b, b + gridDim.x, ...) except for split-K
    const int my_tiles = CONV || ksplit == 1
                             ? ((int)blockIdx.x < ntiles && nk > 0 ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0)
                             : (t0 < ntiles && nk > 0 ? 1 : 0);
    const int total = my_tiles * nk;  // (tile, stage) steps of this CTA
    // accumulator chunks: CH consecutive K stages of a tile (the last chunk
    // of a tile may be shorter); one TMEM chunk buffer, one drain per chunk
    const int nch = (nk + CH - 1) / CH, total_ch = my_tiles * nch;
    auto tile_n0 = [&](int t) { return (t % ntn) * BN; };
    auto tile_m0 = [&](int t) { return (t / ntn) * BM; };
    auto step_tile = [&](int j) { return (int)blockIdx.x + (j / nk) * (int)gridDim.x; };
    // drain groups: the chunks of one tile that land in the same TMEM
    // buffer (every other chunk) are summed there GRP at a time before the
    // accumulator warps add them into registers, so the MMAs of a tile's
    // first 2 * GRP chunks need no drain and run under the previous tile's
    // epilogue.  gpos: the chunk's place in its group; a group ends after
    // GRP chunks or with the buffer's last chunk of the tile.
    // (the chunks of a tile in one buffer are those of one parity of ci)
    auto chunk_group_pos = [&](int ci) { return (ci >> 1) % GRP; };
    auto chunk_group_last = [&](int ci, int gpos) { return gpos == GRP - 1 || ci + 2 >= nch; };

    auto full = [&](int s) { return smem_u32(bars + s); };
    auto conv = [&](int s) { return smem_u32(bars + S + s); };
    auto empty = [&](int s) { return smem_u32(bars + 2 * S + s); };
    auto tfull = [&](int b) { return smem_u32(bars + 3 * S + b); };
    auto tdrain = [&](int b) { return smem_u32(bars + 3 * S + 2 + b); };
    const uint32_t drainbar = smem_u32(bars + 3 * S + 4);
    auto afree = [&](int b) { return smem_u32(bars + 3 * S + 5 + b); };
    auto rbar = [&](int w) { return smem_u32(bars + G::RBAR + w); };
    // GEMM epilogue staging: past the tap table in the conv modes (NHWC output)
    const int stg_off = !CONV ? G::STG_OFF : ((G::TAB_OFF + (cv.tab ? nk_all * BK * 4 : 0) + 1023) & ~1023);
    auto stageA = [&](int s) { return smem + s * G::STAGE; };
    auto stageW = [&](int s) { return smem + s * G::STAGE + A_TILE; };
    auto stageWlo = [&](int s) { return smem + s * G::STAGE + A_TILE + G::W_TILE; };
    int issued = 0;

    if (threadIdx.x == 0) {
        GTL(1184, 0);
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(conv(s), 4 * NAG);  // one arrive per A warp
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull(b), 1);
            mbar_init(tdrain(b), NACC);
        }
        for (int b = 0; b < NAB; ++b) mbar_init(afree(b), 1);
        mbar_init(drainbar, 2);  // one commit per issuing thread
        if constexpr (RES && OUTN)
            for (int w = 0; w < NACC; ++w) mbar_init(rbar(w), 1);
        *abort_flag = 0;
        fence_mbar_init();
        if constexpr (!CONV || (RES && OUTN)) prefetch_tmap(&tmA);  // A, or the residual (RES, NHWC)
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmWlo);
    }
    if (CONV && cv.tab) {
        // tap table: entry k = (plane offset of tap k) << 8 | (ky * kw + kx);
        // entries past K (to the next stage) get tap index 63, a bit no
        // pixel's validity mask has, so they read as zero
        const int khw = cv.kh * cv.kw, kend = (K + BK - 1) / BK * BK;
        for (int k = threadIdx.x; k < kend; k += kThreads) {
            uint32_t e = 63u;
            if (k < K) {
                const int c = k / khw, rr = k - c * khw, ky = rr / cv.kw, kx = rr - ky * cv.kw;
                e = ((uint32_t)(c * cv.H * cv.W + ky * cv.dh * cv.W + kx * cv.dw) << 8) | (uint32_t)rr;
            }
            tab[k] = e;
        }
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_u32(tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // set-up done: wait for the previous kernel's results (launched with PDL)
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) GTL(1185, 0);
    bool ok = true;
    const int agroup = (warp >= W_A0 && warp < W_A0 + 4) ? 0 : (NAG == 2 && warp >= G::W_A1 && warp < G::W_A1 + 4) ? 1 : -1;

    if (warp == W_TMA) {
        if (lane == 0) {
            constexpr uint32_t bytes = CONV ? 2 * G::W_TILE : G::STAGE;
            // (tile, K offset) advanced incrementally: no divisions on the issue path
            int t = t0, k0 = 0, s = 0, ph = 0;
            int n0 = tile_n0(t), m0 = tile_m0(t);
            for (int j = 0; j < total && ok; ++j) {
                if (!mbar_wait(empty(s), ph ^ 1, abort_flag)) { ok = false; break; }
                mbar_arrive_expect_tx(full(s), bytes);
                if constexpr (!CONV) tma_load_2d(smem_u32(stageA(s)), &tmA, full(s), kofs + k0, m0);
                tma_load_2d(smem_u32(stageW(s)), &tmW, full(s), kofs + k0, n0);
                tma_load_2d(smem_u32(stageWlo(s)), &tmWlo, full(s), kofs + k0, n0);
                issued = j + 1;
                if (++s == S) { s = 0; ph ^= 1; }
                k0 += BK;
                if (k0 >= nk * BK) {
                    k0 = 0;
                    t += (int)gridDim.x;
                    n0 = tile_n0(t);
                    m0 = tile_m0(t);
                }
            }
        }
    } else if (warp == W_MMA || warp == W_MMA2) {
        // two issuing threads, even and odd stages: issuing one tcgen05.mma
        // costs its thread ~80-100 SM cycles, more than a 128 x 128 x 8 tf32
        // MMA takes to run, so one thread could not keep the tensor pipe fed
        // (measured: 12 MMAs per stage issued in ~1.6k cycles against ~0.8k
        // of execution).  Stage j uses accumulator chunk j & 1, so each
        // issuer owns one chunk; ring slots and TMEM A buffers are per stage.
        // No barrier can run two phases ahead of an issuer: the A warps and
        // the TMA stay within NAB <= S stages of the oldest unfinished MMA.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            // chunk cidx = CH consecutive K stages of one tile, accumulated
            // by the tensor core into TMEM chunk buffer cidx & 1; issuer
            // (cidx & 1) owns that buffer, so a chunk's stages are ordered
            int grp_n = 0;  // drain groups of buffer b begun so far
            for (int cidx = warp - W_MMA; cidx < total_ch && ok; cidx += 2) {
                const int tt = cidx / nch, ci = cidx - tt * nch, b = cidx & 1;
                const int i0 = ci * CH, i1 = min(nk, i0 + CH);
                const int gpos = chunk_group_pos(ci);
                if (gpos == 0) {
                    // a fresh group: the buffer's previous group must be drained
                    if (!mbar_wait(tdrain(b), (grp_n & 1) ^ 1, abort_flag)) { ok = false; break; }
                    ++grp_n;
                }
                GTL(0, cidx);
                const uint32_t acc = tmem + G::ACC_COL + b * BN;
                for (int i = i0; i < i1 && ok; ++i) {
                    const int j = tt * nk + i, s = j % S;
                    if (!mbar_wait(conv(s), (j / S) & 1, abort_flag)) { ok = false; break; }
                    // implicit conv: the A warps do not wait for the W tiles, so the MMA does
                    if constexpr (CONV) {
                        if (!mbar_wait(full(s), (j / S) & 1, abort_flag)) { ok = false; break; }
                    }
                    tc_fence_after();
                    const int ab = j % NAB;
                    const uint32_t ahi = tmem + G::A_COL + ab * 64, alo = ahi + 32;
                    const uint32_t w = smem_u32(stageW(s)), wlo = smem_u32(stageWlo(s));
#pragma unroll
                    for (int kk = 0; kk < BK / 8; ++kk) {
                        const uint64_t dw = smem_desc_sw128(w + kk * 32), dwl = smem_desc_sw128(wlo + kk * 32);
                        mma_tf32_ts(acc, alo + kk * 8, dw, idesc, gpos != 0 || i != i0 || kk != 0);
                        mma_tf32_ts(acc, ahi + kk * 8, dwl, idesc, 1);
                        mma_tf32_ts(acc, ahi + kk * 8, dw, idesc, 1);
                    }
                    mma_commit(empty(s));
                    mma_commit(afree(ab));
                }
                if (ok && chunk_group_last(ci, gpos)) mma_commit(tfull(b));
                GTL(256, cidx);
            }
        }
    } else if (agroup >= 0) {
        // A warps: warp (w % 4) owns TMEM lanes = tile rows 32*(w%4)..+31;
        // each thread moves its row's K-columns [c0, c0 + NC) of every stage
        // into TMEM as hi = tf32(a) and lo = a - hi
        constexpr int NC = BK / NAG;
        const int q = warp & 3, r = q * 32 + lane, c0 = agroup * NC;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::A_COL;
        auto to_tmem = [&](int b, const float *x) {
#pragma unroll
            for (int h = 0; h < NC / 16; ++h) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const float v = x[h * 16 + u], hv = tf32_hi(v);
                    hi[u] = __float_as_uint(hv);
                    lo[u] = __float_as_uint(__fsub_rn(v, hv));
                }
                tmem_st_32x32b_x16(lane_base + b * 64 + c0 + h * 16, hi);
                tmem_st_32x32b_x16(lane_base + b * 64 + 32 + c0 + h * 16, lo);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
        };
        if constexpr (CONV) {
            // implicit-GEMM conv: each thread gathers its pixel's taps of a
            // stage straight from the NCHW input with 4-byte cp.async into
            // its own row of the ring's A slot, S - 1 steps ahead; lanes are
            // consecutive pixels, so each tap is one coalesced warp access;
            // taps outside the image or past K are zero-filled.  Rows are
            // rotated by r words so the 32 lanes hit 32 banks.
            constexpr int D = S - 1;
            int cur_tile = -1, iy0 = 0, ix0 = 0;
            const float *xr = cv.x;
            const int khw = cv.kh * cv.kw, HW = cv.H * cv.W;
            // table path: incremental (tile, stage) of the next gather, the
            // pixel's validity mask over the kh x kw taps for the current tile
            int gt = (int)blockIdx.x, gi = 0, gj = 0, mt = -1;
            uint64_t vmask = 0;
            auto gather_tab = [&]() {
                if (gt != mt) {
                    mt = gt;
                    const int p = tile_m0(gt) + r;
                    vmask = 0;
                    xr = cv.x;
                    if (p < M) {
                        const int hw = cv.Ho * cv.Wo, n = p / hw, rem = p - n * hw;
                        const int oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
                        const int y0 = oy * cv.sh - cv.pt, x0 = ox * cv.sw - cv.pl;
                        xr = cv.x + (int64_t)n * cv.C * HW + (int64_t)y0 * cv.W + x0;
                        int ky = 0, kx = 0;
                        for (int rr = 0; rr < khw; ++rr) {
                            const int yy = y0 + ky * cv.dh, xx = x0 + kx * cv.dw;
                            if ((unsigned)yy < (unsigned)cv.H && (unsigned)xx < (unsigned)cv.W) vmask |= 1ull << rr;
                            if (++kx == cv.kw) { kx = 0; ++ky; }
                        }
                    }
                }
                const uint32_t row = smem_u32(stageA(gj % S)) + r * 128;
                const uint4 *te = reinterpret_cast<const uint4 *>(tab + gi * BK + c0);
#pragma unroll
                for (int u4 = 0; u4 < NC / 4; ++u4) {
                    const uint4 e4 = te[u4];  // 4 taps, same address in every lane
                    const uint32_t e[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const int u = c0 + u4 * 4 + v;
                        const bool in = (vmask >> (e[v] & 255u)) & 1u;
                        cp_async4(row + (((u + r) & 31) << 2), in ? xr + (e[v] >> 8) : cv.x, in ? 4u : 0u);
                    }
                }
                ++gj;
                if (++gi == nk) { gi = 0; gt += (int)gridDim.x; }
            };
            // NHWC path (cv.nhwc): stage i of a tile is tap (ky, kx) = the
            // i / (C / 32)-th tap and channels [32 (i % (C / 32)), +32); each
            // thread copies its NC channels as NC / 4 16-byte cp.async into
            // chunk slots rotated by r (16-byte chunks, 8 per row)
            int nt_tap = 0, nt_cb = 0, nt_ky = 0, nt_kx = 0, y0n = 0, x0n = 0;
            auto gather_nhwc = [&]() {
                if (gt != mt) {
                    mt = gt;
                    nt_tap = nt_cb = nt_ky = nt_kx = 0;
                    const int p = tile_m0(gt) + r;
                    vmask = 0;
                    xr = cv.x;
                    if (p < M) {
                        const int hw = cv.Ho * cv.Wo, n = p / hw, rem = p - n * hw;
                        const int oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
                        y0n = oy * cv.sh - cv.pt;
                        x0n = ox * cv.sw - cv.pl;
                        xr = cv.x + (int64_t)n * cv.C * HW;
                        int ky = 0, kx = 0;
                        for (int rr = 0; rr < khw; ++rr) {
                            const int yy = y0n + ky * cv.dh, xx = x0n + kx * cv.dw;
                            if ((unsigned)yy < (unsigned)cv.H && (unsigned)xx < (unsigned)cv.W) vmask |= 1ull << rr;
                            if (++kx == cv.kw) { kx = 0; ++ky; }
                        }
                    }
                }
                const uint32_t row = smem_u32(stageA(gj % S)) + r * 128;
                const bool in = (vmask >> nt_tap) & 1u;
                const float *src = in ? xr + ((int64_t)(y0n + nt_ky * cv.dh) * cv.W + (x0n + nt_kx * cv.dw)) * cv.C +
                                            nt_cb * BK + c0
                                      : cv.x;
#pragma unroll
                for (int q4 = 0; q4 < NC / 4; ++q4) {
                    const int qq = c0 / 4 + q4;
                    cp_async16(row + (((qq + r) & 7) << 4), in ? src + q4 * 4 : cv.x, in ? 16u : 0u);
                }
                if (++nt_cb * BK == cv.C) {
                    nt_cb = 0;
                    ++nt_tap;
                    if (++nt_kx == cv.kw) { nt_kx = 0; ++nt_ky; }
                }
                ++gj;
                if (++gi == nk) { gi = 0; gt += (int)gridDim.x; }
            };
            auto gather = [&](int j) {
                if (cv.nhwc) { gather_nhwc(); return; }
                if (cv.tab) { gather_tab(); return; }
                const int t = step_tile(j), i = j % nk;
                if (t != cur_tile) {
                    cur_tile = t;
                    const int p = tile_m0(t) + r;
                    iy0 = -(1 << 20);
                    ix0 = 0;
                    xr = cv.x;
                    if (p < M) {
                        const int hw = cv.Ho * cv.Wo, n = p / hw, rem = p - n * hw;
                        const int oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
                        iy0 = oy * cv.sh - cv.pt;
                        ix0 = ox * cv.sw - cv.pl;
                        xr = cv.x + (int64_t)n * cv.C * HW + (int64_t)iy0 * cv.W + ix0;
                    }
                }
                const uint32_t row = smem_u32(stageA(j % S)) + r * 128;
                const int k = i * BK + lane;
                int off = 0, dy = -(1 << 20), dx = 0;  // taps past K read as zero
                if (k < K) {
                    const int c = k / khw, rr = k - c * khw, ky = rr / cv.kw, kx = rr - ky * cv.kw;
                    dy = ky * cv.dh;
                    dx = kx * cv.dw;
                    off = c * HW + dy * cv.W + dx;
                }
#pragma unroll
                for (int u = c0; u < c0 + NC; ++u) {
                    const int o = __shfl_sync(0xffffffffu, off, u);
                    const int yy = iy0 + __shfl_sync(0xffffffffu, dy, u);
                    const int xx = ix0 + __shfl_sync(0xffffffffu, dx, u);
                    const bool in = (unsigned)yy < (unsigned)cv.H && (unsigned)xx < (unsigned)cv.W;
                    cp_async4(row + (((u + r) & 31) << 2), in ? xr + o : cv.x, in ? 4u : 0u);
                }
            };
            for (int j = 0; j < D; ++j) {
                if (j < total) gather(j);
                cp_async_commit();
            }
            for (int j = 0; j < total && ok; ++j) {
                const int s = j % S, b = j % NAB;
                if (j + D < total) gather(j + D);
                cp_async_commit();
                cp_async_wait<D>();  // this thread's taps of step j have landed
                const float *row = reinterpret_cast<const float *>(stageA(s) + r * 128);
                float x[NC];
                if (cv.nhwc) {
#pragma unroll
                    for (int q4 = 0; q4 < NC / 4; ++q4) {
                        const float4 v4 = *reinterpret_cast<const float4 *>(row + (((c0 / 4 + q4 + r) & 7) << 2));
                        x[q4 * 4] = v4.x;
                        x[q4 * 4 + 1] = v4.y;
                        x[q4 * 4 + 2] = v4.z;
                        x[q4 * 4 + 3] = v4.w;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < NC; ++u) x[u] = row[(c0 + u + r) & 31];
                }
                if (!mbar_wait(afree(b), ((j / NAB) & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                to_tmem(b, x);
                if (lane == 0) mbar_arrive(conv(s));
            }
            cp_async_wait<0>();
        } else {
            for (int j = 0; j < total && ok; ++j) {
                const int s = j % S, b = j % NAB;
                if (!mbar_wait(full(s), (j / S) & 1, abort_flag)) { ok = false; break; }
                if (!mbar_wait(afree(b), ((j / NAB) & 1) ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint8_t *row = stageA(s) + r * 128;
#pragma unroll
                for (int h = 0; h < NC / 16; ++h) {
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        const int c = c0 / 4 + h * 4 + c4;  // 16-byte chunk, 128B-swizzled
                        const float4 v = *reinterpret_cast<const float4 *>(row + (((c ^ (r & 7))) << 4));
                        const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float hv = tf32_hi(x[u]);
                            hi[c4 * 4 + u] = __float_as_uint(hv);
                            lo[c4 * 4 + u] = __float_as_uint(__fsub_rn(x[u], hv));
                        }
                    }
                    tmem_st_32x32b_x16(lane_base + b * 64 + c0 + h * 16, hi);
                    tmem_st_32x32b_x16(lane_base + b * 64 + 32 + c0 + h * 16, lo);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(conv(s));
            }
        }
    } else if (warp >= W_ACC0 && warp < W_ACC0 + NACC) {
        // accumulator / epilogue warps: warp w owns TMEM lanes 32*(w%4)..+31
        // (tile rows) and one GW-column group of the tile
        const int q = warp & 3, grp = (warp - W_ACC0) >> 2;
        constexpr int GW = G::GW;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + G::ACC_COL + grp * GW;
        const int rloc = q * 32 + lane, wi = warp - W_ACC0;
        int drained0 = 0, drained1 = 0;  // drain groups of buffers 0 and 1 so far
        bool rpend = false;              // residual blocks in flight (RES, NHWC output)
        int rpar = 0;
        for (int tt = 0; tt < my_tiles && ok; ++tt) {
            const int t = t0 + tt * (int)gridDim.x, n0 = tile_n0(t), m0 = tile_m0(t);
            if constexpr (RES && OUTN) {
                // the warp's residual rows x columns as GW / 16 blocks of 32 x 16,
                // by TMA, once this warp's stores of the previous tile have read
                // the blocks; landed long before the epilogue needs them
                if (lane == 0) {
                    bulk_wait_group_read0();
                    mbar_arrive_expect_tx(rbar(wi), (GW / 16) * 2048);
#pragma unroll
                    for (int ch = 0; ch < GW / 16; ++ch)
                        tma_load_2d(smem_u32(sresb + (wi * (GW / 16) + ch) * 512), &tmA, rbar(wi),
                                    n0 + grp * GW + ch * 16, m0 + q * 32);
                    rpend = true;
                    rpar = tt & 1;
                }
            } else if constexpr (RES) {
                // the warp's residual block (its 32 pixels x its 64 channels)
                // into shared memory now, read back in the epilogue after a
                // wait on the copy group and a __syncwarp.  With 4 | pixels
                // per image, each copy is 16 bytes: 4 consecutive pixels of one
                // channel (16 per thread; 64 four-byte copies per thread cost
                // ~5.6k cycles of the accumulator warps' time per tile)
                if (cv.img_rows % 4 == 0 && ((uintptr_t)cv.res & 15) == 0) {
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {
                        const int f = lane + 32 * i, rg = f & 7, u = f >> 3;  // 4-pixel group, channel
                        const int grow = m0 + q * 32 + rg * 4, col = n0 + grp * 64 + u;
                        const bool in = grow < M && col < N;
                        const int img = grow / cv.img_rows, pix = grow - img * cv.img_rows;
                        const float *src = in ? cv.res + ((int64_t)img * N + col) * cv.img_rows + pix : cv.res;
                        cp_async16(smem_u32(sres) + (uint32_t)((grp * 64 + u) * BM + q * 32 + rg * 4) * 4, src,
                                   in ? 16u : 0u);
                    }
                } else {
                    const int grow = m0 + rloc;
                    if (grow < M) {
                        const int img = grow / cv.img_rows, pix = grow - img * cv.img_rows;
                        const float *rs = cv.res + (int64_t)img * N * cv.img_rows + pix;
                        const uint32_t d0 = smem_u32(sres) + (uint32_t)(grp * 64 * BM + rloc) * 4;
#pragma unroll 8
                        for (int u = 0; u < 64; ++u) {
                            const int col = n0 + grp * 64 + u;
                            cp_async4(d0 + u * BM * 4, col < N ? rs + col * cv.img_rows : cv.res, col < N ? 4u : 0u);
                        }
                    }
                }
                cp_async_commit();
            }
            float acc[GW];
#pragma unroll
            for (int j = 0; j < GW; ++j) acc[j] = 0.0f;
            for (int ci = 0; ci < nch && ok; ++ci) {
                const int cidx = tt * nch + ci, b = cidx & 1;
                if (!chunk_group_last(ci, chunk_group_pos(ci))) continue;  // the group goes on in TMEM
                const int gn = b ? drained1++ : drained0++;
                if (!mbar_wait(tfull(b), gn & 1, abort_flag)) { ok = false; break; }
                if (warp == W_ACC0 && lane == 0) GTL(512, cidx);
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < GW / 16; ++c) {
                    uint32_t rr[16];
                    tmem_ld_32x32b_x16(lane_base + b * BN + c * 16, rr);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < 16; ++u) acc[c * 16 + u] = __fadd_rn(acc[c * 16 + u], __uint_as_float(rr[u]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tdrain(b));
                if (warp == W_ACC0 && lane == 0) GTL(768, cidx);
            }
            if (!ok) break;
            if constexpr (CONV && !OUTN) {
                if (warp == W_ACC0 && lane == 0) GTL(1024, tt);
                // NCHW output: row = (image, pixel), column = channel; a
                // warp's lanes hold consecutive pixels, so each column store
                // coalesces.  The optional residual (same layout) is added
                // after the bias and before the activation, as a following
                // Add node would.
                // the tile's bias (times beta) in shared memory, double-buffered
                // by tile parity: costs no registers in the store loop
                float *sb = ebias + (tt & 1) * BN;
                for (int c = threadIdx.x - W_ACC0 * 32; c < BN; c += NACC * 32) {
                    const int col = n0 + c;
                    float bv = 0.0f;
                    if (bias && col < N) bv = beta == 1.0f ? __ldg(bias + col) : __fmul_rn(beta, __ldg(bias + col));
                    sb[c] = bv;
                }
                asm volatile("bar.sync 1, %0;" ::"n"(NACC * 32) : "memory");
                if constexpr (RES) {
                    // the residual block: this thread's copies, then the
                    // other lanes' (every lane of the warp reaches this)
                    cp_async_wait<0>();
                    __syncwarp();
                }
                const int grow = m0 + rloc;
                if (grow < M) {
                    const int img = grow / cv.img_rows, pix = grow - img * cv.img_rows;
                    const int64_t o = (int64_t)img * N * cv.img_rows + pix;
                    float *dst = C + o;
                    const int cs = cv.img_rows;  // N * img_rows (one image's output) < 2^31
                    const int cb = n0 + grp * 64;
                    const float *sbg = sb + grp * 64;  // zero where there is no bias
                    const bool relu = epi == LONNX_EPI_RELU;
                    // x * alpha is exact for alpha == 1, so it is applied unconditionally;
                    // Relu keeps NaN -> 0 (x > 0 is false for NaN)
                    if constexpr (!RES) {
#pragma unroll
                        for (int u = 0; u < 64; ++u) {
                            float x = __fadd_rn(__fmul_rn(acc[u], alpha), sbg[u]);
                            x = (relu && !(x > 0.0f)) ? 0.0f : x;
                            if (cb + u < N) dst[(cb + u) * cs] = x;
                        }
                    } else {
                        const float *sr = sres + grp * 64 * BM + rloc;
#pragma unroll
                        for (int u = 0; u < 64; ++u) {
                            float x = __fadd_rn(__fmul_rn(acc[u], alpha), sbg[u]);
                            x = __fadd_rn(x, sr[u * BM]);
                            x = (relu && !(x > 0.0f)) ? 0.0f : x;
                            if (cb + u < N) dst[(cb + u) * cs] = x;
                        }
                    }
                }
                if (warp == W_ACC0 && lane == 0) GTL(1040, tt);
                continue;
            }
            if (warp == W_ACC0 && lane == 0) GTL(1024, tt);
            // row-major epilogue, overlapping the next tile's loads and MMAs:
            // each warp moves its 32 rows x 64 columns out 16 columns at a
            // time through a private 32 x 16 staging block in shared memory
            // (the tail past the ring), so that its stores coalesce along
            // rows; alpha, bias and the activation are applied in a
            // non-unrolled loop (the activation code appears once per value
            // of a float4: an unrolled per-element epilogue with Erf-GELU
            // inlined overflows the instruction cache).
            float *sb = ebias + (tt & 1) * BN;
            for (int c = threadIdx.x - W_ACC0 * 32; c < BN; c += NACC * 32) {
                const int col = n0 + c;
                float bv = 0.0f;
                if (bias && col < N) bv = beta == 1.0f ? __ldg(bias + col) : __fmul_rn(beta, __ldg(bias + col));
                sb[c] = bv;
            }
            if (warp == W_ACC0 && lane == 0) GTL(1056, tt * 8);
            asm volatile("bar.sync 1, %0;" ::"n"(NACC * 32) : "memory");
            if (warp == W_ACC0 && lane == 0) GTL(1056, tt * 8 + 1);
            auto sidx = [](int r, int c4) { return r * 16 + ((c4 ^ ((r >> 1) & 3)) << 2); };
            const int rbase = m0 + q * 32, cbase = n0 + grp * GW;
            const float *sbg = sb + grp * GW;
            if constexpr (RES && OUTN) {
                // residual conv, NHWC output: lane = row; alpha, bias (zero
                // where there is none), the residual and the activation in the
                // order of the NCHW epilogue, written over the residual block,
                // which then leaves by TMA store
                if (lane == 0) {
                    if (!mbar_wait(rbar(wi), rpar, abort_flag)) ok = false;
                    rpend = false;
                }
                ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
                if (!ok) break;
                const bool relu = epi == LONNX_EPI_RELU;
#pragma unroll
                for (int ch = 0; ch < GW / 16; ++ch) {
                    float *blk = sresb + (wi * (GW / 16) + ch) * 512;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 b4 = *reinterpret_cast<const float4 *>(sbg + ch * 16 + 4 * u);  // broadcast
                        const float4 r4 = *reinterpret_cast<const float4 *>(blk + sidx(lane, u));
                        const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, rv[4] = {r4.x, r4.y, r4.z, r4.w};
                        float v[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            float x = __fadd_rn(__fmul_rn(acc[ch * 16 + 4 * u + k], alpha), bb[k]);
                            x = __fadd_rn(x, rv[k]);
                            v[k] = (relu && !(x > 0.0f)) ? 0.0f : x;
                        }
                        *reinterpret_cast<float4 *>(blk + sidx(lane, u)) = make_float4(v[0], v[1], v[2], v[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && cbase + ch * 16 < N) {
                        tma_store_2d(&tmC, smem_u32(blk), cbase + ch * 16, rbase);
                        bulk_commit_group();
                    }
                }
                if (warp == W_ACC0 && lane == 0) GTL(1040, tt);
                continue;
            }
            // 32 x 16 staging block of this warp; cstore: the finished block
            // leaves by TMA store (tmC, 64-byte swizzle) instead of st.global
            float *stg = reinterpret_cast<float *>(smem + stg_off) + (warp - W_ACC0) * 512;
            const bool vec = (ldc & 3) == 0 && (N & 3) == 0 && ((uintptr_t)C & 15) == 0;
#pragma unroll
            for (int ch = 0; ch < GW / 16; ++ch) {
                if (warp == W_ACC0 && lane == 0) GTL(1056, tt * 8 + 2 + ch);
                if (cstore && lane == 0) bulk_wait_group_read0();  // the previous block has left
                __syncwarp();
                // (a conv with an NHWC output always stores by TMA and has no GELU)
                if (OUTN || (cstore && epi != LONNX_EPI_GELU_ERF)) {
                    // lane = row: alpha, the column's bias (the same for every
                    // lane) and Relu straight on the accumulators, then the
                    // finished block goes out by TMA -- no read-back
                    const bool relu = epi == LONNX_EPI_RELU;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 b4 = *reinterpret_cast<const float4 *>(sbg + ch * 16 + 4 * u);  // broadcast
                        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                        float v[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            float x = acc[ch * 16 + 4 * u + k];
                            if (alpha != 1.0f) x = __fmul_rn(x, alpha);
                            if (bias || CONV) x = __fadd_rn(x, bb[k]);
                            v[k] = (relu && !(x > 0.0f)) ? 0.0f : x;
                        }
                        *reinterpret_cast<float4 *>(stg + sidx(lane, u)) = make_float4(v[0], v[1], v[2], v[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && cbase + ch * 16 < N) {
                        tma_store_2d(&tmC, smem_u32(stg), cbase + ch * 16, rbase);
                        bulk_commit_group();
                    }
                    continue;
                }
                if constexpr (OUTN) continue;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    *reinterpret_cast<float4 *>(stg + sidx(lane, u)) = make_float4(
                        acc[ch * 16 + 4 * u], acc[ch * 16 + 4 * u + 1], acc[ch * 16 + 4 * u + 2], acc[ch * 16 + 4 * u + 3]);
                __syncwarp();
                // float4 e4 = lane + 32 i of the 32 x 16 block: row e4 / 4, columns 4 (e4 % 4) ..
#pragma unroll 1
                for (int i = 0; i < 4; ++i) {
                    const int e4 = lane + 32 * i, rr = e4 >> 2, c4i = e4 & 3, c4 = c4i * 4;
                    const int grow = rbase + rr, col0 = cbase + ch * 16 + c4;
                    float *sp = stg + sidx(rr, c4i);
                    const float4 raw = *reinterpret_cast<const float4 *>(sp);
                    float v[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        float x = v[u];
                        if (alpha != 1.0f) x = __fmul_rn(x, alpha);
                        if (bias || CONV) x = __fadd_rn(x, sbg[ch * 16 + c4 + u]);
                        if (epi == LONNX_EPI_RELU) x = x > 0.0f ? x : 0.0f;
                        else if (epi == LONNX_EPI_GELU_ERF) x = lonnx_gelu_fast(x);
                        v[u] = x;
                    }
                    if (cstore) {
                        *reinterpret_cast<float4 *>(sp) = make_float4(v[0], v[1], v[2], v[3]);
                        continue;
                    }
                    if (grow >= M) continue;
                    float *dst = C + (int64_t)grow * ldc + col0;
                    if (vec && col0 + 3 < N) {
                        *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
                        for (int u = 0; u < 4; ++u)
                            if (col0 + u < N) dst[u] = v[u];
                    }
                }
                if (cstore) {
                    fence_proxy_async_smem();  // the block's generic writes, visible to the TMA unit
                    __syncwarp();
                    if (lane == 0 && cbase + ch * 16 < N) {
                        tma_store_2d(&tmC, smem_u32(stg), cbase + ch * 16, rbase);
                        bulk_commit_group();
                    }
                }
            }
            if (warp == W_ACC0 && lane == 0) GTL(1040, tt);
        }
        if (cstore && lane == 0) bulk_wait_group0();  // every block stored before the CTA exits
        if (RES && OUTN && lane == 0 && rpend) mbar_wait(rbar(wi), rpar, nullptr, 400000000ll);  // loads in flight
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
        if ((warp == W_MMA || warp == W_MMA2) && lane == 0) {
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
int encode_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
               int kind);

// Encoded maps are cached per host thread (a map is a pure function of its
// arguments): encoding costs the host more than a small GEMM runs on the
// device, and the graph executor calls with the same buffers every step.
// kind 0: operand loads, box 32 columns x box_rows, 128-byte swizzle;
// kind 1: epilogue stores, box 16 columns x box_rows, 64-byte swizzle.
int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
             int kind = 0) {
    struct Entry {
        const float *base;
        int64_t rows, cols, ld;
        int box, kind;
        CUtensorMap map;
    };
    constexpr int kEntries = 64;
    static thread_local Entry cache[kEntries];
    static thread_local int next = 0;
    for (int i = 0; i < kEntries; ++i) {
        const Entry &e = cache[i];
        if (e.base == base && e.rows == rows && e.cols == cols && e.ld == ld && e.box == box_rows && e.kind == kind &&
            base) {
            *map = e.map;
            return LONNX_OK;
        }
    }
    const int rc = encode_map(map, base, rows, cols, ld, box_rows, kind);
    if (rc == LONNX_OK) {
        cache[next] = Entry{base, rows, cols, ld, box_rows, kind, *map};
        next = (next + 1) % kEntries;
    }
    return rc;
}

int encode_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
               int kind) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return lonnx::set_error(LONNX_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {(cuuint32_t)(kind ? 16 : BK), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, kind ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return lonnx::set_error(LONNX_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LONNX_OK;
}

// The epilogue stores C by TMA when C can be described by a tensor map
// (16-byte aligned, ldc a multiple of 4) and K is not split;
// LONNX_GEMM_TMA_STORE=0 keeps the per-thread global stores.
bool tma_store_enabled() {
    static const bool on = [] {
        const char *e = getenv("LONNX_GEMM_TMA_STORE");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int BN, int MODE>
int launch_tc(lonnx_ctx *ctx, const CUtensorMap &ma, const CUtensorMap &mw, const CUtensorMap &mwlo,
              const float *bias, float *C, int M, int N, int K, int ldc, float alpha, float beta, int epi,
              const lonnx::ConvArgs &cv, int ksplit = 1, int64_t split_stride = 0) {
    CUtensorMap mc = mw;  // unused unless cstore
    int cstore = 0;
    // (the residual conv with an NHWC output always stores by TMA: its
    // epilogue finishes the tile in the TMA-loaded residual blocks)
    if (((MODE == MODE_GEMM && ksplit == 1 && tma_store_enabled()) || MODE == MODE_CONV_NHWC ||
         MODE == MODE_CONV_RES_NHWC) &&
        (ldc & 3) == 0 && ((uintptr_t)C & 15) == 0) {
        const int rc = make_map(&mc, C, M, N, ldc, 32, 1);
        if (rc) return rc;
        cstore = 1;
    }
    using G = Cfg<BN, MODE == MODE_CONV_RES || MODE == MODE_CONV_RES_NHWC>;
    static bool attr_set[64] = {false};
    if (!attr_set[ctx->device & 63]) {
        LONNX_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        G::SMEM));
        attr_set[ctx->device & 63] = true;
    }
    const int64_t tiles = (int64_t)((N + BN - 1) / BN) * ((M + BM - 1) / BM);
    if (tiles >= (1ll << 31)) return lonnx::set_error(LONNX_E_UNSUPPORTED, "gemm_tc: too many tiles");
    // one persistent CTA per SM (split-K: one CTA per tile and split)
    const int64_t grid = ksplit == 1 ? (tiles > ctx->num_sms ? ctx->num_sms : tiles) : tiles * ksplit;
    // the tail of shared memory holds the conv tap table or the GEMM epilogue staging
    const int smem = MODE != MODE_GEMM ? G::SMEM : G::GEMM_SMEM;
    return lonnx::launch_pdl(ctx, k_gemm_tf32x3<BN, MODE>, dim3((unsigned)grid), dim3(kThreads), (size_t)smem, ma, mw,
                             mwlo, mc, bias, C, M, N, K, ldc, alpha, beta, epi, ctx->dev_flags, cv, ksplit,
                             split_stride, cstore);
}

// Split-K finish: C = act(alpha * sum_s ws[s] + beta * bias), the partial
// tiles summed in split order (deterministic), one pass over the workspace.
__global__ void k_splitk_reduce(const float *__restrict__ ws, int splits, int64_t stride, int M, int N, int ldc,
                                const float *__restrict__ bias, float alpha, float beta, int epi,
                                float *__restrict__ C) {
    const int64_t total = (int64_t)M * N;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += step) {
        float x = ws[i];
        for (int sp = 1; sp < splits; ++sp) x = __fadd_rn(x, ws[sp * stride + i]);
        const int m = (int)(i / N), n = (int)(i - (int64_t)m * N);
        if (alpha != 1.0f) x = __fmul_rn(x, alpha);
        if (bias) x = __fadd_rn(x, beta == 1.0f ? bias[n] : __fmul_rn(beta, bias[n]));
        if (epi == LONNX_EPI_RELU) x = x > 0.0f ? x : 0.0f;
        else if (epi == LONNX_EPI_GELU_ERF) x = lonnx_gelu_chain(x);
        C[(int64_t)m * ldc + n] = x;
    }
}

// Tile width for N: 192, 128 or 96, by a cost model of the persistent launch:
// rounds of tiles over the SMs times the relative time of one tile.  A
// 128-wide tile takes ~0.77 of a 192-wide one (its stages are MMA-issue
// bound; measured with the widths forced on the encoder at batch 256:
// 11.2 vs 10.1 ms per step), so the narrower tile wins only when it does not
// add a round: e.g. N = 384 at M = 4096 (96 tiles vs 64, one round each),
// but not at M = 8192 (192 tiles = 2 rounds vs 128 tiles = 1).  A 96-wide
// tile (~0.6) fills one round where 128-wide ones leave SMs idle: N = 384 at
// M = 4096 is 128 tiles for 148 SMs (FFN2 37.9 -> 33.2 us).  The width
// does not change any output element's summation order.
int pick_bn(int M, int N, int sms) {
    static const int forced = [] {
        const char *e = getenv("LONNX_GEMM_BN");
        return e ? atoi(e) : 0;
    }();
    if (forced == 96 || forced == 128 || forced == 192) return forced;
    const int64_t rows = (M + BM - 1) / BM;
    auto rounds = [&](int bn) { return (rows * ((N + bn - 1) / bn) + sms - 1) / sms; };
    // relative tile times, measured on B200: 128-wide ~0.77 and 96-wide
    // ~0.6 of a 192-wide tile; ties go to the wider tile
    const double c192 = (double)rounds(192), c128 = 0.77 * (double)rounds(128), c96 = 0.6 * (double)rounds(96);
    if (c96 < c128 && c96 < c192) return 96;
    return c128 < c192 ? 128 : 192;
}

// Conv tile width: the least padding of M among 128, 192 and 64 (ties to
// the wider tile); 64-channel convs get BN = 64 instead of half-empty tiles.
// With a residual the tile must leave room for it: 128 or 64.
int pick_bn_conv(int M, bool res) {
    int best = 128, waste = (M + 127) / 128 * 128 - M;
    for (int bn : {192, 64}) {
        if (res && bn == 192) continue;
        const int w = (M + bn - 1) / bn * bn - M;
        if (w < waste) { best = bn; waste = w; }
    }
    return best;
}

}  // namespace

namespace lonnx {

// 2-D fp32 tensor map (box = box_rows x 32, 128-byte swizzle) for other
// tensor-core kernels of this library.
int make_tile_map_f32(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    return make_map(map, base, rows, cols, ld, box_rows);
}

int gemm_tc(lonnx_ctx *ctx, const float *A, const float *Whi, const float *Wlo, const float *bias, float *C, int M,
            int N, int K, int lda, int ldw, int ldc, float alpha, float beta, int epi, bool allow_scratch,
            bool split_k) {
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (!Wlo) return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: weight must be pre-split");
    if (M <= 0 || N <= 0 || K <= 0 || (lda & 3) || (ldw & 3) || !al16(A) || !al16(Whi) || !al16(Wlo))
        return set_error(LONNX_E_UNSUPPORTED, "gemm_tc: operands not 16-byte aligned");
    const int bn = pick_bn(M, N, ctx->num_sms);
    CUtensorMap ma, mw, mwlo;
    int rc = make_map(&ma, A, M, K, lda, BM);
    if (rc) return rc;
    rc = make_map(&mw, Whi, N, K, ldw, bn);
    if (rc) return rc;
    rc = make_map(&mwlo, Wlo, N, K, ldw, bn);
    if (rc) return rc;
    const ConvArgs none{};
    // too few output tiles to fill the SMs: split K (each split >= 3 stages,
    // at most 16), partial tiles into a workspace, then a fixed-order sum.
    // Needs a device allocation; only when the caller asks for it (split_k).
    const int64_t tiles = (int64_t)((N + bn - 1) / bn) * ((M + BM - 1) / BM);
    const int nk = (K + BK - 1) / BK;
    int ksplit = 1;
    // (a problem this small is bound by its launches: one kernel, no split)
    if (split_k && allow_scratch && tiles * 2 <= ctx->num_sms && (int64_t)M * N * K >= ((int64_t)1 << 26)) {
        ksplit = (int)(ctx->num_sms / tiles);
        ksplit = std::min(ksplit, std::min(nk / 3, 16));
        if (ksplit > 1) ksplit = std::min(ksplit, nk);  // every split gets at least one stage
        while (ksplit > 1 && (ksplit - 1) * ((nk + ksplit - 1) / ksplit) >= nk) --ksplit;
    }
    if (ksplit > 1) {
        const int64_t stride = (int64_t)M * N;
        void *ws = nullptr;
        rc = ctx_alloc(ctx, (size_t)ksplit * stride * 4, &ws);
        if (rc) return rc;
        float *w = (float *)ws;
        rc = bn == 192  ? launch_tc<192, MODE_GEMM>(ctx, ma, mw, mwlo, nullptr, w, M, N, K, N, 1.0f, 1.0f,
                                                    LONNX_EPI_NONE, none, ksplit, stride)
             : bn == 96 ? launch_tc<96, MODE_GEMM>(ctx, ma, mw, mwlo, nullptr, w, M, N, K, N, 1.0f, 1.0f,
                                                   LONNX_EPI_NONE, none, ksplit, stride)
                        : launch_tc<128, MODE_GEMM>(ctx, ma, mw, mwlo, nullptr, w, M, N, K, N, 1.0f, 1.0f,
                                                    LONNX_EPI_NONE, none, ksplit, stride);
        if (rc == LONNX_OK) {
            int64_t blocks = (stride + 255) / 256;
            if (blocks > (int64_t)ctx->num_sms * 8) blocks = (int64_t)ctx->num_sms * 8;
            k_splitk_reduce<<<(int)blocks, 256, 0, ctx->stream>>>(w, ksplit, stride, M, N, ldc, bias, alpha, beta,
                                                                 epi, C);
            rc = cudaGetLastError() == cudaSuccess ? LONNX_OK : set_error(LONNX_E_CUDA, "split-K reduce launch");
            if (rc == LONNX_OK) ctx->launches++;
        }
        ctx_free(ctx, ws);
        return rc;
    }
    if (bn == 192) return launch_tc<192, MODE_GEMM>(ctx, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi, none);
    if (bn == 96) return launch_tc<96, MODE_GEMM>(ctx, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi, none);
    return launch_tc<128, MODE_GEMM>(ctx, ma, mw, mwlo, bias, C, M, N, K, ldc, alpha, beta, epi, none);
}

int conv_tc(lonnx_ctx *ctx, const ConvArgs &cv, const float *Whi, const float *Wlo, int ldw, const float *bias,
            float *y, int P, int M, int K, int epi) {
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    if (P <= 0 || M <= 0 || K <= 0 || (ldw & 3) || !al16(Whi) || !al16(Wlo) || !cv.x || cv.img_rows <= 0 ||
        (epi != LONNX_EPI_NONE && epi != LONNX_EPI_RELU) || (int64_t)M * cv.img_rows >= (1ll << 31) ||
        (int64_t)cv.C * cv.H * cv.W >= (1ll << 31))
        return set_error(LONNX_E_UNSUPPORTED, "conv_tc: unsupported operands");
    const bool res = cv.res != nullptr;
    const int bn = pick_bn_conv(M, res);
    ConvArgs a = cv;
    const int kend = (K + BK - 1) / BK * BK;
    const int tab_max = bn == 192 ? Cfg<192>::TAB_MAX
                        : bn == 64 ? (res ? Cfg<64, true>::TAB_MAX : Cfg<64>::TAB_MAX)
                                   : (res ? Cfg<128, true>::TAB_MAX : Cfg<128>::TAB_MAX);
    if (cv.out_nhwc && ((M & 3) || !al16(y) || (res && (!cv.nhwc || !al16(cv.res)))))
        return set_error(LONNX_E_UNSUPPORTED, "conv_tc: NHWC output needs M %% 4 == 0, aligned y / res, NHWC x");
    // NHWC output without a residual: the GEMM epilogue's staging blocks sit
    // past the tap table (1024-aligned)
    const int nacc = bn == 192 ? Cfg<192>::NACC : bn == 64 ? Cfg<64>::NACC : Cfg<128>::NACC;
    const int stg_bytes = cv.out_nhwc && !res ? nacc * 2048 + 1024 : 0;
    if (stg_bytes > tab_max * 4) return set_error(LONNX_E_UNSUPPORTED, "conv_tc: no room for the epilogue staging");
    a.tab = !cv.nhwc && kend * 4 + stg_bytes <= tab_max * 4 && cv.kh * cv.kw <= 63 &&
            (int64_t)cv.C * cv.H * cv.W < (1ll << 24);
    if (cv.nhwc && (cv.C % BK || cv.kh * cv.kw > 63 || K != cv.C * cv.kh * cv.kw))
        return set_error(LONNX_E_UNSUPPORTED, "conv_tc: NHWC gather needs C % 32 == 0 and <= 63 taps");
    CUtensorMap mw, mwlo;
    int rc = make_map(&mw, Whi, M, K, ldw, bn);
    if (rc) return rc;
    rc = make_map(&mwlo, Wlo, M, K, ldw, bn);
    if (rc) return rc;
    // the A map is unused in implicit mode (the kernel gathers A itself); the
    // residual conv with an NHWC output passes the residual's map there
    if (res) {
        CUtensorMap mr = mw;
        if (a.out_nhwc) {
            rc = make_map(&mr, cv.res, P, M, M, 32, 1);
            if (rc) return rc;
        }
        if (a.out_nhwc) {
            if (bn == 64)
                return launch_tc<64, MODE_CONV_RES_NHWC>(ctx, mr, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
            return launch_tc<128, MODE_CONV_RES_NHWC>(ctx, mr, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
        }
        if (bn == 64) return launch_tc<64, MODE_CONV_RES>(ctx, mr, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
        return launch_tc<128, MODE_CONV_RES>(ctx, mr, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
    }
    if (a.out_nhwc) {
        if (bn == 192) return launch_tc<192, MODE_CONV_NHWC>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
        if (bn == 64) return launch_tc<64, MODE_CONV_NHWC>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
        return launch_tc<128, MODE_CONV_NHWC>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
    }
    if (bn == 192) return launch_tc<192, MODE_CONV>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
    if (bn == 64) return launch_tc<64, MODE_CONV>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
    return launch_tc<128, MODE_CONV>(ctx, mw, mw, mwlo, bias, y, P, M, K, M, 1.0f, 1.0f, epi, a);
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

#ifdef LONNX_GEMM_TIMELINE
extern "C" LONNX_API int lonnx_debug_gemm_timeline(long long *host, int n) {
    LONNX_CUDA(cudaMemcpyFromSymbol(host, g_gemm_tl, sizeof(long long) * (n < 1192 ? n : 1192)));
    return LONNX_OK;
}
#endif
