// A whole small network in one launch: the chain Conv (+bias, +ReLU) ->
// MaxPool -> ... -> Reshape -> MatMul (+bias) of a batch-1 CNN such as
// mnist-8, on one cluster of CTAs.
//
// Run as separate kernels, a net this size (mnist-8: ~1.6 MFLOP) pays a
// launch and a dependency wait per op for a few microseconds of work each;
// here it is one launch.  Each layer computes its outputs with exactly the
// arithmetic of the kernel the executor would otherwise launch for it:
//   Conv    k_conv2d_direct: sum over (c, ky, kx) in the im2col row order of
//           MathOps.Conv2D with a separate multiply and add, padded taps
//           skipped, then the bias pass and the ReLU
//           (src/Lokad.Onnx.Tensors/MathOps.cs:821-872);
//   MaxPool k_maxpool2d: max over the window clipped to the input, from -inf;
//   MatMul  k_gemm_rowdot_smem: sum over k in order, separate multiply and
//           add (MathOps.cs:380-410), then the bias Add node's one rounding;
// so the outputs are bit-identical to the unfused path.  The executor only
// builds such a chain where that path would take these kernels (small
// convs and products, below the tensor-core threshold).
#include "lonnx_internal.cuh"

namespace {

using lonnx::TinyLayer;
using lonnx::TinyProg;

// Phase marks of CTA 0 (clock64: start, set-up done, each layer done),
// compiled only into a diagnostic build (-DLONNX_TINY_TIMELINE); read back
// with lonnx_debug_tiny_timeline.
#ifdef LONNX_TINY_TIMELINE
__device__ long long g_tiny_tl[64];
#define TTL(i)                                                                  \
    do {                                                                        \
        if (blockIdx.x == 0 && threadIdx.x == 0 && (i) < 64) g_tiny_tl[i] = clock64(); \
    } while (0)
#else
#define TTL(i) \
    do {       \
    } while (0)
#endif

// One output's sum over (c, ky, kx) in order, padded taps skipped.  KW
// known at compile time: a row of taps is unrolled (its loads issue
// together), out-of-range taps predicated off -- the same taps in the same
// order as a bounds test per tap.
template <int KW>
__device__ __forceinline__ float conv_sum(const TinyLayer &L, const float *a, const float *wp, int oy, int ox) {
    const int iy0 = oy * L.sh - L.pt, ix0 = ox * L.sw - L.pl;
    const int ky0 = max(0, -iy0), ky1 = min(L.kh, L.H - iy0);
    float acc = 0.0f;
    for (int c = 0; c < L.C; ++c) {
        for (int ky = ky0; ky < ky1; ++ky) {
            const float *xr = a + (c * L.H + iy0 + ky) * L.W + ix0;
            const float *wr = wp + (c * L.kh + ky) * KW;
            float xv[KW], wv[KW];
#pragma unroll
            for (int kx = 0; kx < KW; ++kx) {
                const bool in = ix0 + kx >= 0 && ix0 + kx < L.W;
                xv[kx] = in ? xr[kx] : 0.0f;
                wv[kx] = wr[kx];
            }
#pragma unroll
            for (int kx = 0; kx < KW; ++kx)
                if (ix0 + kx >= 0 && ix0 + kx < L.W) acc = __fadd_rn(acc, __fmul_rn(wv[kx], xv[kx]));
        }
    }
    return acc;
}
__device__ __forceinline__ float conv_sum_any(const TinyLayer &L, const float *a, const float *wp, int oy, int ox) {
    float acc = 0.0f;
    for (int c = 0; c < L.C; ++c) {
        const float *xp = a + c * L.H * L.W;
        for (int ky = 0; ky < L.kh; ++ky) {
            const int iy = oy * L.sh - L.pt + ky * L.dh;
            if (iy < 0 || iy >= L.H) continue;
            for (int kx = 0; kx < L.kw; ++kx) {
                const int ix = ox * L.sw - L.pl + kx * L.dw;
                if (ix < 0 || ix >= L.W) continue;
                acc = __fadd_rn(acc, __fmul_rn(wp[(c * L.kh + ky) * L.kw + kx], xp[iy * L.W + ix]));
            }
        }
    }
    return acc;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t peer_addr(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_peer(uint32_t a, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A cluster of CTAs (16, or 8 where the device allows no wider cluster).
// Every CTA holds all weights and the current activation in its shared
// memory; each layer's outputs are dealt out over all threads of the
// cluster, and each output is stored into every CTA's next-activation buffer
// (distributed shared memory), then a cluster barrier (release / acquire at
// cluster scope) makes the layer visible everywhere.  (Passing activations
// through global memory instead cost ~4k SM cycles per layer in L2 round
// trips across the two dies.)  Every CTA runs every barrier: no thread
// leaves the layer loop early.
__global__ void __launch_bounds__(256, 1) k_tiny_chain(const __grid_constant__ TinyProg p, const float *__restrict__ x,
                                                       float *__restrict__ y) {
    extern __shared__ float sh[];
    float *act[2] = {sh, sh + p.max_elems};  // then every layer's weights at sh + woff
    TTL(0);
    pdl_wait();
    pdl_trigger();
    const int nt = blockDim.x * gridDim.x;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t ncta = gridDim.x;
#pragma unroll 8
    for (int i = threadIdx.x; i < p.in_elems; i += blockDim.x) act[0][i] = __ldg(x + i);
    for (int l = 0; l < p.n; ++l) {  // every layer's weights, once
        const int nw = p.L[l].op == lonnx::TINY_FC ? p.L[l].K * p.L[l].N
                       : p.L[l].op == lonnx::TINY_CONV ? p.L[l].M * p.L[l].C * p.L[l].kh * p.L[l].kw : 0;
        const float *w = p.L[l].w;
        float *d = sh + p.L[l].woff;
#pragma unroll 8
        for (int i = threadIdx.x; i < nw; i += blockDim.x) d[i] = __ldg(w + i);
    }
    __syncthreads();
    cluster_barrier();  // every CTA of the cluster running before any remote store
    TTL(1);
    int cur = 0;
    for (int l = 0; l < p.n; ++l) {
        const TinyLayer L = p.L[l];  // by value: the inner loops read registers, not the parameter
        if (L.op == lonnx::TINY_VIEW) continue;  // a Reshape: the same elements
        const bool last = l == p.n - 1;
        const float *a = act[cur];
        const float *ws = sh + L.woff;
        const uint32_t nxt = smem_addr(act[cur ^ 1]);
        // output t to global (the last layer) or into every CTA's next buffer
        auto put = [&](int t, float v) {
            if (last) {
                y[t] = v;
            } else {
                for (uint32_t r = 0; r < ncta; ++r) st_peer(peer_addr(nxt + 4u * t, r), v);
            }
        };
        if (L.op == lonnx::TINY_CONV) {
            const int total = L.M * L.Ho * L.Wo, hw = L.Ho * L.Wo;
            for (int t = tid; t < total; t += nt) {
                const int m = t / hw, r = t - m * hw, oy = r / L.Wo, ox = r - oy * L.Wo;
                const float *wp = ws + m * L.C * L.kh * L.kw;
                float acc;
                if (L.dh == 1 && L.dw == 1 && L.kw == 5) acc = conv_sum<5>(L, a, wp, oy, ox);
                else if (L.dh == 1 && L.dw == 1 && L.kw == 3) acc = conv_sum<3>(L, a, wp, oy, ox);
                else if (L.dh == 1 && L.dw == 1 && L.kw == 7) acc = conv_sum<7>(L, a, wp, oy, ox);
                else if (L.dh == 1 && L.dw == 1 && L.kw == 1) acc = conv_sum<1>(L, a, wp, oy, ox);
                else acc = conv_sum_any(L, a, wp, oy, ox);
                if (L.bias) acc = __fadd_rn(acc, __ldg(L.bias + m));
                if (L.relu) acc = acc > 0.0f ? acc : 0.0f;
                put(t, acc);
            }
        } else if (L.op == lonnx::TINY_MAXPOOL) {
            const int total = L.C * L.Ho * L.Wo, hw = L.Ho * L.Wo;
            for (int t = tid; t < total; t += nt) {
                const int c = t / hw, r = t - c * hw, oy = r / L.Wo, ox = r - oy * L.Wo;
                const int r0 = oy * L.sh - L.pt, c0 = ox * L.sw - L.pl;
                const float *xp = a + c * L.H * L.W;
                float mx = -INFINITY;
                for (int i = 0; i < L.kh; ++i)
                    for (int j = 0; j < L.kw; ++j) {
                        const int rr = r0 + i, cc = c0 + j;
                        if (rr >= 0 && rr < L.H && cc >= 0 && cc < L.W) mx = fmaxf(mx, xp[rr * L.W + cc]);
                    }
                put(t, mx);
            }
        } else {  // TINY_FC: [1, K] x [K, N] (+ bias)
            for (int n = tid; n < L.N; n += nt) {
                float acc = 0.0f;
                for (int k = 0; k < L.K; ++k) acc = __fadd_rn(acc, __fmul_rn(a[k], ws[k * L.N + n]));
                if (L.bias) acc = __fadd_rn(acc, __ldg(L.bias + n));
                put(n, acc);
            }
        }
        TTL(2 + l);
        if (!last) {
            cluster_barrier();  // the layer in every CTA's buffer; the old one free for reuse
            cur ^= 1;
        }
    }
}

}  // namespace

namespace lonnx {

int tiny_chain(lonnx_ctx *ctx, const TinyProg &p, const float *x, float *y) {
    if (p.n <= 0 || p.n > TINY_MAX_LAYERS || p.max_elems <= 0 || p.smem_floats <= 0 ||
        p.smem_floats > TINY_MAX_SMEM_FLOATS || !x || !y)
        return set_error(LONNX_E_UNSUPPORTED, "tiny_chain: program outside its limits");
    static bool attr_set[64] = {false};
    if (!attr_set[ctx->device & 63]) {
        LONNX_CUDA(cudaFuncSetAttribute(k_tiny_chain, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)(TINY_MAX_SMEM_FLOATS * sizeof(float))));
        attr_set[ctx->device & 63] = true;
    }
    // the widest cluster this device runs (16 CTAs where non-portable sizes
    // are allowed, else 8): each layer's outputs over as many SMs as possible,
    // since every output is one thread's sequential sum
    static int cluster[64] = {0};
    int &cl = cluster[ctx->device & 63];
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t)p.smem_floats * sizeof(float);
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    if (!cl) {
        cl = 8;
        if (cudaFuncSetAttribute(k_tiny_chain, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
            cudaLaunchConfig_t q = cfg;
            q.gridDim = dim3(16);
            q.dynamicSmemBytes = TINY_MAX_SMEM_FLOATS * sizeof(float);
            int n = 0;
            if (cudaOccupancyMaxPotentialClusterSize(&n, k_tiny_chain, &q) == cudaSuccess && n >= 16) cl = 16;
        }
        cudaGetLastError();
    }
    cfg.gridDim = dim3(cl);
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].val.clusterDim.x = cl;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_tiny_chain, p, x, y);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_error(e, "tiny_chain launch");
    return LONNX_OK;
}

}  // namespace lonnx

#ifdef LONNX_TINY_TIMELINE
extern "C" LONNX_API int lonnx_debug_tiny_timeline(long long *host, int n) {
    LONNX_CUDA(cudaMemcpyFromSymbol(host, g_tiny_tl, sizeof(long long) * (n < 64 ? n : 64)));
    return LONNX_OK;
}
#endif
