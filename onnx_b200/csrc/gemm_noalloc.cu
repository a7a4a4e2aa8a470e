// lonnx_gemm_f32_noalloc: the fp32 GEMM of lonnx_gemm_f32 for callers that
// cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a
// host callback or a plugin hook of another runtime that owns all device
// memory (its pool is fixed up front, so a stray cudaMalloc either fails or
// fragments that pool), or a caller with no lonnx_ctx (creating a context
// allocates its stream and flags).  Such a caller still owns the inputs and
// the output; what lonnx_gemm_f32 allocates on its own is the scratch that
// holds the weight operand split into tf32 high/low parts for the tensor
// cores.  Here that scratch is a fixed, file-scope device array instead.
//
// Limits and sharing:
//   * the array holds one split weight of at most LONNX_NOALLOC_MAX_WEIGHT
//     elements (N * K); larger weights are rejected with LONNX_E_BADARG;
//   * it is 32 MiB + 256 bytes of device memory on every GPU that loads this
//     library, held until the process exits;
//   * every call on a device uses the same array and leaves its contents
//     behind: calls that overlap on the GPU (different streams, or host
//     threads racing on one device) corrupt each other's operands -- order
//     them on one stream or serialise them;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) and clears its flag word; make that first call
//     before any stream capture;
//   * a device-side pipeline wait that expires is recorded in the array's
//     flag word, which this entry point clears and does not report.
#include <mutex>

#include "lonnx_internal.cuh"

#define LONNX_NOALLOC_MAX_WEIGHT (4ll << 20)  // elements of one [N, K] weight

namespace {

// [0, MAX): weight high parts, [MAX, 2 MAX): low parts, then 64 ints of flags
static __device__ __align__(256) float g_noalloc_scratch[2 * LONNX_NOALLOC_MAX_WEIGHT + 64];

struct DevScratch {
    float *ptr = nullptr;
};
DevScratch g_dev[64];
std::mutex g_mu;

int scratch_for_current_device(int *device, float **ptr) {
    int dev = 0;
    LONNX_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return lonnx::set_error(LONNX_E_UNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev[dev].ptr) {
        float *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void **)&p, g_noalloc_scratch);
        if (e != cudaSuccess) return lonnx::cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
        e = cudaMemset(p + 2 * LONNX_NOALLOC_MAX_WEIGHT, 0, 64 * sizeof(int));
        if (e != cudaSuccess) return lonnx::cuda_error(e, "clearing no-alloc flags");
        g_dev[dev].ptr = p;
    }
    *device = dev;
    *ptr = g_dev[dev].ptr;
    return LONNX_OK;
}

}  // namespace

using namespace lonnx;

extern "C" LONNX_API int lonnx_gemm_f32_noalloc(void *stream, const float *A, const float *B, const float *bias,
                                                float *C, int batch, int M, int N, int K, int64_t strideA,
                                                int64_t strideB, int64_t strideC, int transB, float alpha,
                                                float beta, int epilogue) {
    if (!A || !B || !C || batch < 0 || M < 0 || N < 0 || K < 0 || epilogue < 0 || epilogue > 2)
        return set_error(LONNX_E_BADARG, "gemm_noalloc: bad arguments");
    if ((int64_t)N * K > LONNX_NOALLOC_MAX_WEIGHT)
        return set_error(LONNX_E_BADARG,
                         "gemm_noalloc: weight of %d x %d = %lld elements exceeds the fixed scratch of %lld elements "
                         "(use lonnx_gemm_f32)",
                         N, K, (long long)N * K, (long long)LONNX_NOALLOC_MAX_WEIGHT);
    int dev = 0;
    float *scratch = nullptr;
    int rc = scratch_for_current_device(&dev, &scratch);
    if (rc) return rc;
    if (M == 0 || N == 0 || batch == 0) return LONNX_OK;

    // a context on the stack: the caller's stream, flags inside the static
    // array, no allocator use on this path
    lonnx_ctx c;
    c.device = dev;
    c.stream = (cudaStream_t)stream;
    c.dev_flags = (int *)(scratch + 2 * LONNX_NOALLOC_MAX_WEIGHT);
    LONNX_CUDA(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, dev));
    LONNX_CUDA(cudaMemsetAsync(c.dev_flags, 0, 4 * sizeof(int), c.stream));

    // same folding and dispatch rule as lonnx_gemm_f32
    if (batch > 1 && strideB == 0 && strideA == (int64_t)M * K && strideC == (int64_t)M * N &&
        (int64_t)batch * M < (1ll << 31)) {
        M *= batch;
        batch = 1;
    }
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    const bool tc = K > 0 && (int64_t)M * N * K >= gemm_tc_min_work() && K % 4 == 0 && al16(A) && al16(B) &&
                    strideA % 4 == 0 && strideB % 4 == 0 && (transB || N % 4 == 0);
    if (tc) {
        float *hi = scratch, *lo = scratch + LONNX_NOALLOC_MAX_WEIGHT;
        for (int b = 0; b < batch; ++b) {
            if (b == 0 || strideB != 0) {
                rc = split_tf32_nk(&c, B + b * strideB, hi, lo, K, N, transB);
                if (rc) return rc;
            }
            rc = gemm_tc(&c, A + b * strideA, hi, lo, bias, C + b * strideC, M, N, K, K, K, N, alpha, beta, epilogue,
                         /*allow_scratch=*/false);
            if (rc == LONNX_E_UNSUPPORTED && b == 0) break;
            if (rc) return rc;
            if (b == batch - 1) return LONNX_OK;
        }
    }
    return gemm_simt(&c, A, B, bias, C, batch, M, N, K, strideA, strideB, strideC, transB, alpha, beta, epilogue,
                     nullptr);
}
