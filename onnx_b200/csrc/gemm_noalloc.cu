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
//   * the array is only used on the tensor-core path (large, 16-byte aligned
//     operands); the weight-size limit applies there alone, other shapes run
//     on the FFMA kernel with no scratch at all, exactly as lonnx_gemm_f32
//     would route them (LONNX_DISABLE_TC included);
//   * every call looks up the array's device address on the current device
//     (cudaGetSymbolAddress, which allocates nothing); the first call on a
//     device also clears the flag word with a synchronous cudaMemset, so
//     make that first call before any stream capture;
//   * a device-side pipeline wait that expires leaves C incomplete and sets
//     the flag word; the flags are sticky until
//     lonnx_gemm_f32_noalloc_status reads and clears them, so a caller
//     checks a whole sequence of calls with one status query;
//   * cudaDeviceReset reloads the array: call lonnx_gemm_f32_noalloc_status
//     once afterwards to clear the reloaded flag word.
#include <mutex>

#include "lonnx_internal.cuh"

#define LONNX_NOALLOC_MAX_WEIGHT (4ll << 20)  // elements of one [N, K] weight

namespace {

// [0, MAX): weight high parts, [MAX, 2 MAX): low parts, then 64 ints of flags
static __device__ __align__(256) float g_noalloc_scratch[2 * LONNX_NOALLOC_MAX_WEIGHT + 64];

bool g_flags_cleared[64];
std::mutex g_mu;

int *flags_of(float *scratch) { return (int *)(scratch + 2 * LONNX_NOALLOC_MAX_WEIGHT); }

// The array's address on the current device.  Resolved on every call (no
// cached pointer can go stale across a device reset); the flag word is
// cleared synchronously the first time a device is seen.
int scratch_for_current_device(int *device, float **ptr) {
    int dev = 0;
    LONNX_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return lonnx::set_error(LONNX_E_UNSUPPORTED, "device %d out of range", dev);
    float *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void **)&p, g_noalloc_scratch);
    if (e != cudaSuccess) return lonnx::cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_flags_cleared[dev]) {
        e = cudaMemset(flags_of(p), 0, 64 * sizeof(int));
        if (e != cudaSuccess) return lonnx::cuda_error(e, "clearing no-alloc flags");
        g_flags_cleared[dev] = true;
    }
    *device = dev;
    *ptr = p;
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
    c.dev_flags = flags_of(scratch);
    LONNX_CUDA(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, dev));

    // same folding and routing rule as lonnx_gemm_f32 (gemm_dispatch)
    if (batch > 1 && strideB == 0 && strideA == (int64_t)M * K && strideC == (int64_t)M * N &&
        (int64_t)batch * M < (1ll << 31)) {
        M *= batch;
        batch = 1;
    }
    auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    static const bool tc_off = getenv("LONNX_DISABLE_TC") != nullptr;
    const bool tc = !tc_off && K > 0 && (int64_t)M * N * K >= gemm_tc_min_work() && K % 4 == 0 && al16(A) &&
                    al16(B) && strideA % 4 == 0 && strideB % 4 == 0 && (transB || N % 4 == 0);
    if (tc) {
        if ((int64_t)N * K > LONNX_NOALLOC_MAX_WEIGHT)
            return set_error(LONNX_E_BADARG,
                             "gemm_noalloc: weight of %d x %d = %lld elements exceeds the fixed scratch of %lld "
                             "elements (use lonnx_gemm_f32)",
                             N, K, (long long)N * K, (long long)LONNX_NOALLOC_MAX_WEIGHT);
        float *hi = scratch, *lo = scratch + LONNX_NOALLOC_MAX_WEIGHT;
        for (int b = 0; b < batch; ++b) {
            if (b == 0 || strideB != 0) {
                // stream order makes batch b's split wait for batch b-1's GEMM
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

extern "C" LONNX_API int lonnx_gemm_f32_noalloc_status(void *stream) {
    int dev = 0;
    float *scratch = nullptr;
    int rc = scratch_for_current_device(&dev, &scratch);
    if (rc) return rc;
    LONNX_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    int flags[FLAG_COUNT];
    LONNX_CUDA(cudaMemcpy(flags, flags_of(scratch), sizeof(flags), cudaMemcpyDeviceToHost));
    LONNX_CUDA(cudaMemset(flags_of(scratch), 0, sizeof(flags)));
    if (flags[FLAG_TIMEOUT])
        return set_error(LONNX_E_TIMEOUT, "gemm_noalloc: a device-side pipeline wait expired (code %d)",
                         flags[FLAG_TIMEOUT]);
    return LONNX_OK;
}
