// Context, caching device allocator, copies, synchronisation and error
// reporting of the C ABI (include/lonnx.h).
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include "lonnx_internal.cuh"

namespace lonnx {

bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("LONNX_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

}  // namespace lonnx

namespace lonnx {

static thread_local std::string g_last_error;

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_error(cudaError_t e, const char *what) {
    return set_error(LONNX_E_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int device_guard(lonnx_ctx *ctx) {
    if (!ctx) return set_error(LONNX_E_BADARG, "null context");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ctx->device) LONNX_CUDA(cudaSetDevice(ctx->device));
    return LONNX_OK;
}

static size_t round_size(size_t b) {
    // 512-byte granularity below 1 MiB, 64 KiB above: keeps reuse high for
    // the few distinct activation sizes of a graph without much waste.
    if (b == 0) b = 1;
    const size_t g = b < (1u << 20) ? 512 : (64u << 10);
    return (b + g - 1) / g * g;
}

int ctx_alloc(lonnx_ctx *ctx, size_t bytes, void **out) {
    Allocator &A = ctx->alloc;
    const size_t sz = round_size(bytes);
    auto it = A.free_blocks.find(sz);
    if (it != A.free_blocks.end()) {
        *out = it->second;
        A.free_blocks.erase(it);
        A.live[*out] = sz;
        return LONNX_OK;
    }
    if (A.limit && A.bytes_reserved + sz > A.limit)
        return set_error(LONNX_E_OOM, "allocation of %zu bytes exceeds LONNX_MEM_LIMIT (%zu reserved)",
                         bytes, A.bytes_reserved);
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, sz);
    if (e != cudaSuccess) {
        cudaGetLastError();
        // release cached blocks and retry once
        cudaStreamSynchronize(ctx->stream);
        for (auto &kv : A.free_blocks) {
            cudaFree(kv.second);
            A.bytes_reserved -= kv.first;
        }
        A.free_blocks.clear();
        e = cudaMalloc(&p, sz);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(LONNX_E_OOM, "cudaMalloc(%zu) failed: %s", sz, cudaGetErrorString(e));
        }
    }
    A.bytes_reserved += sz;
    A.live[p] = sz;
    *out = p;
    return LONNX_OK;
}

int ctx_free(lonnx_ctx *ctx, void *p) {
    if (!p) return LONNX_OK;
    Allocator &A = ctx->alloc;
    auto it = A.live.find(p);
    if (it == A.live.end()) return set_error(LONNX_E_BADARG, "lonnx_free: pointer %p not allocated by this context", p);
    if (ctx->capturing) {
        ctx->capture_hold.push_back(p);  // stays live until the captured graph is released
        return LONNX_OK;
    }
    A.free_blocks.emplace(it->second, p);
    A.live.erase(it);
    return LONNX_OK;
}

int ctx_scratch(lonnx_ctx *ctx, size_t bytes, void **out) {
    if (bytes > ctx->scratch_bytes) {
        if (ctx->scratch) {
            // the old scratch may still be read by queued kernels
            LONNX_CUDA(cudaStreamSynchronize(ctx->stream));
            ctx_free(ctx, ctx->scratch);
            ctx->scratch = nullptr;
            ctx->scratch_bytes = 0;
        }
        int rc = ctx_alloc(ctx, bytes, &ctx->scratch);
        if (rc) return rc;
        ctx->scratch_bytes = bytes;
    }
    *out = ctx->scratch;
    return LONNX_OK;
}

int ctx_scratch2(lonnx_ctx *ctx, size_t bytes, void **out) {
    if (bytes > ctx->scratch2_bytes) {
        if (ctx->scratch2) {
            LONNX_CUDA(cudaStreamSynchronize(ctx->stream));
            ctx_free(ctx, ctx->scratch2);
            ctx->scratch2 = nullptr;
            ctx->scratch2_bytes = 0;
        }
        int rc = ctx_alloc(ctx, bytes, &ctx->scratch2);
        if (rc) return rc;
        ctx->scratch2_bytes = bytes;
    }
    *out = ctx->scratch2;
    return LONNX_OK;
}

}  // namespace lonnx

using namespace lonnx;

extern "C" {

LONNX_API const char *lonnx_last_error(void) { return g_last_error.c_str(); }

LONNX_API int lonnx_ctx_create(int device, lonnx_ctx **out) {
    if (!out) return set_error(LONNX_E_BADARG, "null output pointer");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(LONNX_E_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
    }
    if (device < 0 || device >= n) return set_error(LONNX_E_BADARG, "device %d out of range [0,%d)", device, n);
    LONNX_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    LONNX_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return set_error(LONNX_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)",
                         device, prop.major, prop.minor);
    lonnx_ctx *c = new lonnx_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if (const char *lim = getenv("LONNX_MEM_LIMIT")) c->alloc.limit = strtoull(lim, nullptr, 10);
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_error(e, "cudaStreamCreate");
    }
    e = cudaMalloc(&c->dev_flags, sizeof(int) * FLAG_COUNT);
    if (e == cudaSuccess) e = cudaMemset(c->dev_flags, 0, sizeof(int) * FLAG_COUNT);
    if (e != cudaSuccess) {
        cudaStreamDestroy(c->stream);
        delete c;
        return cuda_error(e, "cudaMalloc(flags)");
    }
    *out = c;
    return LONNX_OK;
}

LONNX_API int lonnx_ctx_destroy(lonnx_ctx *ctx) {
    if (!ctx) return LONNX_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto &kv : ctx->alloc.free_blocks) cudaFree(kv.second);
    for (auto &kv : ctx->alloc.live) cudaFree(kv.first);
    cudaFree(ctx->dev_flags);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return LONNX_OK;
}

LONNX_API int lonnx_ctx_device(const lonnx_ctx *ctx) { return ctx ? ctx->device : -1; }
LONNX_API void *lonnx_ctx_stream(lonnx_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }
LONNX_API int64_t lonnx_launch_count(const lonnx_ctx *ctx) { return ctx ? ctx->launches : 0; }

LONNX_API int lonnx_malloc(lonnx_ctx *ctx, size_t bytes, void **out) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (!out) return set_error(LONNX_E_BADARG, "null output pointer");
    return ctx_alloc(ctx, bytes, out);
}

LONNX_API int lonnx_free(lonnx_ctx *ctx, void *p) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    return ctx_free(ctx, p);
}

LONNX_API int lonnx_memcpy_h2d(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (bytes == 0) return LONNX_OK;
    if (!dst || !src) return set_error(LONNX_E_BADARG, "null pointer");
    LONNX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return LONNX_OK;
}

LONNX_API int lonnx_memcpy_d2h(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (bytes == 0) return LONNX_OK;
    if (!dst || !src) return set_error(LONNX_E_BADARG, "null pointer");
    LONNX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    LONNX_CUDA(cudaStreamSynchronize(ctx->stream));
    return LONNX_OK;
}

LONNX_API int lonnx_memcpy_d2d(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (bytes == 0) return LONNX_OK;
    if (!dst || !src) return set_error(LONNX_E_BADARG, "null pointer");
    LONNX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    return LONNX_OK;
}

LONNX_API int lonnx_memset(lonnx_ctx *ctx, void *dst, int value, size_t bytes) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (bytes == 0) return LONNX_OK;
    LONNX_CUDA(cudaMemsetAsync(dst, value, bytes, ctx->stream));
    return LONNX_OK;
}

LONNX_API int lonnx_sync(lonnx_ctx *ctx) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    LONNX_CUDA(cudaStreamSynchronize(ctx->stream));
    int flags[FLAG_COUNT];
    LONNX_CUDA(cudaMemcpy(flags, ctx->dev_flags, sizeof(flags), cudaMemcpyDeviceToHost));
    if (flags[FLAG_OOB] || flags[FLAG_TIMEOUT]) {
        LONNX_CUDA(cudaMemset(ctx->dev_flags, 0, sizeof(flags)));
        if (flags[FLAG_TIMEOUT])
            return set_error(LONNX_E_TIMEOUT, "a device-side pipeline wait expired (code %d)", flags[FLAG_TIMEOUT]);
        return set_error(LONNX_E_OOB, "Gather: an index was outside the bounds of the data axis");
    }
    return LONNX_OK;
}

// Test hook for failure detection: one thread waits on a device word that
// nothing sets, gives up after `cycles` SM clocks (a bounded wait, like every
// pipeline wait in this library), records LONNX_E_TIMEOUT in the context's
// flags and returns.  The kernel always terminates; the context stays usable.
static __global__ void k_expire_wait(const volatile int *never, int *flags, long long cycles) {
    const long long t0 = clock64();
    while (*never == 0) {
        if (clock64() - t0 > cycles) {
            atomicExch(flags + lonnx::FLAG_TIMEOUT, 2);
            return;
        }
    }
}

LONNX_API int lonnx_debug_expire_wait(lonnx_ctx *ctx, int64_t cycles) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (cycles <= 0 || cycles > 4000000000ll) return set_error(LONNX_E_BADARG, "cycles out of range");
    // flags[FLAG_COUNT-1] is never written by the library: the word nothing sets
    k_expire_wait<<<1, 1, 0, ctx->stream>>>(ctx->dev_flags + FLAG_COUNT - 1, ctx->dev_flags, cycles);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // extern "C"
