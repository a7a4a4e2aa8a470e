// Pre-processing before the model, on the device: the per-pixel and
// per-token work of the reference's data loaders (Lokad.Onnx.Data).
//
// * Images (Images.cs:92-103, ImageToArrayF): decoded RGBA8 pixels ->
//   float [N, 1, H, W], pixel = ((R + G + B) / 3.0f) / 255.0f, two
//   correctly rounded single-precision divisions, as the reference computes
//   it.  The host decodes (and, for MNIST inputs, converts to grayscale and
//   resizes); the batch goes up as bytes, a quarter of the float tensor.
// * Token batches (Text.cs:126-140, RobertaTokenize over a string array):
//   the token ids of B sequences, concatenated, plus B + 1 offsets ->
//   input_ids [B, L] right-padded with the pad id, attention_mask [B, L]
//   (1 on tokens, 0 on padding), token_type_ids [B, L] (zeros).  Only the
//   ragged ids cross PCIe; the three padded tensors are written in HBM.
#include <algorithm>

#include "lonnx_internal.cuh"

namespace {

__global__ void k_rgba_to_gray_f32(const uchar4 *__restrict__ px, float *__restrict__ y, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        const uchar4 p = px[i];
        const int s = (int)p.x + (int)p.y + (int)p.z;
        y[i] = __fdiv_rn(__fdiv_rn((float)s, 3.0f), 255.0f);
    }
}

// one thread per (sequence, position); offsets are non-decreasing
__global__ void k_token_batch_pad(const int64_t *__restrict__ ids, const int64_t *__restrict__ offsets, int64_t B,
                                  int64_t L, int64_t pad_id, int64_t *__restrict__ ids_out,
                                  int64_t *__restrict__ mask_out, int64_t *__restrict__ type_out) {
    const int64_t n = B * L, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t b = i / L, t = i - b * L;
        const int64_t o = __ldg(offsets + b), len = __ldg(offsets + b + 1) - o;
        const bool tok = t < len;
        if (ids_out) ids_out[i] = tok ? __ldg(ids + o + t) : pad_id;
        if (mask_out) mask_out[i] = tok ? 1 : 0;
        if (type_out) type_out[i] = 0;
    }
}

// a grid-stride launch: one thread per element up to 8 blocks per SM
int blocks_for(lonnx_ctx *ctx, int64_t work) {
    const int64_t b = std::min<int64_t>((work + 255) / 256, (int64_t)ctx->num_sms * 8);
    return (int)std::max<int64_t>(b, 1);
}

}  // namespace

using namespace lonnx;

extern "C" {

LONNX_API int lonnx_image_rgba_to_f32(lonnx_ctx *ctx, const void *rgba, float *y, int64_t n_images, int64_t height,
                                      int64_t width) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (n_images < 0 || height < 0 || width < 0) return set_error(LONNX_E_BADARG, "image: negative size");
    const int64_t n = n_images * height * width;
    if (n == 0) return LONNX_OK;
    if (!rgba || !y) return set_error(LONNX_E_BADARG, "image: null pointer");
    if ((uintptr_t)rgba & 3) return set_error(LONNX_E_BADARG, "image: RGBA pixels must be 4-byte aligned");
    k_rgba_to_gray_f32<<<blocks_for(ctx, n), 256, 0, ctx->stream>>>((const uchar4 *)rgba, y, n);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

LONNX_API int lonnx_token_batch_pad(lonnx_ctx *ctx, const int64_t *ids, const int64_t *offsets, int64_t batch,
                                    int64_t max_len, int64_t pad_id, int64_t *ids_out, int64_t *mask_out,
                                    int64_t *type_out) {
    int rc = device_guard(ctx);
    if (rc) return rc;
    if (batch < 0 || max_len < 0) return set_error(LONNX_E_BADARG, "token batch: negative size");
    if (batch == 0 || max_len == 0) return LONNX_OK;
    if (!offsets || (!ids && ids_out)) return set_error(LONNX_E_BADARG, "token batch: null pointer");
    const int64_t n = batch * max_len;
    k_token_batch_pad<<<blocks_for(ctx, n), 256, 0, ctx->stream>>>(ids, offsets, batch, max_len, pad_id, ids_out,
                                                                 mask_out, type_out);
    LONNX_CHECK_LAUNCH(ctx);
    return LONNX_OK;
}

}  // extern "C"
