/*
 * lonnx.h -- C ABI of liblonnx_cuda.so, the B200 (sm_100a) implementation of
 * Lokad.Onnx's float32 inference hot path.
 *
 * Plain C types only: pointers, sizes, int64 shapes.  Every entry point
 * returns 0 (LONNX_OK) or a negative LONNX_E_* code; the message of the last
 * failure on the calling thread is returned by lonnx_last_error().  A caller
 * maps a non-zero code to OpResult.Failure(op, lonnx_last_error())
 * (src/Lokad.Onnx.Backend/OpResult.cs:34-62) -- no entry point throws.
 *
 * Execution model: one lonnx_ctx per GPU = one device, one non-default CUDA
 * stream, one caching device allocator.  Op entry points only enqueue work on
 * the context's stream (device pointers in, device pointers out);
 * lonnx_sync() waits for it and reports errors the kernels flagged on the
 * device (out-of-range Gather index, bounded pipeline wait that expired).
 * A context is driven by one host thread at a time; contexts on different
 * GPUs are independent (batch sharding needs no collective).
 *
 * Each op cites the reference routine it replaces (paths inside the
 * Lokad/Onnx project).
 */
#ifndef LONNX_H
#define LONNX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LONNX_API __attribute__((visibility("default")))

enum lonnx_status {
    LONNX_OK = 0,
    LONNX_E_BADARG = -1,      /* null pointer, bad enum, bad attribute value     */
    LONNX_E_SHAPE = -2,       /* shapes incompatible (broadcast, matmul, conv)   */
    LONNX_E_OOM = -3,         /* device allocation failed or hit LONNX_MEM_LIMIT */
    LONNX_E_CUDA = -4,        /* CUDA runtime error                              */
    LONNX_E_TIMEOUT = -5,     /* a device-side bounded wait expired              */
    LONNX_E_OOB = -6,         /* a Gather index outside [-dim, dim)              */
    LONNX_E_UNSUPPORTED = -7  /* op/dtype/attribute not supported                */
};

enum lonnx_binary_op { LONNX_ADD = 0, LONNX_SUB = 1, LONNX_MUL = 2, LONNX_DIV = 3, LONNX_POW = 4 };
enum lonnx_unary_op { LONNX_RELU = 0, LONNX_SQRT = 1, LONNX_ERF = 2, LONNX_EXP = 3, LONNX_GELU_ERF = 4 };
enum lonnx_reduce_op { LONNX_REDUCE_SUM = 0, LONNX_REDUCE_MAX = 1, LONNX_REDUCE_MEAN = 2 };
enum lonnx_epilogue { LONNX_EPI_NONE = 0, LONNX_EPI_RELU = 1, LONNX_EPI_GELU_ERF = 2 };

typedef struct lonnx_ctx lonnx_ctx;

/* ---- runtime -------------------------------------------------------------
 * Replaces the reference's managed storage (DenseTensor<T> over Memory<T>,
 * src/Lokad.Onnx.Tensors/DenseTensor.cs:31-42) with device-resident buffers. */
LONNX_API int lonnx_ctx_create(int device, lonnx_ctx **out);
LONNX_API int lonnx_ctx_destroy(lonnx_ctx *ctx);
LONNX_API int lonnx_ctx_device(const lonnx_ctx *ctx);
LONNX_API void *lonnx_ctx_stream(lonnx_ctx *ctx); /* the cudaStream_t */
LONNX_API int lonnx_malloc(lonnx_ctx *ctx, size_t bytes, void **out);
LONNX_API int lonnx_free(lonnx_ctx *ctx, void *ptr);
LONNX_API int lonnx_memcpy_h2d(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes);
LONNX_API int lonnx_memcpy_d2h(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes);
LONNX_API int lonnx_memcpy_d2d(lonnx_ctx *ctx, void *dst, const void *src, size_t bytes);
LONNX_API int lonnx_memset(lonnx_ctx *ctx, void *dst, int value, size_t bytes);
LONNX_API int lonnx_sync(lonnx_ctx *ctx);
LONNX_API const char *lonnx_last_error(void);
/* Failure-detection test hook: enqueue a kernel whose bounded device wait
 * (on a word nothing sets) expires after `cycles` SM clocks; the next
 * lonnx_sync() returns LONNX_E_TIMEOUT and the context stays usable.  Same
 * reporting path as an expired pipeline wait in the tensor-core kernels. */
LONNX_API int lonnx_debug_expire_wait(lonnx_ctx *ctx, int64_t cycles);
/* Count of this library's kernel launches on ctx since creation. */
LONNX_API int64_t lonnx_launch_count(const lonnx_ctx *ctx);

/* ---- element-wise ----------------------------------------------------------
 * Add/Sub/Mul/Div/Pow with numpy broadcasting (rank <= 8): replaces
 * CPUExecutionProvider.Add..Pow (src/Lokad.Onnx.Backend/CPUExecutionProvider.cs:82-236),
 * ITensor.Broadcast (src/Lokad.Onnx.Tensors/ITensor.cs:64-137) and
 * Tensor<float>.VectorizedApply (src/Lokad.Onnx.Tensors/TensorOps.cs:36-123).
 * y has the broadcast shape (see lonnx_broadcast_shape). */
LONNX_API int lonnx_broadcast_shape(const int64_t *a_shape, int a_rank, const int64_t *b_shape,
                                    int b_rank, int64_t *out_shape, int *out_rank);
LONNX_API int lonnx_binary_f32(lonnx_ctx *ctx, int op, const float *a, const int64_t *a_shape,
                               int a_rank, const float *b, const int64_t *b_shape, int b_rank,
                               float *y);
/* Relu/Sqrt/Erf/Exp and the fused GELU 0.5*x*(1+erf(x/sqrt 2)): replaces
 * Tensor<float>.Relu/Sqrt/Erf (TensorOps.cs:1252,315,1353; MathOps.cs:989-1010). */
LONNX_API int lonnx_unary_f32(lonnx_ctx *ctx, int op, const float *x, float *y, int64_t n);

/* Inference BatchNormalization over axis 1 of an [outer, channels, inner]
 * tensor: y = (x - mean[c]) / sqrt(var[c] + eps) * scale[c] + bias[c], each
 * step rounded once in that order (ONNX BatchNormalization, opset 15).  The
 * reference names the op (src/Lokad.Onnx.Base/OpType.cs:17) but has no
 * implementation (CPUExecutionProvider.cs:24-50). */
LONNX_API int lonnx_batchnorm_f32(lonnx_ctx *ctx, const float *x, const float *scale, const float *bias,
                                  const float *mean, const float *var, float eps, float *y, int64_t outer,
                                  int64_t channels, int64_t inner);

/* ---- contractions ----------------------------------------------------------
 * C[b] = alpha * A[b] . op(B[b]) + beta * bias, then the epilogue.
 * A[b]: M x K row-major at A + b*strideA; B[b]: K x N (transB = 0) or N x K
 * (transB = 1) at B + b*strideB; C[b]: M x N at C + b*strideC; bias: N floats
 * or NULL.  fp32 in/out; large shapes run on tcgen05 tensor cores with a
 * 3xTF32 split, small or unaligned ones on an fp32 FFMA kernel.
 * Replaces MathOps.mm_unsafe_vectorized (src/Lokad.Onnx.Tensors/MathOps.cs:380-410)
 * behind Tensor<float>.MatMul2D/MatMul (TensorOps.cs:356-407,600-704) plus
 * the following bias Add node. */
LONNX_API int lonnx_gemm_f32(lonnx_ctx *ctx, const float *A, const float *B, const float *bias,
                             float *C, int batch, int M, int N, int K, int64_t strideA,
                             int64_t strideB, int64_t strideC, int transB, float alpha,
                             float beta, int epilogue);
/* lonnx_gemm_f32 without any device allocation, for callers that cannot
 * allocate device memory (a host callback or a plugin inside a runtime that
 * owns the whole device pool, or code with no lonnx_ctx).  No counterpart in
 * the reference.  Work goes on `stream` (a cudaStream_t) of the current
 * device and is routed exactly as lonnx_gemm_f32 routes it.  Only the
 * tensor-core path needs scratch: there the weight split uses a fixed 32 MiB
 * file-scope device array, so N * K must be <= 4194304 (else
 * LONNX_E_BADARG); the FFMA path (small, unaligned or LONNX_DISABLE_TC) has
 * no limit.  All calls on a device share that array: calls that overlap on
 * the GPU race.  The first call on a device clears the array's flag word
 * synchronously; make it before any stream capture.  Expired device-side
 * waits are recorded in sticky flags: read them with
 * lonnx_gemm_f32_noalloc_status. */
LONNX_API int lonnx_gemm_f32_noalloc(void *stream, const float *A, const float *B, const float *bias,
                                     float *C, int batch, int M, int N, int K, int64_t strideA,
                                     int64_t strideB, int64_t strideC, int transB, float alpha,
                                     float beta, int epilogue);
/* Status of the lonnx_gemm_f32_noalloc calls on the current device since the
 * last query: synchronises `stream`, reads and clears the shared flag word,
 * and returns LONNX_E_TIMEOUT if any call's device-side pipeline wait
 * expired (its C is then incomplete), else LONNX_OK.  Allocates nothing.  No
 * counterpart in the reference. */
LONNX_API int lonnx_gemm_f32_noalloc_status(void *stream);
/* ONNX MatMul with numpy batch broadcasting on the leading dimensions
 * (Tensor<float>.MatMul, TensorOps.cs:600-704).  y has shape
 * broadcast(a[:-2], b[:-2]) + [a[-2], b[-1]]. */
LONNX_API int lonnx_matmul_f32(lonnx_ctx *ctx, const float *a, const int64_t *a_shape, int a_rank,
                               const float *b, const int64_t *b_shape, int b_rank, float *y);
/* NCHW 2-D convolution with explicit pads (top, left, bottom, right), groups,
 * optional bias and fused ReLU: replaces Tensor<float>.Conv2D ->
 * MathOps.Im2col + Conv2D (TensorOps.cs:903-962, MathOps.cs:654-877).
 * y: [N, M, Ho, Wo] with Ho = (H + pt + pb - (dh*(kh-1)+1)) / sh + 1. */
LONNX_API int lonnx_conv2d_f32(lonnx_ctx *ctx, const float *x, const float *w, const float *bias,
                               float *y, int N, int C, int H, int W, int M, int kh, int kw,
                               int sh, int sw, int pt, int pl, int pb, int pr, int dh, int dw,
                               int group, int relu);

/* ---- row kernels -----------------------------------------------------------
 * Softmax over the middle axis of an [outer, len, inner] view: replaces
 * Tensor<float>.Softmax (TensorOps.cs:1312-1330). */
LONNX_API int lonnx_softmax_f32(lonnx_ctx *ctx, const float *x, float *y, int64_t outer,
                                int64_t len, int64_t inner);
/* Row LayerNorm y = (x+res - mean) / sqrt(var + eps) * gamma + beta over the
 * last axis (cols), res nullable: replaces the ReduceMean -> Sub -> Pow ->
 * ReduceMean -> Add -> Sqrt -> Div -> Mul -> Add node chain
 * (TensorOps.cs:1735-1760,259,303,315,291). */
LONNX_API int lonnx_layernorm_f32(lonnx_ctx *ctx, const float *x, const float *res,
                                  const float *gamma, const float *beta, float eps, float *y,
                                  int64_t rows, int cols);
/* ReduceSum/Max/Mean over any axes (keepdims only affects the caller's view
 * of y's shape): replaces TensorOps.cs:1610-1839. */
LONNX_API int lonnx_reduce_f32(lonnx_ctx *ctx, int op, const float *x, const int64_t *shape,
                               int rank, const int64_t *axes, int naxes, float *y);
/* MaxPool2D: replaces Tensor<float>.MaxPool2D (TensorOps.cs:1025-1099). */
LONNX_API int lonnx_maxpool2d_f32(lonnx_ctx *ctx, const float *x, float *y, int N, int C, int H,
                                  int W, int kh, int kw, int sh, int sw, int pt, int pl, int Ho,
                                  int Wo);

/* ---- data movement ---------------------------------------------------------
 * Gather along axis with int64 indices (negative indices wrap once): replaces
 * Tensor<T>.Gather (TensorOps.cs:1410-1446).  data: [outer, dim, inner] view
 * of elem_bytes-sized elements; y: [outer, n_idx, inner].  An index outside
 * [-dim, dim) writes zeros for that row and makes the next lonnx_sync()
 * return LONNX_E_OOB. */
LONNX_API int lonnx_gather(lonnx_ctx *ctx, const void *data, int elem_bytes, int64_t outer,
                           int64_t dim, int64_t inner, const int64_t *idx, int64_t n_idx,
                           void *y);
/* Transpose (rank <= 8): replaces Tensor<T>.Transpose (TensorOps.cs:1358-1407). */
LONNX_API int lonnx_transpose(lonnx_ctx *ctx, const void *x, int elem_bytes,
                              const int64_t *shape, int rank, const int64_t *perm, void *y);
/* Cast int64 -> float32 element-wise (CPUExecutionProvider.Cast, :451). */
LONNX_API int lonnx_cast_i64_f32(lonnx_ctx *ctx, const int64_t *x, float *y, int64_t n);

/* ---- pre-processing before the model -------------------------------------
 * Decoded RGBA8 images [n_images, height, width, 4] (device, 4-byte aligned)
 * -> float [n_images, 1, height, width], pixel = ((R + G + B) / 3.0f) / 255.0f
 * with IEEE single divisions: replaces Images.ImageToArrayF
 * (src/Lokad.Onnx.Data/Images.cs:92-103) after the host has decoded the
 * file (and, for MNIST inputs, made it grayscale and resized it to 28 x 28,
 * Images.cs:166-183). */
LONNX_API int lonnx_image_rgba_to_f32(lonnx_ctx *ctx, const void *rgba, float *y, int64_t n_images,
                                      int64_t height, int64_t width);
/* Token batch: the token ids of `batch` sequences concatenated in `ids`
 * (device), sequence b at [offsets[b], offsets[b + 1]) (device, batch + 1
 * entries) -> input_ids [batch, max_len] right-padded with pad_id,
 * attention_mask [batch, max_len] (1 on tokens, 0 on padding) and
 * token_type_ids [batch, max_len] (0); any output may be NULL; tokens past
 * max_len are dropped.  Replaces the padding loop of Text.RobertaTokenize
 * over a string array (src/Lokad.Onnx.Data/Text.cs:126-140), which pads
 * input_ids with 1 and the other two with 0 up to the longest sequence. */
LONNX_API int lonnx_token_batch_pad(lonnx_ctx *ctx, const int64_t *ids, const int64_t *offsets, int64_t batch,
                                    int64_t max_len, int64_t pad_id, int64_t *ids_out, int64_t *mask_out,
                                    int64_t *type_out);

/* ---- fused encoder ops -------------------------------------------------------
 * Scaled-dot-product attention of one BERT layer, fused: for each batch b and
 * head h, softmax(Q K^T / scale + maskadd[b]) V, with Q, K, V read in place
 * from [B, S, ld] row-major projections (head h at column offset h*dh) and the
 * context written to out [B, S, heads*dh].  maskadd: [B, S] additive mask or
 * NULL.  Replaces the MatMul -> Div -> Add -> Softmax -> MatMul node chain and
 * the Transpose nodes around it (TensorOps.cs:600-704,1312-1330,1358-1407). */
LONNX_API int lonnx_attention_f32(lonnx_ctx *ctx, const float *q, const float *k, const float *v,
                                  int64_t ld_qkv, const float *maskadd, float *out, int B, int S,
                                  int heads, int dh, float scale);

/* ---- graph executor ----------------------------------------------------------
 * Native mirror of ComputationalGraph (src/Lokad.Onnx.Backend/ComputationalGraph.cs:199-336):
 * nodes in file order with name-resolved tensors; float activations stay on
 * the device; a prepare step fuses node chains into the kernels above.
 * dtype codes follow ONNX TensorProto (1 float, 7 int64). */
typedef struct lonnx_graph lonnx_graph;
LONNX_API int lonnx_graph_create(lonnx_ctx *ctx, lonnx_graph **out);
LONNX_API int lonnx_graph_destroy(lonnx_graph *g);
LONNX_API int lonnx_graph_add_initializer(lonnx_graph *g, const char *name, int dtype,
                                          const int64_t *shape, int rank, const void *host_data);
LONNX_API int lonnx_graph_add_node(lonnx_graph *g, const char *op, const char *const *inputs,
                                   int n_in, const char *const *outputs, int n_out);
/* Attributes of the last added node. */
LONNX_API int lonnx_graph_attr_int(lonnx_graph *g, const char *name, int64_t v);
LONNX_API int lonnx_graph_attr_ints(lonnx_graph *g, const char *name, const int64_t *v, int n);
LONNX_API int lonnx_graph_attr_float(lonnx_graph *g, const char *name, float v);
LONNX_API int lonnx_graph_attr_string(lonnx_graph *g, const char *name, const char *v);
LONNX_API int lonnx_graph_attr_floats(lonnx_graph *g, const char *name, const float *v, int n);
/* A tensor-valued attribute (ONNX AttributeProto TENSOR, e.g. Constant's
 * `value`); the data is copied. */
LONNX_API int lonnx_graph_attr_tensor(lonnx_graph *g, const char *name, int dtype, const int64_t *shape,
                                      int rank, const void *data);
LONNX_API int lonnx_graph_add_output(lonnx_graph *g, const char *name);
/* Opset of the model (selects attribute vs input forms, Node.cs:164-174). */
LONNX_API int lonnx_graph_set_opset(lonnx_graph *g, int opset);
/* Call once after the last node.  flags & 1: pattern fusion (GEMM + bias
 * [+ GELU], packed QKV, attention, LayerNorm) with weight re-layout;
 * flags & 2: honour Conv's strides/pads/dilations/group attributes (the
 * reference ignores them, Node.cs:137-138). */
LONNX_API int lonnx_graph_prepare(lonnx_graph *g, int flags);
/* Stage an input: host data copied into device memory on the ctx stream. */
LONNX_API int lonnx_graph_set_input(lonnx_graph *g, const char *name, int dtype,
                                    const int64_t *shape, int rank, const void *host_data);
/* Same, from a device pointer the caller owns (no copy; must outlive execute). */
LONNX_API int lonnx_graph_set_input_device(lonnx_graph *g, const char *name, int dtype,
                                           const int64_t *shape, int rank, const void *dev_data);
LONNX_API int lonnx_graph_execute(lonnx_graph *g);
/* Shape of an output after execute: rank and dims (up to 8). */
LONNX_API int lonnx_graph_output_shape(lonnx_graph *g, const char *name, int64_t *shape,
                                       int *rank);
/* Element type (ONNX TensorProto code) of an output after execute. */
LONNX_API int lonnx_graph_output_dtype(lonnx_graph *g, const char *name, int *dtype);
LONNX_API int lonnx_graph_output_device(lonnx_graph *g, const char *name, const void **dev);
/* Copy an output to host memory (bytes must equal the output's size). */
LONNX_API int lonnx_graph_get_output(lonnx_graph *g, const char *name, void *host, size_t bytes);
/* Release intermediates back to the allocator (ComputationalGraph.Reset, :336-349). */
LONNX_API int lonnx_graph_reset(lonnx_graph *g);
/* Record one execution (inputs already set, shapes then fixed) as a CUDA
 * graph; lonnx_graph_replay re-runs it with one launch.  Buffers used by the
 * captured execution stay reserved for the graph until the next capture,
 * lonnx_graph_reset or lonnx_graph_destroy; device inputs must stay at the
 * same addresses (update their contents in place between replays). */
LONNX_API int lonnx_graph_capture(lonnx_graph *g);
LONNX_API int lonnx_graph_replay(lonnx_graph *g);
/* Nodes after fusion (kernels launched per execute, for reporting). */
LONNX_API int lonnx_graph_num_steps(lonnx_graph *g);

#ifdef __cplusplus
}
#endif
#endif /* LONNX_H */
