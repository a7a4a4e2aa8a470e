// P/Invoke declarations of liblonnx_cuda.so: one [DllImport] per entry point
// of include/lonnx.h, same names, same argument order.  A CPU test in the
// repository (tests/test_host.py::test_csharp_pinvoke_matches_header) parses
// this file against the header so the two cannot drift apart.
//
// Add this file to src/Lokad.Onnx.Backend (AllowUnsafeBlocks=true) and ship
// liblonnx_cuda.so next to the assembly.
namespace Lokad.Onnx.Cuda;

using System;
using System.Runtime.InteropServices;

internal static unsafe class Native
{
    const string Lib = "lonnx_cuda";

    // ---- status codes (enum lonnx_status) ----
    public const int LONNX_OK = 0, LONNX_E_BADARG = -1, LONNX_E_SHAPE = -2, LONNX_E_OOM = -3, LONNX_E_CUDA = -4,
        LONNX_E_TIMEOUT = -5, LONNX_E_OOB = -6, LONNX_E_UNSUPPORTED = -7;
    public const int ADD = 0, SUB = 1, MUL = 2, DIV = 3, POW = 4;
    public const int RELU = 0, SQRT = 1, ERF = 2, EXP = 3, GELU_ERF = 4;
    public const int REDUCE_SUM = 0, REDUCE_MAX = 1, REDUCE_MEAN = 2;

    // ---- runtime ----
    [DllImport(Lib)] public static extern int lonnx_ctx_create(int device, out IntPtr ctx);
    [DllImport(Lib)] public static extern int lonnx_ctx_destroy(IntPtr ctx);
    [DllImport(Lib)] public static extern int lonnx_ctx_device(IntPtr ctx);
    [DllImport(Lib)] public static extern IntPtr lonnx_ctx_stream(IntPtr ctx);
    [DllImport(Lib)] public static extern int lonnx_malloc(IntPtr ctx, nuint bytes, out IntPtr p);
    [DllImport(Lib)] public static extern int lonnx_free(IntPtr ctx, IntPtr p);
    [DllImport(Lib)] public static extern int lonnx_memcpy_h2d(IntPtr ctx, IntPtr dst, void* src, nuint bytes);
    [DllImport(Lib)] public static extern int lonnx_memcpy_d2h(IntPtr ctx, void* dst, IntPtr src, nuint bytes);
    [DllImport(Lib)] public static extern int lonnx_memcpy_d2d(IntPtr ctx, IntPtr dst, IntPtr src, nuint bytes);
    [DllImport(Lib)] public static extern int lonnx_memset(IntPtr ctx, IntPtr dst, int value, nuint bytes);
    [DllImport(Lib)] public static extern int lonnx_sync(IntPtr ctx);
    [DllImport(Lib)] public static extern IntPtr lonnx_last_error();
    [DllImport(Lib)] public static extern int lonnx_debug_expire_wait(IntPtr ctx, long cycles);
    [DllImport(Lib)] public static extern long lonnx_launch_count(IntPtr ctx);

    // ---- element-wise ----
    [DllImport(Lib)] public static extern int lonnx_broadcast_shape(long* a, int ar, long* b, int br, long* outShape, out int outRank);
    [DllImport(Lib)] public static extern int lonnx_binary_f32(IntPtr ctx, int op, IntPtr a, long* aShape, int aRank,
        IntPtr b, long* bShape, int bRank, IntPtr y);
    [DllImport(Lib)] public static extern int lonnx_unary_f32(IntPtr ctx, int op, IntPtr x, IntPtr y, long n);
    [DllImport(Lib)] public static extern int lonnx_batchnorm_f32(IntPtr ctx, IntPtr x, IntPtr scale, IntPtr bias,
        IntPtr mean, IntPtr var, float eps, IntPtr y, long outer, long channels, long inner);

    // ---- contractions ----
    [DllImport(Lib)] public static extern int lonnx_gemm_f32(IntPtr ctx, IntPtr A, IntPtr B, IntPtr bias, IntPtr C,
        int batch, int M, int N, int K, long sA, long sB, long sC, int transB, float alpha, float beta, int epilogue);
    [DllImport(Lib)] public static extern int lonnx_gemm_f32_noalloc(IntPtr stream, IntPtr A, IntPtr B, IntPtr bias,
        IntPtr C, int batch, int M, int N, int K, long sA, long sB, long sC, int transB, float alpha, float beta,
        int epilogue);
    [DllImport(Lib)] public static extern int lonnx_gemm_f32_noalloc_status(IntPtr stream);
    [DllImport(Lib)] public static extern int lonnx_matmul_f32(IntPtr ctx, IntPtr a, long* aShape, int aRank,
        IntPtr b, long* bShape, int bRank, IntPtr y);
    [DllImport(Lib)] public static extern int lonnx_conv2d_f32(IntPtr ctx, IntPtr x, IntPtr w, IntPtr bias, IntPtr y,
        int N, int C, int H, int W, int M, int kh, int kw, int sh, int sw, int pt, int pl, int pb, int pr,
        int dh, int dw, int group, int relu);

    // ---- row kernels ----
    [DllImport(Lib)] public static extern int lonnx_softmax_f32(IntPtr ctx, IntPtr x, IntPtr y, long outer, long len, long inner);
    [DllImport(Lib)] public static extern int lonnx_layernorm_f32(IntPtr ctx, IntPtr x, IntPtr res, IntPtr gamma,
        IntPtr beta, float eps, IntPtr y, long rows, int cols);
    [DllImport(Lib)] public static extern int lonnx_reduce_f32(IntPtr ctx, int op, IntPtr x, long* shape, int rank,
        long* axes, int naxes, IntPtr y);
    [DllImport(Lib)] public static extern int lonnx_maxpool2d_f32(IntPtr ctx, IntPtr x, IntPtr y, int N, int C, int H, int W,
        int kh, int kw, int sh, int sw, int pt, int pl, int Ho, int Wo);

    // ---- data movement ----
    [DllImport(Lib)] public static extern int lonnx_gather(IntPtr ctx, IntPtr data, int elemBytes, long outer, long dim,
        long inner, IntPtr idx, long nIdx, IntPtr y);
    [DllImport(Lib)] public static extern int lonnx_transpose(IntPtr ctx, IntPtr x, int elemBytes, long* shape, int rank,
        long* perm, IntPtr y);
    [DllImport(Lib)] public static extern int lonnx_cast_i64_f32(IntPtr ctx, IntPtr x, IntPtr y, long n);

    // ---- pre-processing before the model (Images.ImageToArrayF, Text.RobertaTokenize padding) ----
    [DllImport(Lib)] public static extern int lonnx_image_rgba_to_f32(IntPtr ctx, IntPtr rgba, IntPtr y, long nImages,
        long height, long width);
    [DllImport(Lib)] public static extern int lonnx_token_batch_pad(IntPtr ctx, IntPtr ids, IntPtr offsets, long batch,
        long maxLen, long padId, IntPtr idsOut, IntPtr maskOut, IntPtr typeOut);

    // ---- fused encoder ops ----
    [DllImport(Lib)] public static extern int lonnx_attention_f32(IntPtr ctx, IntPtr q, IntPtr k, IntPtr v, long ldQkv,
        IntPtr maskadd, IntPtr output, int B, int S, int heads, int dh, float scale);

    // ---- graph executor ----
    [DllImport(Lib)] public static extern int lonnx_graph_create(IntPtr ctx, out IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_destroy(IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_add_initializer(IntPtr g, string name, int dtype, long* shape,
        int rank, void* data);
    [DllImport(Lib)] public static extern int lonnx_graph_add_node(IntPtr g, string op, string[] inputs, int nIn,
        string[] outputs, int nOut);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_int(IntPtr g, string name, long v);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_ints(IntPtr g, string name, long[] v, int n);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_float(IntPtr g, string name, float v);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_floats(IntPtr g, string name, float[] v, int n);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_string(IntPtr g, string name, string v);
    [DllImport(Lib)] public static extern int lonnx_graph_attr_tensor(IntPtr g, string name, int dtype, long* shape,
        int rank, void* data);
    [DllImport(Lib)] public static extern int lonnx_graph_add_output(IntPtr g, string name);
    [DllImport(Lib)] public static extern int lonnx_graph_set_opset(IntPtr g, int opset);
    [DllImport(Lib)] public static extern int lonnx_graph_prepare(IntPtr g, int flags);
    [DllImport(Lib)] public static extern int lonnx_graph_set_input(IntPtr g, string name, int dtype, long* shape,
        int rank, void* data);
    [DllImport(Lib)] public static extern int lonnx_graph_set_input_device(IntPtr g, string name, int dtype, long* shape,
        int rank, IntPtr dev);
    [DllImport(Lib)] public static extern int lonnx_graph_execute(IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_output_shape(IntPtr g, string name, long* shape, out int rank);
    [DllImport(Lib)] public static extern int lonnx_graph_output_dtype(IntPtr g, string name, out int dtype);
    [DllImport(Lib)] public static extern int lonnx_graph_output_device(IntPtr g, string name, out IntPtr dev);
    [DllImport(Lib)] public static extern int lonnx_graph_get_output(IntPtr g, string name, void* host, nuint bytes);
    [DllImport(Lib)] public static extern int lonnx_graph_reset(IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_capture(IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_replay(IntPtr g);
    [DllImport(Lib)] public static extern int lonnx_graph_num_steps(IntPtr g);

    public static string LastError() => Marshal.PtrToStringAnsi(lonnx_last_error()) ?? "";

    /// <summary>Throws CudaException for a non-zero status (used where the reference would throw, e.g.
    /// inside Node.Execute, whose catch turns it into OpResult.Failure).</summary>
    public static void Check(int rc)
    {
        if (rc != LONNX_OK) throw new CudaException(rc, LastError());
    }
}

public sealed class CudaException : Exception
{
    public int Code { get; }
    public CudaException(int code, string message) : base(message) { Code = code; }
}
