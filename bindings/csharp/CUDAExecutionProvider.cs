// CUDAExecutionProvider: the reference's operator API (CPUExecutionProvider,
// src/Lokad.Onnx.Backend/CPUExecutionProvider.cs:56-695) executed on a B200
// through liblonnx_cuda.so.  Every method keeps the CPU provider's signature,
// argument meaning and failure behaviour: validation failures and native
// errors come back as OpResult.Failure(op, message), never as exceptions
// (OpResult.cs:34-62).
//
// Each call runs one node through the native executor (a one-node graph on
// the context's stream), with its inputs' device copies bound in place
// (DeviceStorage) and its outputs returned as host tensors that keep their
// device copy attached, so a chain of CUDA ops uploads each tensor once.
// Whole models should use CudaGraphSession instead, which fuses node chains
// and never leaves the device between nodes.
namespace Lokad.Onnx.Cuda;

using System;
using System.Collections.Generic;
using System.Linq;

using static Lokad.Onnx.OpResult;

public static class CUDAExecutionProvider
{
    /// <summary>Device used by the static operator methods.</summary>
    public static CudaContext Context { get; set; } = null!;

    static CudaContext Ctx => Context ??= CudaContext.Default(0);

    public static readonly OpType[] SupportedOps =
    {
        OpType.Reshape, OpType.Add, OpType.Div, OpType.Sub, OpType.Mul, OpType.Pow, OpType.Conv, OpType.Relu,
        OpType.MaxPool, OpType.MatMul, OpType.Sqrt, OpType.Erf, OpType.Transpose, OpType.Constant, OpType.Cast,
        OpType.Concat, OpType.Shape, OpType.Gather, OpType.Slice, OpType.Unsqueeze, OpType.ReduceSum,
        OpType.ReduceMean, OpType.ReduceMax, OpType.Softmax,
        // beyond the CPU provider: the ResNet-50 ops (ONNX semantics)
        OpType.Gemm, OpType.BatchNormalization, OpType.GlobalAveragePool, OpType.Flatten
    };

    public static bool SupportsOp(OpType op) => SupportedOps.Contains(op);

    static OpResult Run(OpType op, ITensor?[] inputs, params (string Name, object? Value)[] attrs) =>
        NodeRunner.Run(Ctx, op, inputs, attrs, opset: 13, honorConvAttrs: true);

    static OpResult Binary(OpType op, ITensor? A, ITensor? B)
    {
        if (A is null) return MissingInput(op, nameof(A));
        if (B is null) return MissingInput(op, nameof(B));
        if (A.ElementType != B.ElementType) return WrongInputType(op, nameof(B), "Input tensors must be of the same type.", B);
        return Run(op, new[] { A, B });
    }

    public static OpResult Reshape(ITensor? input, ITensor? shape, bool? allow_zero = null)
    {
        var op = OpType.Reshape;
        if (input is null) return MissingInput(op, nameof(input));
        if (shape is null) return MissingInput(op, nameof(shape));
        if (shape.ElementType != TensorElementType.Int64) return WrongInputType(op, nameof(shape), TensorElementType.Int64, shape);
        return Run(op, new[] { input, shape }, ("allowzero", allow_zero is null ? null : (long)(allow_zero.Value ? 1 : 0)));
    }

    public static OpResult Add(ITensor? A, ITensor? B) => Binary(OpType.Add, A, B);
    public static OpResult Sub(ITensor? A, ITensor? B) => Binary(OpType.Sub, A, B);
    public static OpResult Mul(ITensor? A, ITensor? B) => Binary(OpType.Mul, A, B);
    public static OpResult Div(ITensor? A, ITensor? B) => Binary(OpType.Div, A, B);
    public static OpResult Pow(ITensor? A, ITensor? B) => Binary(OpType.Pow, A, B);

    public static OpResult Conv(ITensor? X, ITensor? W, ITensor? B, string? auto_pad = null, int[]? dilations = null,
        int? group = null, int[]? kernel_shape = null, int[]? pads = null, int[]? strides = null)
    {
        var op = OpType.Conv;
        if (X is null) return MissingInput(op, nameof(X));
        if (W is null) return MissingInput(op, nameof(W));
        if (W.ElementType != X.ElementType) return WrongInputType(op, nameof(W), X.ElementType, W, "The weights tensor must be the same type as the input tensor.");
        if (X.Rank != 4) return WrongInputShape(op, nameof(X), 4, X);
        if (W.Rank != 4) return WrongInputShape(op, nameof(W), 4, W);
        if (auto_pad == "NOTSET")
        {
            if (pads is null) return MissingAttribute(op, nameof(pads), "When auto_pad is NOTSET pads must be specified");
            if (!pads.All(p => p == pads[0])) return AttributeNotSupported(op, "pads", string.Join(",", pads), "Asymmetric padding is not supported.");
        }
        // the CPU provider reads pads only under NOTSET: pass them only then
        return Run(op, new[] { X, W, B }, ("auto_pad", auto_pad), ("dilations", dilations), ("group", group),
            ("kernel_shape", kernel_shape), ("pads", auto_pad == "NOTSET" ? pads : null), ("strides", strides));
    }

    public static OpResult Relu(ITensor? X) => X is null ? MissingInput(OpType.Relu, nameof(X)) : Run(OpType.Relu, new[] { X });

    public static OpResult MaxPool(ITensor? X, string? auto_pad = null, int? ceil_mode = null, int[]? dilations = null,
        int[]? kernel_shape = null, int[]? pads = null, int? storage_order = null, int[]? strides = null)
    {
        var op = OpType.MaxPool;
        if (X is null) return MissingInput(op, nameof(X));
        if (X.Rank != 4) return WrongInputShape(op, nameof(X), 4, X);
        if (kernel_shape is null) return MissingAttribute(op, nameof(kernel_shape));
        return Run(op, new[] { X }, ("auto_pad", auto_pad), ("dilations", dilations), ("kernel_shape", kernel_shape),
            ("pads", pads), ("strides", strides));
    }

    public static OpResult MatMul(ITensor? A, ITensor? B)
    {
        var op = OpType.MatMul;
        if (A is null) return MissingInput(op, nameof(A));
        if (B is null) return MissingInput(op, nameof(B));
        return Run(op, new[] { A, B });
    }

    public static OpResult Sqrt(ITensor? A) => A is null ? MissingInput(OpType.Sqrt, nameof(A)) : Run(OpType.Sqrt, new[] { A });

    public static OpResult Erf(ITensor? X) => X is null ? MissingInput(OpType.Erf, nameof(X)) : Run(OpType.Erf, new[] { X });

    public static OpResult Transpose(ITensor? data, int[]? perm = null) =>
        data is null ? MissingInput(OpType.Transpose, nameof(data)) : Run(OpType.Transpose, new[] { data }, ("perm", perm));

    public static OpResult Constant(object? value)
    {
        var op = OpType.Constant;
        if (value is null) return MissingAttribute(op, nameof(value));
        return value switch
        {
            ITensor t => Run(op, Array.Empty<ITensor?>(), ("value", t)),
            float f => Run(op, Array.Empty<ITensor?>(), ("value_float", f)),
            float[] fa => Run(op, Array.Empty<ITensor?>(), ("value_floats", fa)),
            int i => Run(op, Array.Empty<ITensor?>(), ("value_int", (long)i)),
            int[] ia => Run(op, Array.Empty<ITensor?>(), ("value_ints", ia)),
            _ => NotSupported(op)
        };
    }

    public static OpResult Cast(ITensor? input, long to) =>
        input is null ? MissingInput(OpType.Cast, nameof(input)) : Run(OpType.Cast, new[] { input }, ("to", to));

    public static OpResult Concat(ITensor[]? inputs, int? _axis)
    {
        var op = OpType.Concat;
        if (inputs is null) return MissingInput(op, nameof(inputs));
        if (!inputs.All(i => i.ElementType == inputs[0].ElementType))
            return WrongInputType(op, nameof(inputs), "All tensors in a concat operation must have the same type.", inputs[0]);
        return Run(op, inputs, ("axis", (long)(_axis ?? 0)));
    }

    public static OpResult Shape(ITensor? data, int? _start = null, int? _end = null) =>
        data is null ? MissingInput(OpType.Shape, nameof(data))
                     : Run(OpType.Shape, new[] { data }, ("start", _start), ("end", _end));

    public static OpResult Gather(ITensor? data, ITensor? indices, int? axis = null)
    {
        var op = OpType.Gather;
        if (data is null) return MissingInput(op, nameof(data));
        if (indices is null) return MissingInput(op, nameof(indices));
        if (indices.Rank > data.Rank) return WrongInputShape(op, nameof(indices), data.Rank, indices);
        return Run(op, new[] { data, indices }, ("axis", axis));
    }

    public static OpResult Slice(ITensor? data, ITensor? starts, ITensor? ends, ITensor? axes, ITensor? steps)
    {
        var op = OpType.Slice;
        if (data is null) return MissingInput(op, nameof(data));
        if (starts is null) return MissingInput(op, nameof(starts));
        if (ends is null) return MissingInput(op, nameof(ends));
        if (data.Rank == 0) return WrongInputShape(op, nameof(data), data, "Cannot slice a tensor of rank 0");
        if (starts.Rank != 1) return WrongInputShape(op, nameof(starts), starts, "The rank of the starts tensor must be 1");
        if (ends.Rank != 1) return WrongInputShape(op, nameof(ends), ends, "The rank of the ends tensor must be 1");
        if (starts.Dims[0] != ends.Dims[0]) return WrongInputShape(op, nameof(ends), ends, "The ends tensor must be the same length as the start tensor.");
        return Run(op, new[] { data, starts, ends, axes, steps });
    }

    public static OpResult Unsqueeze(ITensor? data, ITensor? axes)
    {
        var op = OpType.Unsqueeze;
        if (data is null) return MissingInput(op, nameof(data));
        if (axes is null) return MissingInput(op, nameof(axes));
        return Run(op, new[] { data, axes });
    }

    public static OpResult Unsqueeze(ITensor? data, int[] axes) =>
        data is null ? MissingInput(OpType.Unsqueeze, nameof(data))
                     : NodeRunner.Run(Ctx, OpType.Unsqueeze, new[] { data }, new (string, object?)[] { ("axes", axes) }, opset: 11, honorConvAttrs: true);

    public static OpResult ReduceSum(ITensor? data, ITensor? axes, int? _keep_dims, int? noop_with_empty_axes) =>
        data is null ? MissingInput(OpType.ReduceSum, nameof(data)) : Run(OpType.ReduceSum, new[] { data, axes }, ("keepdims", _keep_dims));

    public static OpResult ReduceMean(ITensor? data, ITensor? axes, int? _keep_dims, int? noop_with_empty_axes) =>
        data is null ? MissingInput(OpType.ReduceMean, nameof(data)) : Run(OpType.ReduceMean, new[] { data, axes }, ("keepdims", _keep_dims));

    public static OpResult ReduceMax(ITensor? data, ITensor? axes, int? _keep_dims) =>
        data is null ? MissingInput(OpType.ReduceMax, nameof(data)) : Run(OpType.ReduceMax, new[] { data, axes }, ("keepdims", _keep_dims));

    public static OpResult Softmax(ITensor? input, int? _axis) =>
        input is null ? MissingInput(OpType.Softmax, nameof(input)) : Run(OpType.Softmax, new[] { input }, ("axis", _axis));

    // ---- ONNX ops the CPU provider lacks (ResNet-50 coverage, ONNX semantics) ----

    public static OpResult Gemm(ITensor? A, ITensor? B, ITensor? C, float? alpha = null, float? beta = null,
        int? transA = null, int? transB = null)
    {
        var op = OpType.Gemm;
        if (A is null) return MissingInput(op, nameof(A));
        if (B is null) return MissingInput(op, nameof(B));
        if (A.Rank != 2) return WrongInputShape(op, nameof(A), 2, A);
        if (B.Rank != 2) return WrongInputShape(op, nameof(B), 2, B);
        return Run(op, new[] { A, B, C }, ("alpha", alpha), ("beta", beta), ("transA", transA), ("transB", transB));
    }

    public static OpResult BatchNormalization(ITensor? X, ITensor? scale, ITensor? B, ITensor? input_mean,
        ITensor? input_var, float? epsilon = null)
    {
        var op = OpType.BatchNormalization;
        if (X is null) return MissingInput(op, nameof(X));
        if (scale is null) return MissingInput(op, nameof(scale));
        if (B is null) return MissingInput(op, nameof(B));
        if (input_mean is null) return MissingInput(op, nameof(input_mean));
        if (input_var is null) return MissingInput(op, nameof(input_var));
        return Run(op, new[] { X, scale, B, input_mean, input_var }, ("epsilon", epsilon));
    }

    public static OpResult GlobalAveragePool(ITensor? X) =>
        X is null ? MissingInput(OpType.GlobalAveragePool, nameof(X)) : Run(OpType.GlobalAveragePool, new[] { X });

    public static OpResult Flatten(ITensor? input, int? axis = null) =>
        input is null ? MissingInput(OpType.Flatten, nameof(input)) : Run(OpType.Flatten, new[] { input }, ("axis", axis));
}

/// <summary>Runs one node through the native executor and maps native errors to OpResult.Failure.</summary>
internal static unsafe class NodeRunner
{
    public static OpResult Run(CudaContext ctx, OpType op, ITensor?[] inputs, (string Name, object? Value)[] attrs,
        int opset, bool honorConvAttrs)
    {
        if (Native.lonnx_graph_create(ctx.Handle, out var g) != Native.LONNX_OK) return Failure(op, Native.LastError());
        try
        {
            var names = new string[inputs.Length];
            for (int i = 0; i < inputs.Length; i++) names[i] = inputs[i] is null ? "" : "in" + i;
            int nIn = names.Length;
            while (nIn > 0 && names[nIn - 1] == "") nIn--;
            for (int i = 0; i < nIn; i++)
            {
                var t = inputs[i];
                if (t is null) continue;
                var buf = DeviceStorage.ToDevice(t, ctx);
                var shape = DeviceStorage.Shape(t);
                fixed (long* s = shape)
                    if (Native.lonnx_graph_set_input_device(g, names[i], DTypes.Of(t.ElementType), s, shape.Length, buf.Ptr) != 0)
                        return Failure(op, Native.LastError());
            }
            var outs = new[] { "out0" };
            if (Native.lonnx_graph_add_node(g, op.ToString(), names.Take(nIn).ToArray(), nIn, outs, outs.Length) != 0)
                return Failure(op, Native.LastError());
            foreach (var (name, value) in attrs)
            {
                int rc = value switch
                {
                    null => 0,
                    int v => Native.lonnx_graph_attr_int(g, name, v),
                    long v => Native.lonnx_graph_attr_int(g, name, v),
                    float v => Native.lonnx_graph_attr_float(g, name, v),
                    string v => Native.lonnx_graph_attr_string(g, name, v),
                    int[] v => Native.lonnx_graph_attr_ints(g, name, v.Select(x => (long)x).ToArray(), v.Length),
                    long[] v => Native.lonnx_graph_attr_ints(g, name, v, v.Length),
                    float[] v => Native.lonnx_graph_attr_floats(g, name, v, v.Length),
                    ITensor t => AttrTensor(g, name, t),
                    _ => int.MinValue
                };
                if (rc == int.MinValue) return AttributeNotSupported(op, name, value!.ToString() ?? "");
                if (rc != 0) return Failure(op, Native.LastError());
            }
            foreach (var o in outs) Native.Check(Native.lonnx_graph_add_output(g, o));
            Native.Check(Native.lonnx_graph_set_opset(g, opset));
            if (Native.lonnx_graph_prepare(g, honorConvAttrs ? 2 : 0) != 0) return Failure(op, Native.LastError());
            if (Native.lonnx_graph_execute(g) != 0) return Failure(op, Native.LastError());
            var results = new ITensor[outs.Length];
            for (int k = 0; k < outs.Length; k++)
            {
                var shape = new long[8];
                int rank, dtype;
                fixed (long* s = shape) Native.Check(Native.lonnx_graph_output_shape(g, outs[k], s, out rank));
                Native.Check(Native.lonnx_graph_output_dtype(g, outs[k], out dtype));
                Native.Check(Native.lonnx_graph_output_device(g, outs[k], out var dev));
                var dims = shape.Take(rank).Select(d => (int)d).ToArray();
                long bytes = dims.Aggregate(1L, (a, d) => a * d) * DTypes.Size(dtype);
                var buf = new DeviceBuffer(ctx, bytes);  // owned by the result; the graph's copy dies with it
                if (bytes > 0) Native.Check(Native.lonnx_memcpy_d2d(ctx.Handle, buf.Ptr, dev, (nuint)bytes));
                results[k] = DeviceStorage.ToHost(buf, dtype, dims);
            }
            ctx.Sync();
            return Success(op, results);
        }
        catch (CudaException e)
        {
            return Failure(op, e.Message);
        }
        finally
        {
            Native.lonnx_graph_destroy(g);
        }
    }

    static int AttrTensor(IntPtr g, string name, ITensor t)
    {
        var dense = t.ToDenseTensor();
        var shape = DeviceStorage.Shape(dense);
        var bytes = dense switch
        {
            DenseTensor<float> f => System.Runtime.InteropServices.MemoryMarshal.AsBytes(f.Buffer.Span).ToArray(),
            DenseTensor<long> l => System.Runtime.InteropServices.MemoryMarshal.AsBytes(l.Buffer.Span).ToArray(),
            DenseTensor<int> i => System.Runtime.InteropServices.MemoryMarshal.AsBytes(i.Buffer.Span).ToArray(),
            _ => throw new NotSupportedException($"Constant of type {t.ElementType}")
        };
        fixed (long* s = shape)
        fixed (byte* d = bytes)
            return Native.lonnx_graph_attr_tensor(g, name, DTypes.Of(t.ElementType), s, shape.Length, d);
    }
}
