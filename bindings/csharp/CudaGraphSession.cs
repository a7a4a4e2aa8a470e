// CudaGraphSession: a whole ComputationalGraph loaded once onto one GPU and
// executed there -- the fast path behind ComputationalGraph.Execute(...,
// ExecutionProvider.CUDA) (src/Lokad.Onnx.Backend/ComputationalGraph.cs:199-272).
//
// The graph's nodes, attributes and initializers go to the native executor
// once (lonnx_graph_*); lonnx_graph_prepare fuses node chains (GEMM + bias
// [+ GELU], packed QKV, attention, LayerNorm, Conv + Add + Relu,
// Conv + BatchNormalization) and re-lays the weights out for the tensor
// cores.  Each Execute stages the inputs, runs every node on the GPU with the
// activations resident in HBM, and copies only the graph outputs back.
namespace Lokad.Onnx.Cuda;

using System;
using System.Collections.Generic;
using System.Linq;

public sealed unsafe class CudaGraphSession : IDisposable
{
    readonly IntPtr g;
    readonly ComputationalGraph graph;
    public CudaContext Context { get; }

    /// <param name="honorConvAttributes">Apply Conv's strides/pads/dilations/group (ONNX semantics).
    /// False reproduces the reference's per-node dispatch, which drops them (Node.cs:137-138).</param>
    public CudaGraphSession(ComputationalGraph graph, CudaContext? ctx = null, bool fuse = true, bool honorConvAttributes = false)
    {
        this.graph = graph;
        Context = ctx ?? CudaContext.Default(0);
        Native.Check(Native.lonnx_graph_create(Context.Handle, out g));
        Native.Check(Native.lonnx_graph_set_opset(g, graph.OpsetVersion()));
        foreach (var (name, t) in graph.Initializers) AddTensor(name, t, initializer: true);
        foreach (var node in graph.Nodes)
        {
            Native.Check(Native.lonnx_graph_add_node(g, node.Op.ToString(), node.Inputs, node.Inputs.Length,
                node.Outputs, node.Outputs.Length));
            if (node.Attributes is null) continue;
            foreach (var (name, value) in node.Attributes)
            {
                switch (value)
                {
                    case long v: Native.Check(Native.lonnx_graph_attr_int(g, name, v)); break;
                    case int v: Native.Check(Native.lonnx_graph_attr_int(g, name, v)); break;
                    case long[] v: Native.Check(Native.lonnx_graph_attr_ints(g, name, v, v.Length)); break;
                    case int[] v: Native.Check(Native.lonnx_graph_attr_ints(g, name, v.Select(x => (long)x).ToArray(), v.Length)); break;
                    case float v: Native.Check(Native.lonnx_graph_attr_float(g, name, v)); break;
                    case float[] v: Native.Check(Native.lonnx_graph_attr_floats(g, name, v, v.Length)); break;
                    case string v: Native.Check(Native.lonnx_graph_attr_string(g, name, v)); break;
                    case ITensor v: AddTensorAttr(name, v); break;
                    default: break;  // graphs / sparse tensors: not on the float path
                }
            }
        }
        foreach (var o in graph.Outputs.Keys) Native.Check(Native.lonnx_graph_add_output(g, o));
        Native.Check(Native.lonnx_graph_prepare(g, (fuse ? 1 : 0) | (honorConvAttributes ? 2 : 0)));
    }

    void AddTensor(string name, ITensor t, bool initializer)
    {
        var d = t.ToDenseTensor();
        var shape = DeviceStorage.Shape(d);
        WithBytes(d, p =>
        {
            fixed (long* s = shape)
                Native.Check(initializer
                    ? Native.lonnx_graph_add_initializer(g, name, DTypes.Of(d.ElementType), s, shape.Length, p)
                    : Native.lonnx_graph_set_input(g, name, DTypes.Of(d.ElementType), s, shape.Length, p));
        });
    }

    void AddTensorAttr(string name, ITensor t)
    {
        var d = t.ToDenseTensor();
        var shape = DeviceStorage.Shape(d);
        WithBytes(d, p =>
        {
            fixed (long* s = shape) Native.Check(Native.lonnx_graph_attr_tensor(g, name, DTypes.Of(d.ElementType), s, shape.Length, p));
        });
    }

    static void WithBytes(ITensor d, Action<IntPtr> f)
    {
        switch (d)
        {
            case DenseTensor<float> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            case DenseTensor<long> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            case DenseTensor<int> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            case DenseTensor<byte> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            case DenseTensor<bool> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            case DenseTensor<double> x: using (var h = x.Buffer.Pin()) f((IntPtr)h.Pointer); break;
            default: throw new NotSupportedException($"tensor type {d.ElementType}");
        }
    }

    /// <summary>ComputationalGraph.Execute on the GPU: inputs by name, graph outputs returned (and stored in
    /// graph.Outputs like the CPU path does).  Returns false with the failure message on error.</summary>
    public bool Execute(Dictionary<string, ITensor> inputs, out string? error)
    {
        error = null;
        try
        {
            foreach (var (name, t) in inputs)
            {
                if (DeviceStorage.IsOnDevice(t))
                {
                    var shape = DeviceStorage.Shape(t);
                    fixed (long* s = shape)
                        Native.Check(Native.lonnx_graph_set_input_device(g, name, DTypes.Of(t.ElementType), s, shape.Length,
                            DeviceStorage.DevicePtr(t)));
                }
                else AddTensor(name, t, initializer: false);
            }
            Native.Check(Native.lonnx_graph_execute(g));
            foreach (var o in graph.Outputs.Keys.ToList())
            {
                var shape = new long[8];
                int rank, dtype;
                fixed (long* s = shape) Native.Check(Native.lonnx_graph_output_shape(g, o, s, out rank));
                Native.Check(Native.lonnx_graph_output_dtype(g, o, out dtype));
                var dims = shape.Take(rank).Select(x => (int)x).ToArray();
                ITensor host = dtype switch
                {
                    1 => new DenseTensor<float>(dims),
                    7 => new DenseTensor<long>(dims),
                    6 => new DenseTensor<int>(dims),
                    _ => throw new NotSupportedException($"output dtype {dtype}")
                };
                long bytes = dims.Aggregate(1L, (a, x) => a * x) * DTypes.Size(dtype);
                WithBytes(host, p => Native.Check(Native.lonnx_graph_get_output(g, o, (void*)p, (nuint)bytes)));
                host.Name = o;
                graph.Outputs[o] = host;
            }
            return true;
        }
        catch (CudaException e)
        {
            error = e.Message;
            return false;
        }
    }

    /// <summary>Release intermediates back to the context's allocator (ComputationalGraph.Reset, :336-349).</summary>
    public void Reset() => Native.Check(Native.lonnx_graph_reset(g));

    /// <summary>Record one execution as a CUDA graph (inputs set, device-resident); Replay re-runs it with one launch.</summary>
    public void Capture() => Native.Check(Native.lonnx_graph_capture(g));
    public void Replay() => Native.Check(Native.lonnx_graph_replay(g));

    public void Dispose() => Native.lonnx_graph_destroy(g);
}
