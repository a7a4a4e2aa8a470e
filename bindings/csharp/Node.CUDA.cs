// Node.ExecuteCUDA: the CUDA branch of Node.Execute, mirroring ExecuteCPU
// (src/Lokad.Onnx.Backend/Node.cs:121-181) op for op, with the same inputs
// and the same attribute reads -- including Conv's Attr<int[]> reads, which
// see the loader's long[] attributes as absent (Node.cs:137-138), so per-node
// CUDA execution gives the reference's results.
//
// Two one-line changes in the reference wire it in:
//   CPUExecutionProvider.cs:11-14   enum ExecutionProvider { CPU, CUDA }
//   Node.cs:84-106 (Node.Execute)   else if (provider == ExecutionProvider.CUDA) { var r = ExecuteCUDA(graph); ...same output naming as the CPU branch... }
// and ComputationalGraph.Execute (ComputationalGraph.cs:199) passes its
// provider argument on to node.Execute(this, provider).
namespace Lokad.Onnx;

using Lokad.Onnx.Cuda;

using static Lokad.Onnx.OpResult;
using CUDA = Lokad.Onnx.Cuda.CUDAExecutionProvider;

public partial struct Node
{
    public OpResult ExecuteCUDA(ComputationalGraph graph) => Op switch
    {
        OpType.Reshape => CUDA.Reshape(InputTensor(graph, 0), InputTensor(graph, 1), Attr<bool?>("allow_zero")),
        OpType.Add => CUDA.Add(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Sub => CUDA.Sub(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Mul => CUDA.Mul(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Div => CUDA.Div(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Pow => CUDA.Pow(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Sqrt => CUDA.Sqrt(InputTensor(graph, 0)),
        OpType.Conv => CUDA.Conv(InputTensor(graph, 0), InputTensor(graph, 1), InputTensor(graph, 2),
            Attr<string>("auto_pad"), Attr<int[]>("dilations"), Attr<int?>("group"), Attr<int[]>("kernel_shape"),
            Attr<int[]>("pads"), Attr<int[]>("strides")),
        OpType.Relu => CUDA.Relu(InputTensor(graph, 0)),
        OpType.Erf => CUDA.Erf(InputTensor(graph, 0)),
        OpType.MaxPool => CUDA.MaxPool(InputTensor(graph, 0), Attr<string>("auto_pad"), Attr<int?>("ceil_mode"),
            Ints("dilations"), Ints("kernel_shape"), Ints("pads"), Attr<int?>("storage_order"), Ints("strides")),
        OpType.MatMul => CUDA.MatMul(InputTensor(graph, 0), InputTensor(graph, 1)),
        OpType.Transpose => CUDA.Transpose(InputTensor(graph, 0), Ints("perm")),
        OpType.Constant => CUDA.Constant(OneOfAttr("sparse_value", "value", "value_float", "value_floats", "value_int",
            "value_ints", "value_string", "value_strings")),
        OpType.Cast => CUDA.Cast(InputTensor(graph, 0), RequiredInt("to")),
        OpType.Concat => CUDA.Concat(graph.GetInputTensors(Inputs), RequiredInt("axis")),
        OpType.Shape => CUDA.Shape(InputTensor(graph, 0), Int("start"), Int("end")),
        OpType.Gather => CUDA.Gather(InputTensor(graph, 0), InputTensor(graph, 1), Int("axis")),
        OpType.Slice => CUDA.Slice(InputTensor(graph, 0), InputTensor(graph, 1), InputTensor(graph, 2),
            InputTensor(graph, 3), InputTensor(graph, 4)),
        OpType.Unsqueeze => graph.OpsetVersion() switch
        {
            int v when v >= 13 => CUDA.Unsqueeze(InputTensor(graph, 0), InputTensor(graph, 1)),
            _ => CUDA.Unsqueeze(InputTensor(graph, 0), RequiredInts("axes")),
        },
        OpType.ReduceSum => CUDA.ReduceSum(InputTensor(graph, 0), InputTensor(graph, 1), Int("keepdims"), Int("noop_with_empty_axes")),
        OpType.ReduceMean => graph.OpsetVersion() switch
        {
            int v when v >= 13 => CUDA.ReduceMean(InputTensor(graph, 0), InputTensor(graph, 1), Int("keepdims"), Int("noop_with_empty_axes")),
            _ => CUDA.ReduceMean(InputTensor(graph, 0), RequiredInts("axes")?.ToTensor<int>(), Int("keepdims"), Int("noop_with_empty_axes")),
        },
        OpType.ReduceMax => CUDA.ReduceMax(InputTensor(graph, 0), InputTensor(graph, 1), Int("keepdims")),
        OpType.Softmax => CUDA.Softmax(InputTensor(graph, 0), Int("axis")),
        // ONNX ops the CPU branch does not dispatch (ResNet-50 coverage)
        OpType.Gemm => CUDA.Gemm(InputTensor(graph, 0), InputTensor(graph, 1), InputTensor(graph, 2),
            Attr<float?>("alpha"), Attr<float?>("beta"), Int("transA"), Int("transB")),
        OpType.BatchNormalization => CUDA.BatchNormalization(InputTensor(graph, 0), InputTensor(graph, 1),
            InputTensor(graph, 2), InputTensor(graph, 3), InputTensor(graph, 4), Attr<float?>("epsilon")),
        OpType.GlobalAveragePool => CUDA.GlobalAveragePool(InputTensor(graph, 0)),
        OpType.Flatten => CUDA.Flatten(InputTensor(graph, 0), Int("axis")),
        _ => NotSupported(Op)
    };
}
