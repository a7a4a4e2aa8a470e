// Device-resident storage for Lokad.Onnx tensors on a B200.
//
// The reference keeps every tensor in managed memory (DenseTensor<T> over
// Memory<T>, src/Lokad.Onnx.Tensors/DenseTensor.cs:31-42).  This file adds:
//   * CudaContext  -- one GPU: device, stream, caching allocator (lonnx_ctx);
//   * DeviceBuffer -- one allocation from a context, released through lonnx_free
//                     when disposed or finalised (a SafeHandle);
//   * DeviceStorage -- the device copy attached to a host tensor.  A tensor
//                     is uploaded once and its device copy reused by every
//                     later CUDA op (initializers therefore upload once per
//                     context); results of CUDA ops carry their device
//                     buffer, so a chain of CUDA ops never re-uploads.
namespace Lokad.Onnx.Cuda;

using System;
using System.Collections.Concurrent;
using System.Linq;
using System.Runtime.CompilerServices;
using System.Runtime.InteropServices;

public sealed class CudaContext : SafeHandle
{
    static readonly ConcurrentDictionary<int, CudaContext> defaults = new();

    public int Device { get; }
    public IntPtr Handle => handle;

    public CudaContext(int device) : base(IntPtr.Zero, true)
    {
        Native.Check(Native.lonnx_ctx_create(device, out var h));
        SetHandle(h);
        Device = device;
    }

    /// <summary>The process-wide context of one GPU (created on first use).</summary>
    public static CudaContext Default(int device = 0) => defaults.GetOrAdd(device, d => new CudaContext(d));

    public override bool IsInvalid => handle == IntPtr.Zero;
    protected override bool ReleaseHandle() => Native.lonnx_ctx_destroy(handle) == Native.LONNX_OK;

    /// <summary>Waits for the context's stream; reports device-side flags (Gather out of range, expired waits).</summary>
    public void Sync() => Native.Check(Native.lonnx_sync(handle));
}

public sealed class DeviceBuffer : SafeHandle
{
    public CudaContext Context { get; }
    public long Bytes { get; }
    public IntPtr Ptr => handle;

    public DeviceBuffer(CudaContext ctx, long bytes) : base(IntPtr.Zero, true)
    {
        Context = ctx;
        Bytes = bytes;
        Native.Check(Native.lonnx_malloc(ctx.Handle, (nuint)Math.Max(bytes, 1), out var p));
        SetHandle(p);
    }

    public override bool IsInvalid => handle == IntPtr.Zero;
    protected override bool ReleaseHandle() => Native.lonnx_free(Context.Handle, handle) == Native.LONNX_OK;
}

/// <summary>ONNX TensorProto element codes used by the native library.</summary>
public static class DTypes
{
    public static int Of(TensorElementType t) => t switch
    {
        TensorElementType.Float => 1,
        TensorElementType.UInt8 => 2,
        TensorElementType.Int32 => 6,
        TensorElementType.Int64 => 7,
        TensorElementType.Bool => 9,
        TensorElementType.Double => 11,
        _ => throw new NotSupportedException($"Element type {t} has no device representation.")
    };

    public static int Size(int dtype) => dtype switch { 1 => 4, 2 => 1, 6 => 4, 7 => 8, 9 => 1, 11 => 8, _ => 0 };
}

public static unsafe class DeviceStorage
{
    // host tensor -> its device copy (the buffer lives as long as the tensor does)
    static readonly ConditionalWeakTable<ITensor, DeviceBuffer> copies = new();

    public static bool IsOnDevice(ITensor t) => copies.TryGetValue(t, out _);

    public static IntPtr DevicePtr(ITensor t) => copies.TryGetValue(t, out var b) ? b.Ptr : IntPtr.Zero;

    /// <summary>The tensor's device copy on `ctx`, uploading it on first use (stream-ordered).</summary>
    public static DeviceBuffer ToDevice<T>(DenseTensor<T> t, CudaContext ctx) where T : unmanaged
    {
        if (copies.TryGetValue(t, out var b) && b.Context == ctx) return b;
        var bytes = (long)t.Length * sizeof(T);
        b = new DeviceBuffer(ctx, bytes);
        using (var pin = t.Buffer.Pin())
            Native.Check(Native.lonnx_memcpy_h2d(ctx.Handle, b.Ptr, pin.Pointer, (nuint)bytes));
        copies.AddOrUpdate(t, b);
        return b;
    }

    /// <summary>A host tensor holding `buf`'s contents, with `buf` attached as its device copy.</summary>
    public static DenseTensor<T> ToHost<T>(DeviceBuffer buf, int[] dims) where T : unmanaged
    {
        var t = new DenseTensor<T>(dims);
        var bytes = (long)t.Length * sizeof(T);
        if (bytes > buf.Bytes) throw new ArgumentException("device buffer smaller than the tensor");
        using (var pin = t.Buffer.Pin())
            Native.Check(Native.lonnx_memcpy_d2h(buf.Context.Handle, pin.Pointer, buf.Ptr, (nuint)bytes));
        copies.AddOrUpdate(t, buf);
        return t;
    }

    /// <summary>Uploads any supported dense tensor (float, int64, int32, uint8, bool, double).</summary>
    public static DeviceBuffer ToDevice(ITensor t, CudaContext ctx) => t switch
    {
        DenseTensor<float> f => ToDevice(f, ctx),
        DenseTensor<long> l => ToDevice(l, ctx),
        DenseTensor<int> i => ToDevice(i, ctx),
        DenseTensor<byte> u => ToDevice(u, ctx),
        DenseTensor<bool> z => ToDevice(z, ctx),
        DenseTensor<double> d => ToDevice(d, ctx),
        _ => ToDevice(t.ToDenseTensor(), ctx)
    };

    public static ITensor ToHost(DeviceBuffer buf, int dtype, int[] dims) => dtype switch
    {
        1 => ToHost<float>(buf, dims),
        2 => ToHost<byte>(buf, dims),
        6 => ToHost<int>(buf, dims),
        7 => ToHost<long>(buf, dims),
        9 => ToHost<bool>(buf, dims),
        11 => ToHost<double>(buf, dims),
        _ => throw new NotSupportedException($"dtype {dtype}")
    };

    public static long[] Shape(ITensor t) => t.Dims.Select(d => (long)d).ToArray();
}
