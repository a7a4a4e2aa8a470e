// Pre-processing on the device for Lokad.Onnx.Data callers.
//
// Images.ImageToArrayF (src/Lokad.Onnx.Data/Images.cs:92-103) loops over
// the pixels of a decoded ImageSharp image on the CPU; ImageToTensor below
// copies the image's RGBA8 rows to the GPU once and converts them there
// (lonnx_image_rgba_to_f32: ((R + G + B) / 3.0f) / 255.0f, the same two
// float divisions).  The MNIST variant keeps the reference's ImageSharp
// steps (Grayscale, Resize(28, 28): Images.cs:166-183) before the upload.
//
// Text.RobertaTokenize over a string array (Text.cs:76-146) pads every
// sequence to the longest on the CPU; PadBatch below uploads the ragged ids
// once and writes the padded input_ids / attention_mask / token_type_ids in
// HBM (lonnx_token_batch_pad), as DenseTensor<long> [B, longest] results
// whose device copies are attached, so the encoder reads them in place.
namespace Lokad.Onnx.Cuda;

using System;
using System.Collections.Generic;
using System.Linq;

using SixLabors.ImageSharp;
using SixLabors.ImageSharp.PixelFormats;
using SixLabors.ImageSharp.Processing;

public static unsafe class Preprocess
{
    /// <summary>A decoded image as float [1, 1, H, W] (Images.ImageToArrayF), converted on the GPU.</summary>
    public static DenseTensor<float> ImageToTensor(Image<Rgba32> image, CudaContext? ctx = null)
    {
        ctx ??= CudaContext.Default();
        int h = image.Height, w = image.Width;
        var rgba = new byte[(long)h * w * 4];
        image.CopyPixelDataTo(rgba);  // row-major RGBA8, the layout the kernel reads
        using var src = new DeviceBuffer(ctx, rgba.LongLength);
        fixed (byte* p = rgba)
            Native.Check(Native.lonnx_memcpy_h2d(ctx.Handle, src.Ptr, p, (nuint)rgba.LongLength));
        var dst = new DeviceBuffer(ctx, (long)h * w * sizeof(float));
        Native.Check(Native.lonnx_image_rgba_to_f32(ctx.Handle, src.Ptr, dst.Ptr, 1, h, w));
        return DeviceStorage.ToHost<float>(dst, new[] { 1, 1, h, w });  // synchronises before src is freed
    }

    /// <summary>Images.LoadMnistImageFromFile on the GPU: grayscale, 28 x 28, then ImageToTensor.</summary>
    public static DenseTensor<float>? LoadMnistImage(string file, CudaContext? ctx = null)
    {
        if (!System.IO.File.Exists(file)) return null;
        using var image = Image.Load<Rgba32>(file);
        image.Mutate(i => i.Grayscale());
        image.Mutate(i => i.Resize(28, 28));
        return ImageToTensor(image, ctx);
    }

    /// <summary>
    /// The padding of Text.RobertaTokenize(string[]): token-id sequences ->
    /// input_ids (padded with 1), attention_mask (1 / 0), token_type_ids (0),
    /// each [B, longest], padded on the GPU.
    /// </summary>
    public static ITensor[] PadBatch(IReadOnlyList<long[]> sequences, CudaContext? ctx = null, long padId = 1)
    {
        ctx ??= CudaContext.Default();
        int b = sequences.Count, longest = b == 0 ? 0 : sequences.Max(s => s.Length);
        var offsets = new long[b + 1];
        for (int i = 0; i < b; ++i) offsets[i + 1] = offsets[i] + sequences[i].Length;
        var flat = new long[Math.Max(offsets[b], 1)];
        for (int i = 0; i < b; ++i) Array.Copy(sequences[i], 0, flat, offsets[i], sequences[i].Length);
        using var dIds = new DeviceBuffer(ctx, flat.LongLength * sizeof(long));
        using var dOff = new DeviceBuffer(ctx, offsets.LongLength * sizeof(long));
        fixed (long* pf = flat, po = offsets)
        {
            Native.Check(Native.lonnx_memcpy_h2d(ctx.Handle, dIds.Ptr, pf, (nuint)(flat.LongLength * sizeof(long))));
            Native.Check(Native.lonnx_memcpy_h2d(ctx.Handle, dOff.Ptr, po, (nuint)(offsets.LongLength * sizeof(long))));
        }
        long bytes = (long)b * longest * sizeof(long);
        var ids = new DeviceBuffer(ctx, bytes);
        var mask = new DeviceBuffer(ctx, bytes);
        var types = new DeviceBuffer(ctx, bytes);
        Native.Check(Native.lonnx_token_batch_pad(ctx.Handle, dIds.Ptr, dOff.Ptr, b, longest, padId, ids.Ptr, mask.Ptr,
                                                 types.Ptr));
        var dims = new[] { b, longest };
        return new ITensor[]
        {
            DeviceStorage.ToHost<long>(ids, dims).WithName("input_ids"),
            DeviceStorage.ToHost<long>(mask, dims).WithName("attention_mask"),
            DeviceStorage.ToHost<long>(types, dims).WithName("token_type_ids"),
        };
    }
}
