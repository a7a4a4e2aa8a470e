"""Pre-processing before the model: the reference's data loaders
(src/Lokad.Onnx.Data/Images.cs and Text.cs), with the per-element work on
the GPU (csrc/preprocess.cu) and only decoding and tokenizing on the host.

Images.  ``load_images`` decodes files with Pillow (RGBA; for MNIST inputs
grayscale, then a 28 x 28 bicubic resize, as Images.cs:166-183 asks of
ImageSharp), stacks them as RGBA8 bytes and converts them on the device:
pixel = ((R + G + B) / 3.0f) / 255.0f into [N, 1, H, W], the arithmetic of
Images.ImageToArrayF (Images.cs:92-103).  The conversion is bit-exact; the
decoder and the resampler are Pillow's, not ImageSharp's, so resized pixels
are not pinned to the reference.

Text.  ``token_batch`` is the padding loop of Text.RobertaTokenize over a
string array (Text.cs:126-140) on the device: the ragged token ids go up
once, and input_ids (padded with 1), attention_mask (1 / 0) and
token_type_ids (0) are written in HBM as [B, longest].  ``XLMRobertaTokenizer``
turns text into ids with a SentencePiece model file and the XLM-R id
conventions (<s> 0, <pad> 1, </s> 2, <unk> 3, SentencePiece ids shifted by
one, at most 512 ids with the two specials, truncating the text:
Text.cs:60,106 call Encode(text, null, 512, OnlyFirst, 0)).  The reference
downloads the multilingual-e5-small model file; nothing here does, and the
caller passes its path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .tensor import Context, DeviceTensor

XLMR_BOS, XLMR_PAD, XLMR_EOS, XLMR_UNK = 0, 1, 2, 3
MAX_TOKENS = 512


def decode_image(path: str, mnist: bool = False) -> np.ndarray:
    """One image file as RGBA8 [H, W, 4] (grayscale 28 x 28 for MNIST)."""
    from PIL import Image
    im = Image.open(path).convert("RGBA")
    if mnist:
        im = im.convert("L").resize((28, 28), Image.BICUBIC).convert("RGBA")
    return np.ascontiguousarray(np.asarray(im, dtype=np.uint8))


def rgba_to_tensor(rgba: np.ndarray, ctx: Context | None = None) -> DeviceTensor:
    """RGBA8 [H, W, 4] or [N, H, W, 4] -> float [N, 1, H, W] on the device
    (Images.ImageToArrayF per image)."""
    ctx = ctx or Context.default()
    a = np.ascontiguousarray(rgba, dtype=np.uint8)
    if a.ndim == 3:
        a = a[None]
    if a.ndim != 4 or a.shape[-1] != 4:
        raise ValueError(f"expected RGBA pixels [N, H, W, 4], got {a.shape}")
    n, h, w, _ = a.shape
    src = DeviceTensor.from_host(ctx, a)
    out = DeviceTensor(ctx, (n, 1, h, w), np.float32)
    N.check(N.lib.lonnx_image_rgba_to_f32(ctx.handle, src.ptr, out.ptr, n, h, w))
    out._src = src  # keep the bytes alive until the stream has read them
    return out


def load_images(paths, mnist: bool = False, ctx: Context | None = None) -> DeviceTensor:
    """Image files of one size -> float [N, 1, H, W] on the device."""
    imgs = [decode_image(p, mnist) for p in paths]
    if len({im.shape for im in imgs}) != 1:
        raise ValueError("images of different sizes cannot share a batch")
    return rgba_to_tensor(np.stack(imgs), ctx)


def token_batch(sequences, ctx: Context | None = None, pad_id: int = XLMR_PAD) -> dict:
    """Token-id sequences -> {input_ids, attention_mask, token_type_ids}, each
    an int64 DeviceTensor [B, longest], right-padded as Text.cs:126-140 pads."""
    ctx = ctx or Context.default()
    seqs = [np.asarray(s, dtype=np.int64).ravel() for s in sequences]
    b = len(seqs)
    lens = np.array([len(s) for s in seqs], dtype=np.int64)
    longest = int(lens.max()) if b else 0
    offsets = np.zeros(b + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    flat = np.concatenate(seqs) if b and offsets[-1] else np.zeros(1, np.int64)
    d_ids, d_off = DeviceTensor.from_host(ctx, flat), DeviceTensor.from_host(ctx, offsets)
    out = {k: DeviceTensor(ctx, (b, longest), np.int64) for k in ("input_ids", "attention_mask", "token_type_ids")}
    N.check(N.lib.lonnx_token_batch_pad(ctx.handle, d_ids.ptr, d_off.ptr, b, longest, pad_id,
                                        out["input_ids"].ptr, out["attention_mask"].ptr,
                                        out["token_type_ids"].ptr))
    for t in out.values():
        t._src = (d_ids, d_off)
    return out


class XLMRobertaTokenizer:
    """Text -> XLM-R token ids from a SentencePiece model (the tokenizer of
    multilingual-e5-small that Text.cs:29-70 loads)."""

    def __init__(self, model_path: str | None = None, model_proto: bytes | None = None):
        import sentencepiece as spm
        self.sp = spm.SentencePieceProcessor()
        if model_proto is not None:
            self.sp.LoadFromSerializedProto(model_proto)
        elif model_path is not None:
            self.sp.Load(model_path)
        else:
            raise ValueError("a SentencePiece model path or proto is required")

    def piece_id(self, spm_id: int) -> int:
        """A SentencePiece id in the XLM-R vocabulary: shifted by one past the
        four specials; SentencePiece's unknown (0) maps to <unk>."""
        return spm_id + 1 if spm_id else XLMR_UNK

    def encode(self, text: str, max_len: int = MAX_TOKENS) -> list:
        ids = [self.piece_id(i) for i in self.sp.EncodeAsIds(text)]
        return [XLMR_BOS] + ids[:max(max_len - 2, 0)] + [XLMR_EOS]

    def batch(self, texts, ctx: Context | None = None, max_len: int = MAX_TOKENS) -> dict:
        """Texts -> padded device tensors (Text.RobertaTokenize over an array)."""
        return token_batch([self.encode(t, max_len) for t in texts], ctx)
