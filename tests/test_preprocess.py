"""Pre-processing before the model, host side (no GPU): the oracle's
restatements of Images.ImageToArrayF (src/Lokad.Onnx.Data/Images.cs:92-103)
and of the padding loop of Text.RobertaTokenize (Text.cs:126-140), and the
XLM-R id conventions of the tokenizer wrapper.

The image oracle is pinned to the committed mnist fixture, which the
generator (tests/golden/make_mnist8_fixture.py) made from the reference's
own test images with Images.cs:166-183's steps."""
import io
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("digit", [4, 2, 5])
def test_image_oracle_matches_fixture(digit):
    from onnx_b200.preprocess import decode_image
    rgba = decode_image(os.path.join(GOLDEN, f"mnist{digit}.png"), mnist=True)
    assert rgba.shape == (28, 28, 4) and rgba.dtype == np.uint8
    ref = np.load(os.path.join(GOLDEN, "mnist8.npz"))[f"image/mnist{digit}"]
    assert np.array_equal(O.image_to_array_f(rgba), ref)


def test_image_oracle_arithmetic():
    """((R + G + B) / 3.0f) / 255.0f: the alpha channel is ignored, white is
    exactly 1, and each division is one float32 rounding."""
    px = np.array([[[255, 255, 255, 0], [0, 0, 0, 255], [1, 2, 4, 9], [200, 13, 77, 128]]], np.uint8)
    got = O.image_to_array_f(px).reshape(-1)
    want = [np.float32(np.float32(s) / np.float32(3)) / np.float32(255) for s in (765, 0, 7, 290)]
    assert got.dtype == np.float32 and list(got) == want
    assert got[0] == 1.0 and got[1] == 0.0


def test_roberta_pad_reference_semantics():
    ids, mask, types = O.roberta_pad([[0, 10, 2], [0, 11, 12, 13, 2], [0, 2]])
    assert ids.tolist() == [[0, 10, 2, 1, 1], [0, 11, 12, 13, 2], [0, 2, 1, 1, 1]]
    assert mask.tolist() == [[1, 1, 1, 0, 0], [1, 1, 1, 1, 1], [1, 1, 0, 0, 0]]
    assert types.tolist() == [[0] * 5] * 3
    assert ids.dtype == mask.dtype == types.dtype == np.int64


def _tiny_model():
    """A small SentencePiece model trained in memory (the multilingual-e5
    model file is not shipped), with XLM-R's SentencePiece layout: <unk> 0,
    <s> 1, </s> 2, pieces from 3."""
    spm = pytest.importorskip("sentencepiece")
    text = ["the quick brown fox jumps over the lazy dog", "a b c d e f g h i j k l m n o p",
            "graphics processing units run kernels", "tokens padded to the longest sequence"] * 20
    buf = io.BytesIO()
    spm.SentencePieceTrainer.train(sentence_iterator=iter(text), model_writer=buf, vocab_size=40,
                                   model_type="unigram", character_coverage=1.0, minloglevel=2)
    return buf.getvalue()


def test_xlmr_tokenizer_conventions():
    from onnx_b200.preprocess import XLMR_BOS, XLMR_EOS, XLMR_UNK, XLMRobertaTokenizer
    tok = XLMRobertaTokenizer(model_proto=_tiny_model())
    ids = tok.encode("the quick fox")
    raw = tok.sp.EncodeAsIds("the quick fox")
    assert ids[0] == XLMR_BOS and ids[-1] == XLMR_EOS
    assert ids[1:-1] == [i + 1 if i else XLMR_UNK for i in raw]  # SentencePiece ids shifted past the specials
    assert all(i >= 4 or i == XLMR_UNK for i in ids[1:-1])
    assert XLMR_UNK in tok.encode("中")  # a character the model never saw
    long = tok.encode("a b c d e f g h " * 200)
    assert len(long) == 512 and long[0] == XLMR_BOS and long[-1] == XLMR_EOS  # OnlyFirst truncation at 512
    assert len(tok.encode("a b c", max_len=4)) == 4
