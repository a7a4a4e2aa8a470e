"""Pre-processing on the device (csrc/preprocess.cu) against the oracle's
restatements of Images.ImageToArrayF (src/Lokad.Onnx.Data/Images.cs:92-103)
and of Text.RobertaTokenize's padding loop (Text.cs:126-140): bit-exact.
End to end, the reference's MNIST test images decoded from their PNG files
and converted on the GPU give the reference's known answers through its
mnist-8 model (tests/Lokad.Onnx.Backend.Tests/GraphTests.cs:15-30)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("n,h,w", [(1, 28, 28), (5, 37, 53), (3, 224, 224), (2, 1, 1)])
def test_rgba_to_tensor_bit_exact(ctx, n, h, w):
    from onnx_b200.preprocess import rgba_to_tensor
    rgba = np.random.default_rng(n * h + w).integers(0, 256, (n, h, w, 4), dtype=np.uint8)
    rgba[0, 0, 0, :3] = 255  # white is exactly 1
    got = rgba_to_tensor(rgba, ctx).to_host()
    assert got.shape == (n, 1, h, w) and got.dtype == np.float32
    for i in range(n):
        assert np.array_equal(got[i:i + 1], O.image_to_array_f(rgba[i]))
    assert got[0, 0, 0, 0] == 1.0


def test_image_files_to_mnist_known_answers(ctx):
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.preprocess import load_images
    digits = (4, 2, 5)
    x = load_images([os.path.join(GOLDEN, f"mnist{d}.png") for d in digits], mnist=True, ctx=ctx)
    host = x.to_host()
    arr = np.load(os.path.join(GOLDEN, "mnist8.npz"))
    cg = ComputationalGraph.load(os.path.join(GOLDEN, "mnist-8.onnx"), ctx)
    for i, (digit, thresh) in enumerate(zip(digits, (0.9, 0.9, 0.48))):
        assert np.array_equal(host[i:i + 1], arr[f"image/mnist{digit}"])
        out = cg.execute({"Input3": host[i:i + 1]})["Plus214_Output_0"]
        p = O.softmax(out.reshape(-1))
        assert p.argmax() == digit and p[digit] > thresh


@pytest.mark.parametrize("lens", [[3, 5, 2], [7], [1, 1, 1, 1], [128] * 4 + [17, 0, 64]])
def test_token_batch_bit_exact(ctx, lens):
    from onnx_b200.preprocess import token_batch
    rng = np.random.default_rng(sum(lens))
    seqs = [list(rng.integers(4, 250000, n)) for n in lens]
    got = token_batch(seqs, ctx)
    ids, mask, types = O.roberta_pad(seqs)
    assert np.array_equal(got["input_ids"].to_host(), ids)
    assert np.array_equal(got["attention_mask"].to_host(), mask)
    assert np.array_equal(got["token_type_ids"].to_host(), types)


def test_token_batch_feeds_encoder(ctx):
    """Ragged sequences padded on the device run through the encoder exactly
    as the same padded tensors uploaded from the host."""
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.preprocess import token_batch
    g = G.e5_encoder(layers=2, vocab=1000, seq=24, seed=2)
    rng = np.random.default_rng(5)
    seqs = [[0] + list(rng.integers(4, 1000, n)) + [2] for n in (22, 9, 15)]
    dev = token_batch(seqs, ctx)
    ids, mask, types = O.roberta_pad(seqs)
    host = {"input_ids": ids, "attention_mask": mask, "token_type_ids": types}
    a = ComputationalGraph(g, ctx).execute(dev)
    b = ComputationalGraph(g, ctx).execute(host)
    for k in g.outputs:
        assert np.array_equal(a[k], b[k])
