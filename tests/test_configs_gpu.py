"""Parity of the benchmarked configurations themselves against the oracle.

Each test runs the exact graph, weights and inputs the benchmark times --
the 12-layer full-width e5-shaped encoder at batch 256 and at batch 32, and
ResNet-50 at batch 64 x 3 x 224 x 224 -- on the GPU, and compares a sample of
the batch rows with the oracle run on those rows alone.  Every op of both
models is independent across batch rows (no reduction mixes rows; the GEMMs
and convs never split K by batch size), so the sampled rows of the full-batch
GPU run must equal what the oracle computes for them, within the parity rule
|gpu - ref| <= 1e-4 + 1e-4 |ref|.  The worst errors are printed (run with -s)
so they can be quoted.

The reference computes these graphs with ComputationalGraph.Execute
(src/Lokad.Onnx.Backend/ComputationalGraph.cs:199-272); the oracle restates
that executor and its CPU kernels.
"""
import numpy as np
import pytest

from conftest import close
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SEQ = 128


def _err_report(what, gpu, ref):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(gpu - ref)
    rel = err / np.maximum(np.abs(ref), 1e-30)
    big = np.abs(ref) > 1e-3
    print(f"\n[parity] {what}: max abs {err.max():.3e}, max rel (|ref|>1e-3) "
          f"{(rel[big].max() if big.any() else 0.0):.3e}, max err/bound "
          f"{(err / (1e-4 + 1e-4 * np.abs(ref))).max():.3f}")


@pytest.fixture(scope="module")
def e5_bench_graph():
    """The benchmark's graph: 12 layers, hidden 384, 12 heads, FFN 1536,
    vocab 250037, seq 128, weights N(0, 0.02) from seed 0."""
    from onnx_b200 import graphs as G
    g = G.e5_encoder(seq=SEQ, seed=0)
    return g


def _e5_rows_vs_oracle(ctx, g, batch, seed, rows):
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    inp = G.e5_inputs(batch, SEQ, seed=seed)
    cg = ComputationalGraph(g, ctx)
    got = cg.execute(inp)
    del cg
    sub = {k: np.ascontiguousarray(v[rows]) for k, v in inp.items()}
    ref = O.execute(g, sub)
    for name in g.outputs:
        _err_report(f"e5 batch {batch} rows {list(rows)[:4]}.. output {name}", got[name][rows], ref[name])
        close(got[name][rows], ref[name])


def test_e5_12_layers_batch256_bench_rows(ctx, e5_bench_graph):
    """The headline workload: the batch-256 inputs of the benchmark (seed 100),
    all 256 rows run on the GPU, rows 0-7 and 248-255 checked."""
    rows = np.r_[0:8, 248:256]
    _e5_rows_vs_oracle(ctx, e5_bench_graph, 256, 100, rows)


def test_e5_12_layers_batch32(ctx, e5_bench_graph):
    """The batch-32 configuration (the benchmark's seed-7 inputs), where the
    executor picks 128-wide GEMM tiles; a spread of rows checked."""
    rows = np.array([0, 5, 11, 17, 23, 31])
    _e5_rows_vs_oracle(ctx, e5_bench_graph, 32, 7, rows)


def test_resnet50_224_batch64_vs_oracle(ctx):
    """ResNet-50 v1 at the benchmarked input: batch 64 x 3 x 224 x 224 from
    seed 0 on the GPU, images 0 and 63 against the oracle with the Conv
    attributes applied."""
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    g = G.resnet50(seed=0)
    x = np.random.default_rng(0).uniform(0, 1, (64, 3, 224, 224)).astype(np.float32)
    got = ComputationalGraph(g, ctx, honor_conv_attrs=True).execute({"data": x})["logits"]
    for i in (0, 63):
        ref = O.execute(g, {"data": x[i:i + 1]}, honor_conv_attrs=True)["logits"]
        _err_report(f"resnet50 224^2 image {i}", got[i:i + 1], ref)
        close(got[i:i + 1], ref)
