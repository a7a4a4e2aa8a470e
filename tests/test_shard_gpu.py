"""Batch sharding on the GPU executor: two ranks (gloo, two processes on
cuda:0) each run their contiguous slice of a batch through their own graph
replica and gather the pooled embeddings on the host in rank order.  The
concatenation must equal one full-batch run bit for bit -- every op is
row-independent and the GEMMs never split K by batch size, so a sequence's
embedding does not depend on which rows share its GPU."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BATCH, SEQ, VOCAB = 13, 64, 3000  # odd batch: shards of 7 and 6 rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.shard import run_sharded
    from onnx_b200.tensor import Context
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = G.e5_encoder(layers=2, vocab=VOCAB, seq=SEQ, seed=6)
    cg = ComputationalGraph(g, Context(0))
    out = run_sharded(lambda sl: {"e": cg.execute(sl)["sentence_embedding"]}, G.e5_inputs(BATCH, SEQ, VOCAB, seed=6))
    if rank == 0:
        q.put(out["e"])
    dist.destroy_process_group()


def test_sharded_gpu_replicas_match_full_batch(ctx):
    import multiprocessing as mp
    from onnx_b200 import graphs as G
    from onnx_b200.graph import ComputationalGraph
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = G.e5_encoder(layers=2, vocab=VOCAB, seq=SEQ, seed=6)
    full = ComputationalGraph(g, ctx).execute(G.e5_inputs(BATCH, SEQ, VOCAB, seed=6))["sentence_embedding"]
    assert got.shape == full.shape == (BATCH, 384)
    assert np.array_equal(got, full)
