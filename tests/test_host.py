"""CPU-only checks: the C ABI library loads and exports every entry point the
header declares, host-side logic that runs without a GPU (broadcast shapes,
error reporting without a device), the synthetic graph builders, and the
batch-sharding path as two gloo ranks on the CPU."""
import os
import re
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol():
    from onnx_b200 import _native as N
    hdr = open(os.path.join(ROOT, "include", "lonnx.h")).read()
    declared = re.findall(r"LONNX_API\s+[\w\s\*]+?\b(lonnx_\w+)\s*\(", hdr)
    assert len(declared) > 40
    missing = [d for d in declared if not hasattr(N.lib, d)]
    assert not missing, missing
    assert set(declared) <= set(N._SIGS), set(declared) - set(N._SIGS)


def test_broadcast_shape_host_logic():
    import ctypes
    from onnx_b200 import _native as N
    out = (ctypes.c_int64 * 8)()
    r = ctypes.c_int()
    for a, b, exp in [((1, 8, 28, 28), (8, 1, 1), (1, 8, 28, 28)), ((5, 1, 7), (1, 6, 1), (5, 6, 7)),
                      ((), (3,), (3,)), ((2, 12, 128, 128), (2, 1, 1, 128), (2, 12, 128, 128))]:
        N.check(N.lib.lonnx_broadcast_shape(N.shape_arr(a), len(a), N.shape_arr(b), len(b), out, ctypes.byref(r)))
        assert tuple(out[:r.value]) == exp
    rc = N.lib.lonnx_broadcast_shape(N.shape_arr((3, 4)), 2, N.shape_arr((5,)), 1, out, ctypes.byref(r))
    assert rc == -2 and b"broadcast" in N.lib.lonnx_last_error()


def test_context_creation_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from onnx_b200 import _native as N
    from onnx_b200.tensor import Context
    with pytest.raises(N.LonnxError) as e:
        Context(0)
    assert e.value.code == -4


def test_null_arguments_return_badarg():
    from onnx_b200 import _native as N
    assert N.lib.lonnx_gemm_f32(None, None, None, None, None, 1, 1, 1, 1, 0, 0, 0, 0, 1.0, 1.0, 0) == -1
    assert N.lib.lonnx_graph_execute(None) == -1


def test_graph_builders():
    from onnx_b200 import graphs as G
    g = G.e5_encoder(layers=2, vocab=100, seq=16)
    ops = [n.op for n in g.nodes]
    assert ops.count("MatMul") == 2 * 8 and ops.count("Softmax") == 2 and ops.count("Erf") == 2
    assert g.initializers["word_embeddings"].shape == (100, 384)
    inp = G.e5_inputs(5, 16, 100)
    assert inp["input_ids"].dtype == np.int64 and inp["attention_mask"][:, 0].all()
    assert G.e5_flops_per_seq() == 5737807872
    assert len(G.mnist8().nodes) == 12


def test_oracle_e5_small_runs():
    from onnx_b200 import graphs as G
    from oracle import oracle as O
    g = G.e5_encoder(layers=1, vocab=200, seq=8)
    out = O.execute(g, G.e5_inputs(3, 8, 200))
    assert out["sentence_embedding"].shape == (3, 384)
    assert np.isfinite(out["sentence_embedding"]).all()


def test_shard_bounds():
    from onnx_b200.shard import shard_bounds
    assert [shard_bounds(256, 8, r) for r in (0, 7)] == [(0, 32), (224, 256)]
    assert [shard_bounds(5, 2, r) for r in (0, 1)] == [(0, 3), (3, 5)]
    assert shard_bounds(1, 4, 3) == (1, 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import os as _os
    import sys
    sys.path.insert(0, ROOT)
    _os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from onnx_b200 import graphs as G
    from onnx_b200.shard import run_sharded
    from oracle import oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = G.e5_encoder(layers=1, vocab=300, seq=8, seed=4)
    inp = G.e5_inputs(5, 8, 300, seed=4)
    full = run_sharded(lambda x: O.execute(g, x), inp)
    if rank == 0:
        q.put(full["sentence_embedding"])
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_replicas_gloo_world2():
    """Two CPU ranks each run their slice of the batch (CPU oracle as the
    per-rank executor) and gather on the host: the result equals one
    unsharded run, row for row."""
    import multiprocessing as mp
    from onnx_b200 import graphs as G
    from oracle import oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = G.e5_encoder(layers=1, vocab=300, seq=8, seed=4)
    ref = O.execute(g, G.e5_inputs(5, 8, 300, seed=4))["sentence_embedding"]
    assert np.array_equal(got, ref)


def _rank_fail_main(rank, world, port, q):
    import datetime
    import os as _os
    import sys
    sys.path.insert(0, ROOT)
    _os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from onnx_b200.shard import run_sharded
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))

    def execute(x):
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        return {"y": x["x"] * 2}
    try:
        run_sharded(execute, {"x": np.arange(6, dtype=np.float32).reshape(6, 1)})
        q.put((rank, "finished"))
    except Exception as e:  # rank 1: its own exception; rank 0: the gather times out / sees the peer gone
        q.put((rank, type(e).__name__))


def test_sharded_rank_failure_is_detected_gloo():
    """A rank that fails between steps: the other rank's host-side gather ends
    with an error (process-group timeout or peer loss) instead of hanging."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fail_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "RuntimeError"
    assert res[0] != "finished"


_DIV_SQRT2_C = r"""
#include <math.h>
#include <stdint.h>
#include <string.h>
/* The device helper lonnx_div_sqrt2 (onnx_b200/csrc/lonnx_internal.cuh),
   restated with libm's correctly rounded fmaf: counts the inputs among
   `count` bit patterns (start, start+step, ...) whose result differs from
   IEEE float division by fl(sqrt 2). */
static float div_sqrt2(float x) {
    const float c = 1.41421353816986083984375f, r = 0.707106769084930419921875f;
    const float ax = fabsf(x);
    if (!(ax > 0x1p-100f && ax < INFINITY)) return x / c;
    const float q0 = x * r;
    const float rem = fmaf(-q0, c, x);
    return fmaf(rem, r, q0);
}
long long mismatches(uint32_t start, uint32_t step, long long count) {
    long long bad = 0;
    uint32_t u = start;
    for (long long i = 0; i < count; ++i, u += step) {
        float x, q, ref;
        memcpy(&x, &u, 4);
        if (x != x) continue;
        volatile float c = 1.41421353816986083984375f;
        ref = x / c;
        q = div_sqrt2(x);
        uint32_t a, b;
        memcpy(&a, &ref, 4);
        memcpy(&b, &q, 4);
        bad += a != b;
    }
    return bad;
}
"""


def test_div_sqrt2_correctly_rounded(tmp_path):
    """The GELU chain's x / fl(sqrt 2) uses one Markstein correction step
    instead of a division; it must equal IEEE division bit for bit.  Every
    float in [1, 2) and [2^-100, 2^-99) plus a strided sample of all 2^32
    patterns (the full range was checked exhaustively when the helper was
    written)."""
    import ctypes
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    src = tmp_path / "d.c"
    src.write_text(_DIV_SQRT2_C)
    so = tmp_path / "d.so"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-shared", "-fPIC", "-o", str(so), str(src), "-lm"],
                   check=True)
    lib = ctypes.CDLL(str(so))
    lib.mismatches.restype = ctypes.c_longlong
    lib.mismatches.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_longlong]
    assert lib.mismatches(0x3F800000, 1, 1 << 23) == 0
    assert lib.mismatches(0x0D800000, 1, 1 << 23) == 0  # 2^-100 .. 2^-99
    assert lib.mismatches(0x80000000, 1, 1 << 23) == 0  # negative subnormals and tiny
    assert lib.mismatches(7, 997, (1 << 32) // 997) == 0


def test_bench_reference_arm_contract():
    """`bench.py --impl reference` (the reference's CPU algorithm through the
    oracle restatement, no GPU) prints one JSON line with the bench contract:
    the same metric and unit as the GPU arm, a cpu_baseline description and
    an e2e block with zero host-device bytes."""
    import json
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert line["impl"] == "reference"
    assert line["unit"] == "seq/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["metric"].startswith("e5-small encoder throughput")
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "seq/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
