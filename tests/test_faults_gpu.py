"""Failure detection on the GPU without faulting it: every failure here is
made on the host or by a bounded device wait that is allowed to expire.
The reference maps failures to OpResult.Failure (src/Lokad.Onnx.Backend/OpResult.cs:34-62)
and stops the executor at the first failed node (ComputationalGraph.cs:245-250)."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_expired_device_wait_reports_timeout_and_context_survives(ctx):
    from onnx_b200 import _native as N
    from onnx_b200.provider import CUDAExecutionProvider as P
    N.check(N.lib.lonnx_debug_expire_wait(ctx.handle, 2_000_000))  # ~1 ms
    with pytest.raises(N.LonnxError) as e:
        ctx.sync()
    assert e.value.code == -5
    ctx.sync()  # flag cleared
    r = P.Add(np.ones(3, np.float32), np.ones(3, np.float32))
    assert r.Status == "Success" and np.array_equal(r.Outputs[0], [2, 2, 2])


_OOM = r"""
import sys, numpy as np
sys.path.insert(0, {root!r})
from onnx_b200 import _native as N, graphs as G
from onnx_b200.tensor import Context, DeviceTensor
from onnx_b200.graph import ComputationalGraph
ctx = Context(0)
try:
    DeviceTensor(ctx, (64 << 20,), np.float32)          # 256 MB > cap
    print("NO-OOM")
except N.LonnxError as e:
    print("OOM", e.code)
small = DeviceTensor.from_host(ctx, np.arange(8, dtype=np.float32))   # still works under the cap
print("OK", small.to_host().sum())
"""


def test_allocation_cap_reports_oom():
    env = dict(os.environ, LONNX_MEM_LIMIT=str(64 << 20))
    out = subprocess.run([sys.executable, "-c", _OOM.format(root=ROOT)], env=env, capture_output=True, text=True,
                         timeout=120).stdout
    assert "OOM -3" in out and "OK 28.0" in out, out


def test_graph_failure_stops_with_message(ctx):
    """A node that cannot run (incompatible broadcast) fails the execution with
    the op's message instead of producing outputs."""
    from onnx_b200 import _native as N
    from onnx_b200.graph import ComputationalGraph
    from onnx_b200.graphs import GraphDef, Node
    g = GraphDef([Node("Add", ["a", "b"], ["c"]), Node("Relu", ["c"], ["d"])], {}, ["a", "b"], ["d"])
    cg = ComputationalGraph(g, ctx)
    with pytest.raises(N.LonnxError) as e:
        cg.execute({"a": np.ones((3, 4), np.float32), "b": np.ones((5,), np.float32)})
    assert e.value.code == -2 and "broadcast" in e.value.message
    out = cg.execute({"a": np.ones((3, 4), np.float32), "b": np.ones((4,), np.float32)})["d"]
    assert np.array_equal(out, 2 * np.ones((3, 4)))
