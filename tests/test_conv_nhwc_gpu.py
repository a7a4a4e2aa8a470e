"""The NHWC conv chain (graph.cpp mark_nhwc): conv-chain values stored as
[N, H, W, C] between tensor-core convs, MaxPool and the global average pool.

The layout changes no sum: the 1x1 convs contract their channels in the same
order from either layout, the 3x3 convs gather NHWC in both modes, the
epilogue applies alpha, bias, residual and Relu in the same order, MaxPool
is exact and the H x W reduction reproduces the NCHW kernel's order.  So
every output must be bit-identical to the same graph run with the pass off
(LONNX_CONV_NHWC=0, read once per process: each mode runs in a child
process), and within the parity rule of the oracle, which restates the
reference's Conv / MaxPool / ReduceMean (TensorOps.cs:903-962,1025-1099,
1610-1839).
"""
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from conftest import close
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r'''
import sys, numpy as np
sys.path.insert(0, %r)
sys.path.insert(0, %r)
from onnx_b200.tensor import Context
from onnx_b200.graph import ComputationalGraph
import nhwc_cases
ctx = Context(0)
g, feed, outs = nhwc_cases.build(sys.argv[2])
cg = ComputationalGraph(g, ctx, honor_conv_attrs=True)
l0 = ctx.launches
res = cg.execute(feed)
launches = ctx.launches - l0
np.savez(sys.argv[1], launches=launches, **{k: res[k] for k in outs})
print("ok")
'''


def _run(case, nhwc):
    with tempfile.TemporaryDirectory() as d:
        f = os.path.join(d, "out.npz")
        env = dict(os.environ)
        env.pop("LONNX_CONV_NHWC", None)
        if not nhwc:
            env["LONNX_CONV_NHWC"] = "0"
        code = _CHILD % (ROOT, os.path.join(ROOT, "tests"))
        r = subprocess.run([sys.executable, "-c", code, f, case], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
        z = np.load(f)
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("case", ["resnet50_small", "mixed_readers", "projection_residual", "pool_shapes"])
def test_nhwc_chain_bit_identical_and_vs_oracle(case):
    import nhwc_cases
    on, off = _run(case, True), _run(case, False)
    g, feed, outs = nhwc_cases.build(case)
    ref = O.execute(g, feed, honor_conv_attrs=True)
    for k in outs:
        assert np.array_equal(on[k], off[k]), (case, k, float(np.abs(on[k] - off[k]).max()))
        close(on[k], ref[k])
    # the pass ran: NCHW mode pays a transpose in front of every 3x3 conv
    if nhwc_cases.has_3x3(case):
        assert int(on["launches"]) < int(off["launches"]), (int(on["launches"]), int(off["launches"]))
