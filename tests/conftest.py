import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    # the library is built in-tree; build it when a checkout has none yet
    if not os.path.exists(os.path.join(ROOT, "onnx_b200", "liblonnx_cuda.so")):
        from onnx_b200 import build
        build.build()


@pytest.fixture(scope="session")
def ctx():
    from onnx_b200.tensor import Context
    return Context.default(0)


def close(gpu, ref, atol=1e-4, rtol=1e-4):
    """Parity rule: |gpu - ref| <= atol + rtol * |ref| element-wise."""
    import numpy as np
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    err = np.abs(gpu - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{bad.sum()} of {bad.size} elements out of tolerance; worst at {i}: "
                             f"gpu={gpu[i]!r} ref={ref[i]!r} err={err[i]:.3g}")
    return float(err.max()) if err.size else 0.0
