"""ctypes binding of liblonnx_cuda.so (the C ABI declared in include/lonnx.h).

The product path has no CPU fallback: importing this module fails loudly when
the library is missing, and creating a context fails when no B200 is visible.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("LONNX_LIBRARY") or os.path.join(_HERE, "liblonnx_cuda.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m onnx_b200.build` "
                      "(there is no CPU fallback for this path)")

lib = ctypes.CDLL(LIB_PATH)

c_int, c_i64, c_f32, c_size, c_vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
i64p = ctypes.POINTER(ctypes.c_int64)
c_char_p = ctypes.c_char_p

_SIGS = {
    "lonnx_ctx_create": (c_int, [c_int, ctypes.POINTER(c_vp)]),
    "lonnx_ctx_destroy": (c_int, [c_vp]),
    "lonnx_ctx_device": (c_int, [c_vp]),
    "lonnx_ctx_stream": (c_vp, [c_vp]),
    "lonnx_malloc": (c_int, [c_vp, c_size, ctypes.POINTER(c_vp)]),
    "lonnx_free": (c_int, [c_vp, c_vp]),
    "lonnx_memcpy_h2d": (c_int, [c_vp, c_vp, c_vp, c_size]),
    "lonnx_memcpy_d2h": (c_int, [c_vp, c_vp, c_vp, c_size]),
    "lonnx_memcpy_d2d": (c_int, [c_vp, c_vp, c_vp, c_size]),
    "lonnx_memset": (c_int, [c_vp, c_vp, c_int, c_size]),
    "lonnx_sync": (c_int, [c_vp]),
    "lonnx_last_error": (c_char_p, []),
    "lonnx_launch_count": (c_i64, [c_vp]),
    "lonnx_debug_expire_wait": (c_int, [c_vp, c_i64]),
    "lonnx_broadcast_shape": (c_int, [i64p, c_int, i64p, c_int, i64p, ctypes.POINTER(c_int)]),
    "lonnx_binary_f32": (c_int, [c_vp, c_int, c_vp, i64p, c_int, c_vp, i64p, c_int, c_vp]),
    "lonnx_unary_f32": (c_int, [c_vp, c_int, c_vp, c_vp, c_i64]),
    "lonnx_gemm_f32": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_i64,
                               c_i64, c_int, c_f32, c_f32, c_int]),
    "lonnx_gemm_f32_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_i64,
                                       c_i64, c_int, c_f32, c_f32, c_int]),
    "lonnx_gemm_f32_noalloc_status": (c_int, [c_vp]),
    "lonnx_matmul_f32": (c_int, [c_vp, c_vp, i64p, c_int, c_vp, i64p, c_int, c_vp]),
    "lonnx_conv2d_f32": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp] + [c_int] * 17),
    "lonnx_softmax_f32": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64]),
    "lonnx_layernorm_f32": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_f32, c_vp, c_i64, c_int]),
    "lonnx_reduce_f32": (c_int, [c_vp, c_int, c_vp, i64p, c_int, i64p, c_int, c_vp]),
    "lonnx_maxpool2d_f32": (c_int, [c_vp, c_vp, c_vp] + [c_int] * 12),
    "lonnx_gather": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "lonnx_transpose": (c_int, [c_vp, c_vp, c_int, i64p, c_int, i64p, c_vp]),
    "lonnx_cast_i64_f32": (c_int, [c_vp, c_vp, c_vp, c_i64]),
    "lonnx_image_rgba_to_f32": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64]),
    "lonnx_token_batch_pad": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "lonnx_batchnorm_f32": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_f32, c_vp, c_i64, c_i64, c_i64]),
    "lonnx_attention_f32": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_int, c_int, c_int,
                                    c_int, c_f32]),
    "lonnx_graph_create": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "lonnx_graph_destroy": (c_int, [c_vp]),
    "lonnx_graph_add_initializer": (c_int, [c_vp, c_char_p, c_int, i64p, c_int, c_vp]),
    "lonnx_graph_add_node": (c_int, [c_vp, c_char_p, ctypes.POINTER(c_char_p), c_int,
                                     ctypes.POINTER(c_char_p), c_int]),
    "lonnx_graph_attr_int": (c_int, [c_vp, c_char_p, c_i64]),
    "lonnx_graph_attr_ints": (c_int, [c_vp, c_char_p, i64p, c_int]),
    "lonnx_graph_attr_float": (c_int, [c_vp, c_char_p, c_f32]),
    "lonnx_graph_attr_string": (c_int, [c_vp, c_char_p, c_char_p]),
    "lonnx_graph_attr_floats": (c_int, [c_vp, c_char_p, ctypes.POINTER(c_f32), c_int]),
    "lonnx_graph_attr_tensor": (c_int, [c_vp, c_char_p, c_int, i64p, c_int, c_vp]),
    "lonnx_graph_add_output": (c_int, [c_vp, c_char_p]),
    "lonnx_graph_set_opset": (c_int, [c_vp, c_int]),
    "lonnx_graph_prepare": (c_int, [c_vp, c_int]),
    "lonnx_graph_set_input": (c_int, [c_vp, c_char_p, c_int, i64p, c_int, c_vp]),
    "lonnx_graph_set_input_device": (c_int, [c_vp, c_char_p, c_int, i64p, c_int, c_vp]),
    "lonnx_graph_execute": (c_int, [c_vp]),
    "lonnx_graph_output_shape": (c_int, [c_vp, c_char_p, i64p, ctypes.POINTER(c_int)]),
    "lonnx_graph_output_dtype": (c_int, [c_vp, c_char_p, ctypes.POINTER(c_int)]),
    "lonnx_graph_output_device": (c_int, [c_vp, c_char_p, ctypes.POINTER(c_vp)]),
    "lonnx_graph_get_output": (c_int, [c_vp, c_char_p, c_vp, c_size]),
    "lonnx_graph_reset": (c_int, [c_vp]),
    "lonnx_graph_capture": (c_int, [c_vp]),
    "lonnx_graph_replay": (c_int, [c_vp]),
    "lonnx_graph_num_steps": (c_int, [c_vp]),
}

for _name, (_res, _args) in _SIGS.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args

STATUS = {0: "OK", -1: "BADARG", -2: "SHAPE", -3: "OOM", -4: "CUDA", -5: "TIMEOUT", -6: "OOB",
          -7: "UNSUPPORTED"}


class LonnxError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"[{STATUS.get(code, code)}] {message}")
        self.code = code
        self.message = message


def check(rc: int) -> None:
    if rc != 0:
        raise LonnxError(rc, lib.lonnx_last_error().decode(errors="replace"))


def shape_arr(shape):
    n = len(shape)
    arr = (ctypes.c_int64 * max(n, 1))(*[int(s) for s in shape])
    return arr


def exported_symbols():
    """Names declared in include/lonnx.h that the loaded library exports."""
    return [n for n in _SIGS if hasattr(lib, n)]
