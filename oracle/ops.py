"""ctypes bindings of the C oracle (oracle/ops.c). Test infrastructure only."""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "liboracle.so"

_lib = None
_F = ctypes.POINTER(ctypes.c_float)
_H = ctypes.POINTER(ctypes.c_uint16)


def build() -> Path:
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < (HERE / "ops.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def _h(a: np.ndarray):
    assert a.dtype == np.float16 and a.flags.c_contiguous
    return a.ctypes.data_as(_H)


def conv2d(x, w, stride=(1, 1), pads=(0, 0, 0, 0), dilation=(1, 1), bn=None, relu=False, residual=None,
           eps=1e-5) -> np.ndarray:
    """Direct conv (+BN [+residual] [+ReLU]) in the reference loop order."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    oh = (h + pads[0] + pads[2] - dilation[0] * (r - 1) - 1) // stride[0] + 1
    ow = (wd + pads[1] + pads[3] - dilation[1] * (s - 1) - 1) // stride[1] + 1
    y = np.empty((n, k, oh, ow), np.float32)
    mode = 0
    zeros = np.zeros(k, np.float32)
    scale = bias = mean = var = zeros
    if bn is not None:
        scale, bias, mean, var = (np.ascontiguousarray(v, np.float32) for v in bn)
        mode = 3 if residual is not None else (2 if relu else 1)
    res = np.ascontiguousarray(residual, np.float32) if residual is not None else y
    lib().oracle_conv2d(_f(x), _f(w), _f(scale), _f(bias), _f(mean), _f(var), _f(res), _f(y),
                        n, c, h, wd, k, r, s, oh, ow, stride[0], stride[1], pads[0], pads[1],
                        dilation[0], dilation[1], ctypes.c_float(eps), mode)
    return y


def batch_norm(x, scale, bias, mean, var, eps=1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    spatial = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    args = [np.ascontiguousarray(v, np.float32) for v in (scale, bias, mean, var)]
    lib().oracle_batch_norm(_f(x), *map(_f, args), _f(y), ctypes.c_long(x.size), x.shape[1], spatial,
                            ctypes.c_float(eps))
    return y


def relu(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oracle_relu(_f(x), _f(y), ctypes.c_long(x.size))
    return y


def add(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    y = np.empty_like(a)
    lib().oracle_add(_f(a), _f(b), _f(y), ctypes.c_long(a.size))
    return y


def add_relu(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    y = np.empty_like(a)
    lib().oracle_add_relu(_f(a), _f(b), _f(y), ctypes.c_long(a.size))
    return y


def max_pool(x, kernel=(3, 3), stride=(2, 2), pads=(1, 1, 1, 1), dilation=(1, 1)) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n, c, h, w = x.shape
    oh = (h + pads[0] + pads[2] - (dilation[0] * (kernel[0] - 1) + 1)) // stride[0] + 1
    ow = (w + pads[1] + pads[3] - (dilation[1] * (kernel[1] - 1) + 1)) // stride[1] + 1
    y = np.empty((n, c, oh, ow), np.float32)
    lib().oracle_max_pool(_f(x), _f(y), n, c, h, w, oh, ow, kernel[0], kernel[1], stride[0], stride[1],
                          pads[0], pads[1], dilation[0], dilation[1])
    return y


def global_average_pool(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n, c, h, w = x.shape
    y = np.empty((n, c, 1, 1), np.float32)
    lib().oracle_global_average_pool(_f(x), _f(y), n, c, h, w)
    return y


def gemm_f32(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    y = np.empty((a.shape[0], b.shape[1]), np.float32)
    lib().oracle_gemm_f32(_f(a), _f(b), _f(y), a.shape[0], b.shape[1], a.shape[1])
    return y


def gemm_f16(a, b, gelu=False) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    y = np.empty((a.shape[0], b.shape[1]), np.float16)
    lib().oracle_gemm_f16(_h(a), _h(b), _h(y), a.shape[0], b.shape[1], a.shape[1], int(gelu))
    return y


def gelu_f16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float16)
    y = np.empty_like(x)
    lib().oracle_gelu_f16(_h(x), _h(y), ctypes.c_long(x.size))
    return y


def add_f16(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    y = np.empty_like(a)
    lib().oracle_add_f16(_h(a), _h(b), _h(y), ctypes.c_long(a.size))
    return y


def layer_norm_f16(x, scale, bias, residual=None, eps=1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float16)
    rows, cols = x.shape
    y = np.empty_like(x)
    scratch = np.empty(cols, np.float32)
    res = _h(np.ascontiguousarray(residual, np.float16)) if residual is not None else None
    lib().oracle_layer_norm_f16(_h(x), res, _h(np.ascontiguousarray(scale, np.float16)),
                                _h(np.ascontiguousarray(bias, np.float16)), _h(y), rows, cols,
                                ctypes.c_float(eps), _f(scratch))
    return y


def softmax_f16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float16)
    y = np.empty_like(x)
    lib().oracle_softmax_f16(_h(x), _h(y), x.shape[0], x.shape[1])
    return y


def _declare() -> None:
    l = lib()
    l.oracle_layer_norm_f16.argtypes = [_H, _H, _H, _H, _H, ctypes.c_int, ctypes.c_int, ctypes.c_float, _F]


_declare()
