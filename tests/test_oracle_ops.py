"""The C oracle (oracle/ops.c) against independent float64 / PyTorch
computations on small ragged shapes, for every op the GPU parity tests
compare against: dilated and residual convolutions, BatchNorm, the
elementwise ops, pooling, both GEMMs, GELU, (Skip)LayerNorm and Softmax.
CPU only; the oracle is test infrastructure and this pins it."""

from __future__ import annotations

from math import erf

import numpy as np
import pytest

from oracle import ops as oracle
from tests.helpers import assert_close

def _bn(rng, k):
    return (rng.uniform(0.5, 1.5, k).astype(np.float32), rng.normal(0, 0.1, k).astype(np.float32),
            rng.normal(0, 0.1, k).astype(np.float32), rng.uniform(0.5, 1.5, k).astype(np.float32))


def _torch_bn(t, bn, torch):
    scale, bias, mean, var = (torch.from_numpy(v).double() for v in bn)
    return torch.nn.functional.batch_norm(t, mean, var, scale, bias, training=False, eps=1e-5)


@pytest.mark.parametrize("stride,pads,dilation", [((1, 1), (2, 3, 2, 3), (2, 3)), ((3, 2), (0, 1, 0, 1), (1, 2))])
def test_conv_dilated_strided_vs_torch(stride, pads, dilation):
    rng = np.random.default_rng(101)
    import torch
    import torch.nn.functional as F

    x = rng.standard_normal((2, 6, 13, 17)).astype(np.float32)
    w = rng.standard_normal((5, 6, 3, 3)).astype(np.float32)
    bn = _bn(rng, 5)
    ours = oracle.conv2d(x, w, stride=stride, pads=pads, dilation=dilation, bn=bn, relu=True)
    xt = F.pad(torch.from_numpy(x).double(), (pads[1], pads[3], pads[0], pads[2]))
    t = F.conv2d(xt, torch.from_numpy(w).double(), stride=stride, dilation=dilation)
    t = F.relu(_torch_bn(t, bn, torch))
    assert_close(ours, t.numpy(), atol=1e-5, rtol=1e-5, what=f"conv {stride} {pads} {dilation}")


def test_conv_bn_residual_relu_vs_torch():
    rng = np.random.default_rng(102)
    import torch
    import torch.nn.functional as F

    x = rng.standard_normal((3, 8, 7, 9)).astype(np.float32)
    w = rng.standard_normal((4, 8, 1, 1)).astype(np.float32)
    bn = _bn(rng, 4)
    res = rng.standard_normal((3, 4, 7, 9)).astype(np.float32)
    ours = oracle.conv2d(x, w, bn=bn, residual=res)
    t = _torch_bn(F.conv2d(torch.from_numpy(x).double(), torch.from_numpy(w).double()), bn, torch)
    t = F.relu(t + torch.from_numpy(res).double())
    assert_close(ours, t.numpy(), atol=1e-5, rtol=1e-5, what="conv+bn+residual+relu")


def test_batch_norm_and_elementwise():
    rng = np.random.default_rng(103)
    import torch

    x = rng.standard_normal((2, 5, 3, 7)).astype(np.float32)
    b = rng.standard_normal(x.shape).astype(np.float32)
    bn = _bn(rng, 5)
    assert_close(oracle.batch_norm(x, *bn), _torch_bn(torch.from_numpy(x).double(), bn, torch).numpy(),
                 atol=1e-5, rtol=1e-5, what="batch_norm")
    # Elementwise FP32 ops are one rounding each: bit-exact against numpy.
    assert np.array_equal(oracle.relu(x), np.maximum(x, 0))
    assert np.array_equal(oracle.add(x, b), x + b)
    assert np.array_equal(oracle.add_relu(x, b), np.maximum(x + b, 0))


@pytest.mark.parametrize("kernel,stride,pads,dilation", [((3, 3), (2, 2), (1, 1, 1, 1), (1, 1)),
                                                         ((2, 3), (1, 2), (0, 1, 0, 1), (1, 1)),
                                                         ((3, 2), (2, 1), (1, 0, 1, 0), (2, 1))])
def test_max_pool_shapes_vs_torch(kernel, stride, pads, dilation):
    rng = np.random.default_rng(104)
    import torch
    import torch.nn.functional as F

    x = rng.standard_normal((2, 3, 11, 8)).astype(np.float32)
    ours = oracle.max_pool(x, kernel=kernel, stride=stride, pads=pads, dilation=dilation)
    ref = F.max_pool2d(torch.from_numpy(x), kernel_size=kernel, stride=stride, padding=(pads[0], pads[1]),
                       dilation=dilation).numpy()
    assert np.array_equal(ours, ref)  # a max is exact


def test_max_pool_nan_is_maxnum():
    """The reference reduces with tl.maximum(acc, tap) from acc = -inf
    (resnet.py:171-181); its default NaN mode is IEEE maxNum, which returns
    the non-NaN operand. np.fmax has the same rule, so a window reduction
    with np.fmax from -inf is an independent statement of the reference."""
    rng = np.random.default_rng(106)
    x = rng.standard_normal((2, 3, 9, 10)).astype(np.float32)
    x.flat[::4] = np.nan
    x[0, 0, :2, :2] = np.nan  # the whole in-range window of output (0, 0, 0, 0)
    ours = oracle.max_pool(x)
    n, c, h, w = x.shape
    oh, ow = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    expected = np.full((n, c, oh, ow), -np.inf, np.float32)
    for i in range(oh):
        for j in range(ow):
            for a in range(3):
                for b in range(3):
                    ih, iw = 2 * i - 1 + a, 2 * j - 1 + b
                    if 0 <= ih < h and 0 <= iw < w:
                        expected[:, :, i, j] = np.fmax(expected[:, :, i, j], x[:, :, ih, iw])
    assert np.array_equal(ours, expected)
    assert ours[0, 0, 0, 0] == -np.inf


def test_gemm_f32_vs_float64():
    rng = np.random.default_rng(105)
    a = rng.standard_normal((19, 67)).astype(np.float32)
    b = rng.standard_normal((67, 23)).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert_close(oracle.gemm_f32(a, b), ref, atol=1e-4, rtol=1e-5, what="gemm f32")


def _gelu64(v):
    return 0.5 * v * (1.0 + np.vectorize(erf)(v / np.sqrt(2.0)))


def _ulps_f16(a, b):
    """Distance in FP16 units in the last place (same-sign values)."""
    ai = a.astype(np.float16).view(np.int16).astype(np.int32)
    bi = b.astype(np.float16).view(np.int16).astype(np.int32)
    return np.abs(ai - bi)


def test_gelu_f16_vs_exact_erf():
    rng = np.random.default_rng(106)
    x = np.linspace(-6, 6, 4001).astype(np.float16)
    ours = oracle.gelu_f16(x)
    ref = _gelu64(x.astype(np.float64))
    # FP32 math then one rounding to FP16: within one FP16 ulp of the exact value.
    big = np.abs(ref) > 1e-3
    assert _ulps_f16(ours[big], ref[big]).max() <= 1
    assert np.abs(ours[~big].astype(np.float64) - ref[~big]).max() < 1e-3


def test_gemm_gelu_f16_vs_float64():
    rng = np.random.default_rng(107)
    a = (rng.standard_normal((9, 96)) * 0.5).astype(np.float16)
    b = (rng.standard_normal((96, 40)) * 0.2).astype(np.float16)
    acc = a.astype(np.float64) @ b.astype(np.float64)
    assert_close(oracle.gemm_f16(a, b), acc, atol=2e-3, rtol=2e-3, what="gemm f16")
    assert_close(oracle.gemm_f16(a, b, gelu=True), _gelu64(acc), atol=2e-3, rtol=2e-3, what="gemm gelu f16")


@pytest.mark.parametrize("with_residual", [False, True])
def test_layer_norm_f16_vs_float64(with_residual):
    rng = np.random.default_rng(108)
    x = rng.standard_normal((7, 300)).astype(np.float16)
    res = rng.standard_normal((7, 300)).astype(np.float16) if with_residual else None
    gamma = rng.uniform(0.5, 1.5, 300).astype(np.float16)
    beta = rng.normal(0, 0.1, 300).astype(np.float16)
    ours = oracle.layer_norm_f16(x, gamma, beta, residual=res)
    v = x.astype(np.float64) + (res.astype(np.float64) if with_residual else 0.0)
    mean = v.mean(axis=1, keepdims=True)
    var = ((v - mean) ** 2).mean(axis=1, keepdims=True)
    ref = (v - mean) / np.sqrt(var + 1e-5) * gamma.astype(np.float64) + beta.astype(np.float64)
    # FP32 statistics, one FP16 rounding of the result (half an ulp is 4.9e-4 relative).
    assert_close(ours, ref, atol=1e-3, rtol=1e-3, what=f"layer norm residual={with_residual}")


def test_softmax_f16_vs_float64():
    rng = np.random.default_rng(109)
    x = (rng.standard_normal((5, 129)) * 4).astype(np.float16)
    ours = oracle.softmax_f16(x)
    v = x.astype(np.float64)
    e = np.exp(v - v.max(axis=1, keepdims=True))
    ref = e / e.sum(axis=1, keepdims=True)
    assert_close(ours, ref, atol=1e-3, rtol=2e-3, what="softmax")
    assert np.allclose(ours.astype(np.float64).sum(axis=1), 1.0, atol=2e-2)
