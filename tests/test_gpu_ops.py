"""Per-op parity on the GPU: single-node graphs compiled by the engine and
run through the C ABI, every candidate of the op (pack variants and unfused
decompositions), against the C oracle on the same seeded inputs.

Tolerances: MaxPool, ReLU, Add, AddRelu and FP16 Add are bit-exact; FP32
convolution/GEMM 1e-4 abs + 1e-4 rel (the reference's own check,
tests/cpp/test_cuda.cpp:168-180 and benchmarks/resnet50_compare.py:199-200)
scaled by sqrt(K)/sqrt(64) for long reductions; FP16 paths 2e-2 abs + 2e-2 rel
(test_cuda.cpp:432); BN/GAP 1e-5 rel.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

import cutriton_b200 as ct
from oracle import ops as oracle
from tests.helpers import assert_bitexact, assert_close, run_graph

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)


def randn(*shape, dtype=np.float32, scale=1.0):
    return (RNG.standard_normal(shape) * scale).astype(dtype)


def bn_params(c):
    return (RNG.uniform(0.5, 1.5, c).astype(np.float32), (RNG.standard_normal(c) * 0.1).astype(np.float32),
            (RNG.standard_normal(c) * 0.1).astype(np.float32), RNG.uniform(0.5, 1.5, c).astype(np.float32))


def conv_model(x_shape, w, stride, pad, op, residual_shape=None, dilation=(1, 1)):
    model = ct.Model()
    model.add_input("x", list(x_shape))
    model.add_constant("w", w, layout="OIHW")
    k = w.shape[0]
    names = ["x", "w"]
    if op != "Conv":
        for n, v in zip(("scale", "bias", "mean", "var"), bn_params(k)):
            model.add_constant(n, v, layout="")
            names.append(n)
    if op == "FusedConvBatchNormAddRelu":
        model.add_input("res", list(residual_shape))
        names.append("res")
    attrs = dict(strides=list(stride), pads=[pad[0], pad[1], pad[0], pad[1]], dilations=list(dilation))
    if op != "Conv":
        attrs["batchnorm_epsilon"] = 1e-5
    model.add_node("conv", op, names, ["y"], **attrs)
    model.add_output("y")
    return model


CONV_CASES = [
    # (N, C, H, W, K, R, stride, pad)
    (1, 3, 32, 32, 64, 7, 2, 3),      # stem-like, C=3
    (2, 64, 14, 14, 64, 1, 1, 0),     # 1x1
    (2, 64, 15, 15, 96, 3, 1, 1),     # 3x3, odd spatial
    (1, 128, 14, 14, 128, 3, 2, 1),   # 3x3 stride 2
    (2, 256, 7, 7, 100, 1, 2, 0),     # 1x1 stride 2, K not multiple of 64
    (1, 37, 9, 11, 19, 3, 1, 1),      # ragged everything
    (8, 64, 56, 56, 256, 1, 1, 0),    # > 2 persistent tiles per CTA (128-channel tiles)
    (8, 64, 56, 56, 64, 1, 1, 0),     # > 1 persistent tile per CTA (64-channel tiles)
    (2, 3, 224, 224, 64, 7, 2, 3),    # the ResNet stem: TMA input windows (small-channel variant)
    (2, 3, 20, 20, 64, 7, 2, 3),      # C=3, tiles straddle images: dense-k global gather of that variant
    (3, 1, 12, 12, 16, 3, 1, 1),      # C=1, one k block: dense-k global gather, K = 9
    (3, 64, 14, 14, 128, 1, 1, 0),    # 1x1 at 14x14: tiles straddle images, per-quarter TMA boxes
    (2, 128, 28, 28, 160, 1, 1, 0),   # 1x1 at 28x28, ragged channel tile (K = 160)
]


def conv_bn_oracle(x, w, stride, pad, bn, relu, residual=None):
    return oracle.conv2d(x, w, stride=(stride, stride), pads=(pad, pad, pad, pad), bn=bn, relu=relu,
                         residual=residual, eps=1e-5)


@pytest.mark.parametrize("case", CONV_CASES)
@pytest.mark.parametrize("op", ["Conv", "FusedConvBatchNorm", "FusedConvBatchNormRelu", "FusedConvBatchNormAddRelu"])
def test_conv_family_all_candidates(cuda, case, op):
    n, c, h, w_, k, r, stride, pad = case
    x = randn(n, c, h, w_)
    w = randn(k, c, r, r, scale=math.sqrt(2.0 / (c * r * r)))
    oh = (h + 2 * pad - r) // stride + 1
    ow = (w_ + 2 * pad - r) // stride + 1
    residual = randn(n, k, oh, ow) if op == "FusedConvBatchNormAddRelu" else None
    rng_state = RNG.bit_generator.state
    model = conv_model(x.shape, w, (stride, stride), (pad, pad), op, residual_shape=(n, k, oh, ow))
    RNG.bit_generator.state = rng_state
    bn = bn_params(k) if op != "Conv" else None
    expected = conv_bn_oracle(x, w, stride, pad, bn, op in ("FusedConvBatchNormRelu", "FusedConvBatchNormAddRelu"),
                              residual)
    inputs = {"x": x}
    if residual is not None:
        inputs["res"] = residual
    engine = ct.build_engine(model)
    kdim = c * r * r
    tol = 1e-4 * max(1.0, math.sqrt(kdim / 64.0))
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, inputs, {"y": ((n, k, oh, ow), np.float32)}, candidate=(0, index))
        assert_close(out["y"], expected, atol=tol, rtol=tol, what=f"{op} {case} {cand}")


@pytest.mark.parametrize("shape", [(2, 64, 112, 112), (3, 5, 7, 9), (1, 1, 1, 1), (2, 3, 9, 128)])
def test_max_pool_bitexact(cuda, shape):
    x = randn(*shape)
    x.flat[::7] = -np.inf
    model = ct.Model()
    model.add_input("x", list(shape))
    model.add_node("pool", "MaxPool", ["x"], ["y"], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1],
                   dilations=[1, 1])
    model.add_output("y")
    expected = oracle.max_pool(x)
    engine = ct.build_engine(model)
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, {"x": x}, {"y": (expected.shape, np.float32)}, candidate=(0, index))
        assert_bitexact(out["y"], expected, f"MaxPool {cand}")


@pytest.mark.parametrize("shape", [(2, 8, 112, 112), (2, 5, 9, 13)])
def test_max_pool_nan_bitexact(cuda, shape):
    """NaN inputs: the reference's tl.maximum (resnet.py:178-180, default
    propagate_nan=NONE, i.e. IEEE maxNum) returns the non-NaN operand, so a
    NaN tap is skipped and a window of NaN taps only yields -inf (the
    accumulator's start value). The oracle's `v > best` scan has the same
    result; every candidate must match it bit for bit."""
    x = randn(*shape)
    x.flat[::5] = np.nan
    x[0, 0, :3, :3] = np.nan   # output (0, 0, 0, 0): every in-range tap NaN
    x[-1, -1, -3:, -3:] = np.nan
    model = ct.Model()
    model.add_input("x", list(shape))
    model.add_node("pool", "MaxPool", ["x"], ["y"], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1],
                   dilations=[1, 1])
    model.add_output("y")
    expected = oracle.max_pool(x)
    assert expected[0, 0, 0, 0] == -np.inf and not np.isnan(expected).any()
    engine = ct.build_engine(model)
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, {"x": x}, {"y": (expected.shape, np.float32)}, candidate=(0, index))
        assert_bitexact(out["y"], expected, f"MaxPool NaN {cand}")


@pytest.mark.parametrize("shape", [(4, 2048, 7, 7), (3, 17, 5, 3), (3, 50, 9, 9), (2, 3, 10, 10)])
def test_global_average_pool(cuda, shape):
    """Every candidate; the staged kernel sums each plane serially like the
    reference (resnet.py:185-198) and the oracle, so it must match bit for
    bit; the warp-per-plane kernel sums in a tree (1e-5 relative)."""
    x = randn(*shape)
    model = ct.Model()
    model.add_input("x", list(shape))
    model.add_node("gap", "GlobalAveragePool", ["x"], ["y"])
    model.add_output("y")
    expected = oracle.global_average_pool(x)
    engine = ct.build_engine(model)
    candidates = engine.ops()[0]["candidates"]
    assert any("staged" in c for c in candidates) == (shape[2] <= 9 and shape[3] <= 9)
    for index, cand in enumerate(candidates):
        out, _ = run_graph(model, {"x": x}, {"y": ((shape[0], shape[1], 1, 1), np.float32)}, candidate=(0, index))
        if "staged" in cand:
            assert_bitexact(out["y"], expected, f"GAP {cand}")
        else:
            assert_close(out["y"], expected, atol=1e-6, rtol=1e-5, what=f"GAP {cand}")


@pytest.mark.parametrize("numel_shape", [(2, 64, 56, 56), (1, 3, 7, 5), (4099,)])
@pytest.mark.parametrize("op", ["Relu", "Add", "AddRelu"])
def test_elementwise_f32_bitexact(cuda, numel_shape, op):
    layout = "NCHW" if len(numel_shape) == 4 else ""
    a = randn(*numel_shape)
    b = randn(*numel_shape)
    model = ct.Model()
    model.add_input("a", list(numel_shape), layout=layout)
    ins = ["a"]
    feeds = {"a": a}
    if op != "Relu":
        model.add_input("b", list(numel_shape), layout=layout)
        ins.append("b")
        feeds["b"] = b
    model.add_node("op", op, ins, ["y"])
    model.add_output("y")
    expected = {"Relu": lambda: oracle.relu(a), "Add": lambda: oracle.add(a, b),
                "AddRelu": lambda: oracle.add_relu(a, b)}[op]()
    engine = ct.build_engine(model)
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, feeds, {"y": (numel_shape, np.float32)}, candidate=(0, index))
        assert_bitexact(out["y"], expected, f"{op} {cand}")


@pytest.mark.parametrize("shape", [(2, 64, 28, 28), (1, 5, 3, 3)])
def test_batch_norm(cuda, shape):
    x = randn(*shape)
    scale, bias, mean, var = bn_params(shape[1])
    model = ct.Model()
    model.add_input("x", list(shape))
    for n, v in zip(("s", "b", "m", "v"), (scale, bias, mean, var)):
        model.add_constant(n, v, layout="")
    model.add_node("bn", "BatchNormalization", ["x", "s", "b", "m", "v"], ["y"], epsilon=1e-5)
    model.add_output("y")
    out, _ = run_graph(model, {"x": x}, {"y": (shape, np.float32)})
    assert_close(out["y"], oracle.batch_norm(x, scale, bias, mean, var), atol=1e-5, rtol=1e-5, what="BN")


@pytest.mark.parametrize("mnk", [(256, 1000, 2048), (17, 33, 65), (1, 1000, 2048)])
def test_gemm_f32(cuda, mnk):
    m, n, k = mnk
    a = randn(m, k)
    b = randn(k, n, scale=0.01)
    model = ct.Model()
    model.add_input("a", [m, k], layout="")
    model.add_constant("b", b, layout="")
    model.add_node("fc", "Gemm", ["a", "b"], ["y"])
    model.add_output("y")
    expected = oracle.gemm_f32(a, b)
    engine = ct.build_engine(model)
    tol = 1e-4 * max(1.0, math.sqrt(k / 64.0))
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, {"a": a}, {"y": ((m, n), np.float32)}, candidate=(0, index))
        assert_close(out["y"], expected, atol=tol, rtol=tol, what=f"Gemm f32 {cand}")


@pytest.mark.parametrize("mnk", [(256, 3072, 768), (17, 512, 128), (128, 768, 3072), (33, 200, 72),
                                 # persistent kernel, several tiles per CTA: 192-wide tiles with a partial
                                 # last tile (N not a multiple of 192), 192-wide at N = 768, 256-wide tiles
                                 (1280, 2560, 64), (2048, 4864, 128), (4096, 768, 512), (4096, 3072, 256)])
@pytest.mark.parametrize("op", ["Gemm", "GemmGelu"])
def test_gemm_f16(cuda, mnk, op):
    m, n, k = mnk
    a = randn(m, k, dtype=np.float16)
    b = randn(k, n, dtype=np.float16, scale=0.02)
    model = ct.Model()
    model.add_input("a", [m, k], dtype=np.float16, layout="")
    model.add_constant("b", b, layout="")
    model.add_node("proj", op, ["a", "b"], ["y"])
    model.add_output("y")
    expected = oracle.gemm_f16(a, b, gelu=(op == "GemmGelu"))
    engine = ct.build_engine(model)
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, {"a": a}, {"y": ((m, n), np.float16)}, candidate=(0, index))
        assert_close(out["y"], expected, atol=2e-2, rtol=2e-2, what=f"{op} {mnk} {cand}")


@pytest.mark.parametrize("shape", [(4096, 768), (17, 512), (3, 1000)])
def test_gelu_and_add_f16(cuda, shape):
    x = randn(*shape, dtype=np.float16)
    y = randn(*shape, dtype=np.float16)
    model = ct.Model()
    model.add_input("x", list(shape), dtype=np.float16, layout="")
    model.add_node("g", "Gelu", ["x"], ["out"])
    model.add_output("out")
    out, _ = run_graph(model, {"x": x}, {"out": (shape, np.float16)})
    assert_close(out["out"], oracle.gelu_f16(x), atol=1e-3, rtol=1e-3, what="Gelu")
    model = ct.Model()
    model.add_input("x", list(shape), dtype=np.float16, layout="")
    model.add_input("y", list(shape), dtype=np.float16, layout="")
    model.add_node("a", "Add", ["x", "y"], ["out"])
    model.add_output("out")
    out, _ = run_graph(model, {"x": x, "y": y}, {"out": (shape, np.float16)})
    assert_bitexact(out["out"], oracle.add_f16(x, y), "Add f16")


@pytest.mark.parametrize("shape", [(4096, 768), (17, 512), (5, 1024), (3, 33)])
def test_layer_norms_and_softmax_f16(cuda, shape):
    rows, cols = shape
    x = randn(rows, cols, dtype=np.float16)
    r = randn(rows, cols, dtype=np.float16)
    g = RNG.uniform(0.5, 1.5, cols).astype(np.float16)
    b = randn(cols, dtype=np.float16, scale=0.1)
    model = ct.Model()
    model.add_input("x", [rows, cols], dtype=np.float16, layout="")
    model.add_input("r", [rows, cols], dtype=np.float16, layout="")
    model.add_constant("g", g, layout="")
    model.add_constant("b", b, layout="")
    model.add_node("add", "Add", ["x", "r"], ["s"])
    model.add_node("ln", "LayerNormalization", ["s", "g", "b"], ["y"], axis=-1, epsilon=1e-5)
    model.add_output("y")
    engine = ct.build_engine(model)
    assert [o["op_type"] for o in engine.ops()] == ["SkipLayerNormalization"]
    for index, cand in enumerate(engine.ops()[0]["candidates"]):
        out, _ = run_graph(model, {"x": x, "r": r}, {"y": (shape, np.float16)}, candidate=(0, index))
        # The unfused candidate rounds x + r to FP16 before normalising.
        expected = (oracle.layer_norm_f16(x, g, b, residual=r) if not cand.startswith("unfused")
                    else oracle.layer_norm_f16(oracle.add_f16(x, r), g, b))
        assert_close(out["y"], expected, atol=2e-2, rtol=2e-2, what=f"SkipLN {cand}")
    model = ct.Model()
    model.add_input("x", [rows, cols], dtype=np.float16, layout="")
    model.add_node("sm", "Softmax", ["x"], ["y"])
    model.add_output("y")
    out, _ = run_graph(model, {"x": x}, {"y": (shape, np.float16)})
    assert_close(out["y"], oracle.softmax_f16(x), atol=1e-3, rtol=1e-2, what="Softmax")
