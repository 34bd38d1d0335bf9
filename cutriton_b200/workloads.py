"""Graphs and seeded weights of the benchmark workloads.

* ResNet-50 v1.5 (FP32, NCHW/OIHW) with the node structure of the
  reference's own builder (benchmarks/resnet50_native.cpp:63-189): every
  conv is Conv -> BatchNormalization(epsilon 1e-5) [-> Relu], the stride sits
  on the 3x3 of each bottleneck, the block tail is Add -> Relu, then
  GlobalAveragePool -> Flatten -> Gemm (fc weight [2048, 1000], no bias node).
* Transformer FFN (FP16): Gemm(x, W1) -> Gelu -> Gemm(., W2) -> Add(., x) ->
  LayerNormalization, which the passes fuse into GemmGelu, Gemm and
  SkipLayerNormalization.

Weights come in two flavours: ``"baseline"`` — the seeded distributions of
the benchmark configs (Kaiming-normal fan_out convs; BN gamma ~ U(0.5, 1.5),
beta ~ N(0, 0.1), mean ~ N(0, 0.1), var ~ U(0.5, 1.5); FC ~ N(0, 0.01)) —
and ``"pattern"`` — the reference benchmark's deterministic integer pattern
((i*17 + seed*13) % 19 - 9) * 0.02 / sqrt(fan_in) with BN scale 1, bias 0.01,
mean 0, var 0.99999 (resnet50_native.cpp:107-144).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import Model


@dataclass(frozen=True)
class ConvLayer:
    prefix: str
    cin: int
    cout: int
    kernel: int
    stride: int
    pad: int
    relu: bool


def resnet50_layers() -> list[tuple[str, object]]:
    """Ordered layer program: ("conv", ConvLayer) | ("maxpool", value) |
    ("block_add", prefix) markers, mirroring the reference builder."""
    program: list[tuple[str, object]] = [("conv", ConvLayer("stem", 3, 64, 7, 2, 3, True)), ("maxpool", None)]
    channels = 64
    for stage, (blocks, planes) in enumerate(zip((3, 4, 6, 3), (64, 128, 256, 512))):
        for block in range(blocks):
            stride = 2 if stage != 0 and block == 0 else 1
            prefix = f"layer{stage + 1}_block{block + 1}"
            program.append(("conv", ConvLayer(prefix + "_conv1", channels, planes, 1, 1, 0, True)))
            program.append(("conv", ConvLayer(prefix + "_conv2", planes, planes, 3, stride, 1, True)))
            program.append(("conv", ConvLayer(prefix + "_conv3", planes, planes * 4, 1, 1, 0, False)))
            if stride != 1 or channels != planes * 4:
                program.append(("conv", ConvLayer(prefix + "_downsample", channels, planes * 4, 1, stride, 0, False)))
            program.append(("block_add", prefix))
            channels = planes * 4
    return program


def resnet50_weights(mode: str = "baseline", seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    weights: dict[str, np.ndarray] = {}
    pattern_seed = 1

    def pattern(shape: tuple[int, ...], fan_in: int) -> np.ndarray:
        nonlocal pattern_seed
        count = math.prod(shape)
        idx = np.arange(count, dtype=np.int64)
        ints = (idx * 17 + pattern_seed * 13) % 19 - 9
        pattern_seed += 1
        scale = np.float32(0.02 / math.sqrt(float(fan_in)))
        return (ints.astype(np.float32) * scale).reshape(shape)

    for kind, item in resnet50_layers():
        if kind != "conv":
            continue
        layer: ConvLayer = item  # type: ignore[assignment]
        shape = (layer.cout, layer.cin, layer.kernel, layer.kernel)
        c = layer.cout
        if mode == "pattern":
            weights[layer.prefix + "_weight"] = pattern(shape, layer.cin * layer.kernel * layer.kernel)
            weights[layer.prefix + "_scale"] = np.ones(c, np.float32)
            weights[layer.prefix + "_bias"] = np.full(c, 0.01, np.float32)
            weights[layer.prefix + "_mean"] = np.zeros(c, np.float32)
            weights[layer.prefix + "_variance"] = np.full(c, 0.99999, np.float32)
        elif mode == "baseline":
            std = math.sqrt(2.0 / (layer.cout * layer.kernel * layer.kernel))
            weights[layer.prefix + "_weight"] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
            weights[layer.prefix + "_scale"] = rng.uniform(0.5, 1.5, c).astype(np.float32)
            weights[layer.prefix + "_bias"] = (rng.standard_normal(c) * 0.1).astype(np.float32)
            weights[layer.prefix + "_mean"] = (rng.standard_normal(c) * 0.1).astype(np.float32)
            weights[layer.prefix + "_variance"] = rng.uniform(0.5, 1.5, c).astype(np.float32)
        else:
            raise ValueError(f"unknown weight mode {mode}")
    if mode == "pattern":
        weights["fc_weight"] = pattern((2048, 1000), 2048)
    else:
        weights["fc_weight"] = (rng.standard_normal((2048, 1000), dtype=np.float32) * np.float32(0.01))
    return weights


def resnet50_input(batch: int, seed: int = 0, mode: str = "baseline") -> np.ndarray:
    if mode == "pattern":
        idx = np.arange(batch * 3 * 224 * 224, dtype=np.int64)
        return (((idx % 29) - 14).astype(np.float32) / np.float32(29.0)).reshape(batch, 3, 224, 224)
    rng = np.random.default_rng(seed + 1000)
    return rng.standard_normal((batch, 3, 224, 224), dtype=np.float32)


def build_resnet50(weights: dict[str, np.ndarray], batch: int = 1, dynamic_batch: bool = False) -> Model:
    """The reference benchmark graph; `dynamic_batch` marks axis 0 dynamic."""
    model = Model()
    model.add_input("input", [-1 if dynamic_batch else batch, 3, 224, 224])
    value = "input"
    block_input = "input"
    conv_outputs: dict[str, str] = {}
    for kind, item in resnet50_layers():
        if kind == "maxpool":
            model.add_node("stem_maxpool", "MaxPool", [value], ["stem_pool"], kernel_shape=[3, 3], strides=[2, 2],
                           pads=[1, 1, 1, 1], dilations=[1, 1])
            value = "stem_pool"
            block_input = value
            continue
        if kind == "block_add":
            prefix = item  # type: ignore[assignment]
            main = conv_outputs[prefix + "_conv3"]
            identity = conv_outputs.get(prefix + "_downsample", block_input)
            model.add_node(prefix + "_add", "Add", [main, identity], [prefix + "_sum"])
            model.add_node(prefix + "_relu", "Relu", [prefix + "_sum"], [prefix + "_output"])
            value = prefix + "_output"
            block_input = value
            continue
        layer: ConvLayer = item  # type: ignore[assignment]
        p = layer.prefix
        source = block_input if p.endswith("_downsample") or p.endswith("_conv1") else value
        model.add_constant(p + "_weight", weights[p + "_weight"], layout="OIHW")
        for suffix in ("_scale", "_bias", "_mean", "_variance"):
            model.add_constant(p + suffix, weights[p + suffix], layout="")
        model.add_node(p + "_conv_node", "Conv", [source, p + "_weight"], [p + "_conv"],
                       strides=[layer.stride, layer.stride], pads=[layer.pad] * 4, dilations=[1, 1])
        model.add_node(p + "_bn_node", "BatchNormalization",
                       [p + "_conv", p + "_scale", p + "_bias", p + "_mean", p + "_variance"], [p + "_bn"],
                       epsilon=1e-5)
        out = p + "_bn"
        if layer.relu:
            model.add_node(p + "_relu_node", "Relu", [out], [p + "_relu"])
            out = p + "_relu"
        conv_outputs[p] = out
        if not p.endswith("_downsample"):
            value = out
    model.add_node("global_average_pool", "GlobalAveragePool", [value], ["gap"])
    model.add_node("flatten", "Flatten", ["gap"], ["flattened"])
    model.add_constant("fc_weight", weights["fc_weight"], layout="")
    model.add_node("classifier", "Gemm", ["flattened", "fc_weight"], ["output"])
    model.add_output("output")
    return model


def ffn_weights(hidden: int, inner: int, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    return {
        "w1": (rng.standard_normal((hidden, inner)) * 0.02).astype(np.float16),
        "w2": (rng.standard_normal((inner, hidden)) * 0.02).astype(np.float16),
        "gamma": np.ones(hidden, np.float16),
        "beta": np.zeros(hidden, np.float16),
    }


def ffn_input(tokens: int, hidden: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed + 1000)
    return rng.standard_normal((tokens, hidden)).astype(np.float16)


def build_ffn(weights: dict[str, np.ndarray], tokens: int, hidden: int, inner: int) -> Model:
    model = Model()
    model.add_input("x", [tokens, hidden], dtype=np.float16, layout="")
    model.add_constant("w1", weights["w1"], layout="")
    model.add_constant("w2", weights["w2"], layout="")
    model.add_constant("gamma", weights["gamma"], layout="")
    model.add_constant("beta", weights["beta"], layout="")
    model.add_node("up_projection", "Gemm", ["x", "w1"], ["projected"])
    model.add_node("activation", "Gelu", ["projected"], ["activated"])
    model.add_node("down_projection", "Gemm", ["activated", "w2"], ["contracted"])
    model.add_node("residual_add", "Add", ["contracted", "x"], ["sum"])
    model.add_node("output_norm", "LayerNormalization", ["sum", "gamma", "beta"], ["output"], axis=-1, epsilon=1e-5)
    model.add_output("output")
    return model


def resnet50_flops_per_image() -> float:
    """Algorithmic FLOPs (2 per multiply-add) of one 224x224 image."""
    total = 0.0
    h = 224
    block_h = h
    for kind, item in resnet50_layers():
        if kind == "maxpool":
            h = (h + 2 - 3) // 2 + 1
            block_h = h
            continue
        if kind == "block_add":
            block_h = h
            continue
        layer: ConvLayer = item  # type: ignore[assignment]
        in_h = block_h if layer.prefix.endswith(("_conv1", "_downsample")) else h
        out_h = (in_h + 2 * layer.pad - layer.kernel) // layer.stride + 1
        total += 2.0 * out_h * out_h * layer.cout * layer.cin * layer.kernel * layer.kernel
        if not layer.prefix.endswith("_downsample"):
            h = out_h
    return total + 2.0 * 2048 * 1000
