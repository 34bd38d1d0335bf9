"""PyTorch-eager CPU restatement of the reference's comparison models.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (see oracle/__init__.py).

* ResNet-50 v1.5 FP32 as benchmarks/resnet50_compare.py:36-141 of the
  reference builds it (conv2d without bias -> inference batch_norm eps 1e-5
  [-> relu]; bottleneck with the stride on the 3x3; relu(main + identity);
  max_pool 3x3/2 pad 1; adaptive average pool; flatten; logits = x @ fc).
* Transformer FFN FP16 as transformer_ffn_compare.py:52-60 restated for the
  two-GEMM block of the benchmark config: layer_norm(gelu(x @ W1) @ W2 + x).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def _conv_bn(x: torch.Tensor, w: dict[str, torch.Tensor], prefix: str, stride: int, pad: int,
             relu: bool) -> torch.Tensor:
    y = F.conv2d(x, w[prefix + "_weight"], bias=None, stride=stride, padding=pad)
    y = F.batch_norm(y, w[prefix + "_mean"], w[prefix + "_variance"], w[prefix + "_scale"], w[prefix + "_bias"],
                     training=False, eps=1e-5)
    return F.relu(y) if relu else y


def resnet50_forward(x: torch.Tensor, weights: dict[str, torch.Tensor]) -> torch.Tensor:
    from cutriton_b200.workloads import resnet50_layers

    value = None
    block_input = x
    outputs: dict[str, torch.Tensor] = {}
    current = x
    for kind, item in resnet50_layers():
        if kind == "maxpool":
            current = F.max_pool2d(current, kernel_size=3, stride=2, padding=1)
            block_input = current
            continue
        if kind == "block_add":
            prefix = item
            identity = outputs.get(prefix + "_downsample", block_input)
            current = F.relu(outputs[prefix + "_conv3"] + identity)
            block_input = current
            outputs = {}
            continue
        layer = item
        source = block_input if layer.prefix.endswith(("_conv1", "_downsample")) else current
        out = _conv_bn(source, weights, layer.prefix, layer.stride, layer.pad, layer.relu)
        outputs[layer.prefix] = out
        if not layer.prefix.endswith("_downsample"):
            current = out
    value = F.adaptive_avg_pool2d(current, (1, 1)).flatten(1)
    return value @ weights["fc_weight"]


def resnet50_logits(x: np.ndarray, weights: dict[str, np.ndarray], threads: int | None = None) -> np.ndarray:
    if threads:
        torch.set_num_threads(threads)
    tw = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in weights.items()}
    with torch.inference_mode():
        return resnet50_forward(torch.from_numpy(np.ascontiguousarray(x)), tw).numpy()


def ffn_forward(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gamma: torch.Tensor,
                beta: torch.Tensor) -> torch.Tensor:
    hidden = x.shape[-1]
    projected = F.gelu(x @ w1, approximate="none")
    return F.layer_norm(projected @ w2 + x, (hidden,), gamma, beta, 1e-5)


def ffn_output(x: np.ndarray, weights: dict[str, np.ndarray], dtype=torch.float32) -> np.ndarray:
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dtype) for k, v in weights.items()}
    with torch.inference_mode():
        out = ffn_forward(torch.from_numpy(np.ascontiguousarray(x)).to(dtype), t["w1"], t["w2"], t["gamma"], t["beta"])
    return out.float().numpy()
