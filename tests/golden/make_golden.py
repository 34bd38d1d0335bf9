"""Generates the golden vectors under tests/golden/ (run in the build
container, where the reference checkout is importable; the GPU box only reads
the committed .npz files).

* resnet50_pattern_bs1.npz — logits of the reference's own PyTorch ResNet-50
  (benchmarks/resnet50_compare.py: ResNet50 class, WeightFactory pattern
  weights, make_input pattern input) on CPU, batch 1.
* stem_known_answer.npz — the ResNet-stem known answer of the reference's
  tests/cpp/test_cuda.cpp:444-479 (one-hot 7x7 conv weights, BN identity,
  ReLU, global average pool, FC (i % 11 - 5) / 101), restated in numpy.
* ffn17_known_answer.npz — the FP16 FFN known answer of test_cuda.cpp:
  336-393 (tokens 17, hidden 128, intermediate 512; GEMM, exact GELU,
  residual add, LayerNorm), restated in numpy (float64 statistics).

Usage: python tests/golden/make_golden.py --reference /path/to/checkout
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def resnet50_pattern(reference: Path) -> None:
    import torch

    sys.path.insert(0, str(reference / "benchmarks"))
    import resnet50_compare  # the reference's own model definition

    device = torch.device("cpu")
    torch.set_num_threads(8)
    model = resnet50_compare.ResNet50(device).eval()
    with torch.inference_mode():
        logits = model(resnet50_compare.make_input(device)).numpy()
    np.savez_compressed(HERE / "resnet50_pattern_bs1.npz", logits=logits.astype(np.float32))


def stem_known_answer() -> None:
    x = ((np.arange(3 * 224 * 224) % 29) - 14).astype(np.float32) / np.float32(29.0)
    x = x.reshape(3, 224, 224)
    conv_w = np.zeros((64, 3, 7, 7), np.float32)
    for oc in range(64):
        conv_w[oc, oc % 3, 3, 3] = np.float32(0.05) * np.float32(1 + oc % 5)
    fc = (((np.arange(64 * 1000) % 11) - 5).astype(np.float32) / np.float32(101.0)).reshape(64, 1000)
    pooled = np.zeros(64, np.float64)
    for oc in range(64):
        w = np.float32(0.05) * np.float32(1 + oc % 5)
        taps = x[oc % 3, 0:224:2, 0:224:2] * w  # stride 2, the one-hot tap sits at the pad offset
        pooled[oc] = np.maximum(taps, 0).astype(np.float64).sum() / (112.0 * 112.0)
    expected = (pooled.astype(np.float32)[None, :] @ fc).astype(np.float32)
    np.savez_compressed(HERE / "stem_known_answer.npz", conv_weight=conv_w, fc_weight=fc, expected=expected)


def ffn17_known_answer() -> None:
    tokens, hidden, inner = 17, 128, 512
    x = (((np.arange(tokens * hidden) % 23) - 11).astype(np.float32) / np.float32(37.0)).reshape(tokens, hidden)
    residual = (((np.arange(tokens * inner) % 17) - 8).astype(np.float32) / np.float32(53.0)).reshape(tokens, inner)
    weight = (((np.arange(hidden * inner) % 19) - 9).astype(np.float32) / np.float32(181.0)).reshape(hidden, inner)
    cols = np.arange(inner)
    scale = (np.float32(0.9) + np.float32(0.001) * (cols % 13).astype(np.float32)).astype(np.float32)
    bias = (((cols % 7) - 3).astype(np.float32) / np.float32(100.0)).astype(np.float32)
    projected = x.astype(np.float32) @ weight.astype(np.float32)
    erf = np.vectorize(math.erf)
    activated = 0.5 * projected * (1.0 + erf(projected * 0.7071067811865476))
    total = activated + residual
    mean = total.astype(np.float64).mean(axis=1, keepdims=True)
    var = ((total - mean) ** 2).mean(axis=1, keepdims=True)
    expected = ((total - mean) / np.sqrt(var + 1e-5) * scale + bias).astype(np.float32)
    np.savez_compressed(HERE / "ffn17_known_answer.npz", x=x, residual=residual, weight=weight, scale=scale,
                        bias=bias, expected=expected)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True,
                        help="checkout of the reference project (read only)")
    args = parser.parse_args()
    stem_known_answer()
    ffn17_known_answer()
    resnet50_pattern(args.reference)


if __name__ == "__main__":
    main()
