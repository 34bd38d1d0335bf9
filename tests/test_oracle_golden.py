"""Pins the CPU oracle against the golden vectors (no GPU): the C
restatement of the reference kernels reproduces the reference test suite's
known answers, and the PyTorch restatement reproduces the reference's own
PyTorch ResNet-50 logits."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from cutriton_b200 import workloads
from oracle import ops as oracle
from oracle import torch_ref
from tests.helpers import assert_close

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_oracle_stem_known_answer():
    g = np.load(GOLDEN / "stem_known_answer.npz")
    x = (((np.arange(3 * 224 * 224) % 29) - 14).astype(np.float32) / np.float32(29.0)).reshape(1, 3, 224, 224)
    ones, zeros = np.ones(64, np.float32), np.zeros(64, np.float32)
    y = oracle.conv2d(x, g["conv_weight"], stride=(2, 2), pads=(3, 3, 3, 3),
                      bn=(ones, zeros, zeros, np.full(64, 0.99999, np.float32)), relu=True)
    pooled = oracle.global_average_pool(y).reshape(1, 64)
    logits = oracle.gemm_f32(pooled, g["fc_weight"])
    assert_close(logits, g["expected"], atol=1e-4, rtol=1e-4, what="oracle stem")


def test_oracle_ffn17_known_answer():
    g = np.load(GOLDEN / "ffn17_known_answer.npz")
    x = g["x"].astype(np.float16)
    h = oracle.gemm_f16(x, g["weight"].astype(np.float16), gelu=True)
    y = oracle.layer_norm_f16(h, g["scale"].astype(np.float16), g["bias"].astype(np.float16),
                              residual=g["residual"].astype(np.float16))
    assert_close(y, g["expected"], atol=2e-2, rtol=2e-2, what="oracle ffn17")


def test_torch_restatement_matches_reference_model():
    logits = torch_ref.resnet50_logits(workloads.resnet50_input(1, mode="pattern"), workloads.resnet50_weights("pattern"))
    golden = np.load(GOLDEN / "resnet50_pattern_bs1.npz")["logits"]
    assert_close(logits, golden, atol=1e-7, rtol=1e-5, what="torch restatement")


def test_oracle_conv_matches_torch_small():
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(7)
    x = rng.standard_normal((2, 5, 9, 11)).astype(np.float32)
    w = rng.standard_normal((7, 5, 3, 3)).astype(np.float32)
    bn = tuple(rng.uniform(0.5, 1.5, 7).astype(np.float32) for _ in range(4))
    ours = oracle.conv2d(x, w, stride=(2, 1), pads=(1, 2, 1, 2), bn=bn, relu=True)
    t = F.conv2d(torch.from_numpy(x), torch.from_numpy(w), stride=(2, 1), padding=(1, 2))
    t = F.relu(F.batch_norm(t, torch.from_numpy(bn[2]), torch.from_numpy(bn[3]), torch.from_numpy(bn[0]),
                            torch.from_numpy(bn[1]), training=False, eps=1e-5))
    assert_close(ours, t.numpy(), atol=1e-5, rtol=1e-5, what="oracle conv vs torch")


def test_oracle_fp16_rounding_matches_numpy():
    rng = np.random.default_rng(3)
    a = (rng.standard_normal(20000) * 300).astype(np.float16)
    b = (rng.standard_normal(20000) * 0.01).astype(np.float16)
    # Add of two halves: exact sum rounded once (numpy rounds float64 -> float16 correctly).
    expected = (a.astype(np.float64) + b.astype(np.float64)).astype(np.float16)
    assert np.array_equal(oracle.add_f16(a, b).view(np.uint16), expected.view(np.uint16))
    x = (rng.standard_normal((8, 64)) * 3).astype(np.float16)
    w = (rng.standard_normal((64, 16)) * 0.1).astype(np.float16)
    ref = (x.astype(np.float32) @ w.astype(np.float32))
    assert_close(oracle.gemm_f16(x, w), ref, atol=1e-2, rtol=1e-2, what="oracle gemm f16")


def test_oracle_max_pool_and_gap():
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 3, 13, 10)).astype(np.float32)
    ours = oracle.max_pool(x)
    ref = F.max_pool2d(torch.from_numpy(x), kernel_size=3, stride=2, padding=1).numpy()
    assert np.array_equal(ours, ref)
    assert_close(oracle.global_average_pool(x)[:, :, 0, 0], x.mean(axis=(2, 3)), atol=1e-6, rtol=1e-5, what="gap")
