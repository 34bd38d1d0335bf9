"""Parity at the benchmarked configurations.

The headline numbers come from ResNet-50 at 256 images per GPU and the FP16
FFN block at config 1 (M=4096, H=768, I=3072) and config 4 (H=1024, I=4096).
These tests run exactly those graphs through the engine and compare a fixed
sample of their rows with the oracle:

* FFN: every output row depends only on its own input row, so the C oracle
  (oracle/ops.c, GEMM with FP32 accumulation and RNE FP16 stores, erf-GELU on
  the accumulator, SkipLayerNorm in FP32) is evaluated on the sampled rows
  alone. Bar: absolute max|d| <= 2e-2 (the FFN bound of the benchmark config;
  the reference's own check is tests/cpp/test_cuda.cpp:432).
* ResNet-50 bs256: each image is independent, so the PyTorch CPU restatement
  (oracle/torch_ref.py, pinned to the reference model's logits) runs on the
  sampled images. Bar: max|d| <= 1e-3 * max|logit| and identical top-1.
* The down-projection GEMM alone at M=4096, K=3072 (many tile rows).

Samples cover the first and last pixel/row tiles, tiles that straddle two
images (every 7x7 / 14x14 / 28x28 layer has them) and rows spread over the
middle.
"""

from __future__ import annotations

import numpy as np
import pytest

from cutriton_b200 import workloads
from oracle import ops as oracle
from tests.helpers import run_graph

pytestmark = pytest.mark.gpu

FFN_BOUND = 2e-2


def sample_rows(total: int, tile: int = 128, spread: int = 96, seed: int = 0) -> np.ndarray:
    """First and last tile, the rows either side of every 8th tile boundary,
    and `spread` seeded rows over the rest."""
    rows = set(range(min(tile, total))) | set(range(max(0, total - tile), total))
    for boundary in range(tile, total, 8 * tile):
        rows.update((boundary - 1, boundary))
    rows.update(np.random.default_rng(seed).integers(0, total, spread).tolist())
    return np.array(sorted(rows), dtype=np.int64)


def ffn_oracle_rows(x: np.ndarray, w: dict[str, np.ndarray], rows: np.ndarray) -> np.ndarray:
    xs = np.ascontiguousarray(x[rows])
    h = oracle.gemm_f16(xs, w["w1"], gelu=True)
    y = oracle.gemm_f16(h, w["w2"])
    return oracle.layer_norm_f16(y, w["gamma"], w["beta"], residual=xs)


@pytest.mark.parametrize("tokens,hidden,inner", [(4096, 768, 3072),   # config 1
                                                 (8192, 1024, 4096)])  # config 4, one rank's slice at 8 GPUs
def test_ffn_benchmark_config_vs_oracle(cuda, tokens, hidden, inner):
    w = workloads.ffn_weights(hidden, inner, seed=0)
    x = workloads.ffn_input(tokens, hidden, seed=0)
    out, engine = run_graph(workloads.build_ffn(w, tokens, hidden, inner), {"x": x},
                            {"output": ((tokens, hidden), np.float16)}, enable_cuda_graph=True)
    assert [o["op_type"] for o in engine.ops()] == ["GemmGelu", "Gemm", "SkipLayerNormalization"]
    got = out["output"].astype(np.float64)
    assert np.isfinite(got).all()
    rows = sample_rows(tokens)
    expected = ffn_oracle_rows(x, w, rows).astype(np.float64)
    err = np.abs(got[rows] - expected).max()
    assert err <= FFN_BOUND, f"FFN {tokens}x{hidden}x{inner}: max|d| = {err:.3e} > {FFN_BOUND}"


@pytest.mark.parametrize("op", ["Gemm", "GemmGelu"])
def test_down_projection_gemm_full_tiles(cuda, op):
    import cutriton_b200 as ct

    m, n, k = 4096, 768, 3072
    rng = np.random.default_rng(21)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = (rng.standard_normal((k, n)) * 0.02).astype(np.float16)
    model = ct.Model()
    model.add_input("a", [m, k], dtype=np.float16, layout="")
    model.add_constant("b", b, layout="")
    model.add_node("proj", op, ["a", "b"], ["y"])
    model.add_output("y")
    out, _ = run_graph(model, {"a": a}, {"y": ((m, n), np.float16)})
    rows = sample_rows(m)
    expected = oracle.gemm_f16(np.ascontiguousarray(a[rows]), b, gelu=(op == "GemmGelu")).astype(np.float64)
    err = np.abs(out["y"][rows].astype(np.float64) - expected).max()
    assert err <= FFN_BOUND, f"{op} {m}x{n}x{k}: max|d| = {err:.3e}"


def resnet_sample(batch: int) -> np.ndarray:
    """First 8, last 8 and a few middle images of the batch."""
    middle = [batch // 2 - 1, batch // 2, 127, 128, 129]
    picked = set(range(min(8, batch))) | set(range(max(0, batch - 8), batch))
    picked.update(i for i in middle if 0 <= i < batch)
    return np.array(sorted(picked), dtype=np.int64)


def test_resnet50_bs256_sampled_images_vs_torch(cuda):
    from oracle import torch_ref

    batch = 256
    weights = workloads.resnet50_weights("baseline", seed=0)
    x = workloads.resnet50_input(batch, seed=0)
    out, _ = run_graph(workloads.build_resnet50(weights, batch=batch), {"input": x},
                       {"output": ((batch, 1000), np.float32)}, enable_residual_fusion=True, enable_cuda_graph=True)
    got = out["output"].astype(np.float64)
    assert np.isfinite(got).all()
    picked = resnet_sample(batch)
    expected = torch_ref.resnet50_logits(np.ascontiguousarray(x[picked]), weights).astype(np.float64)
    bound = 1e-3 * np.abs(expected).max()
    err = np.abs(got[picked] - expected).max()
    assert err <= bound, f"ResNet-50 bs256: max|d| = {err:.3e} > {bound:.3e}"
    assert (got[picked].argmax(axis=1) == expected.argmax(axis=1)).all(), "top-1 differs"
