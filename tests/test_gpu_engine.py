"""Engine-level GPU tests: the reference's CUDA integration cases
(tests/cpp/test_cuda.cpp) on the sm_100a pack, plus whole-network parity.

* ResNet stem known answer (test_cuda.cpp:444-576) against the golden vector.
* FP16 FFN tokens=17 known answer (test_cuda.cpp:336-440), tolerance 2e-2.
* Profiling events (Flatten untimed), repeat run, output rebinding, external
  stream, CUDA Graph LRU counts over a dynamic profile, tuning cache written
  once and reused without rewrite.
* ResNet-50 with the reference benchmark's pattern weights against the
  logits of the reference's own PyTorch model (golden), and ResNet-50 with
  the benchmark-config weights against the PyTorch CPU restatement:
  max|d| <= 1e-3 * max|logit|, identical top-1.
* FFN (config-1 shape family) against the C oracle, 2e-2.
"""

from __future__ import annotations

import os
import time
from pathlib import Path

import numpy as np
import pytest

import cutriton_b200 as ct
from cutriton_b200 import workloads
from oracle import ops as oracle
from tests.helpers import assert_close, run_graph

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def stem_model(conv_w, fc_w, input_shape=(1, 3, 224, 224)):
    model = ct.Model()
    model.add_input("input", list(input_shape))
    model.add_constant("conv_w", conv_w, layout="OIHW")
    model.add_constant("bn_scale", np.ones(64, np.float32), layout="")
    model.add_constant("bn_bias", np.zeros(64, np.float32), layout="")
    model.add_constant("bn_mean", np.zeros(64, np.float32), layout="")
    model.add_constant("bn_var", np.full(64, 0.99999, np.float32), layout="")
    model.add_constant("fc_w", fc_w, layout="")
    model.add_node("conv", "Conv", ["input", "conv_w"], ["conv_y"], pads=[3, 3, 3, 3], strides=[2, 2],
                   dilations=[1, 1])
    model.add_node("bn", "BatchNormalization", ["conv_y", "bn_scale", "bn_bias", "bn_mean", "bn_var"], ["bn_y"],
                   epsilon=1e-5)
    model.add_node("relu", "Relu", ["bn_y"], ["relu_y"])
    model.add_node("gap", "GlobalAveragePool", ["relu_y"], ["gap_y"])
    model.add_node("flatten", "Flatten", ["gap_y"], ["flat_y"])
    model.add_node("gemm", "Gemm", ["flat_y", "fc_w"], ["output"])
    model.add_output("output")
    return model


def stem_input(shape=(1, 3, 224, 224)):
    n = int(np.prod(shape))
    return (((np.arange(n) % 29) - 14).astype(np.float32) / np.float32(29.0)).reshape(shape)


def test_stem_known_answer_and_runtime_features(cuda):
    import torch

    golden = np.load(GOLDEN / "stem_known_answer.npz")
    model = stem_model(golden["conv_weight"], golden["fc_weight"])
    engine = ct.build_engine(model, enable_cuda_graph=True, enable_profiling=True, tuning_mode=ct.TUNING_DISABLED)
    assert [o["op_type"] for o in engine.ops()] == ["FusedConvBatchNormRelu", "GlobalAveragePool", "Flatten", "Gemm"]
    ctx = engine.create_context()
    x = torch.from_numpy(stem_input()).to(cuda)
    y = torch.empty(1, 1000, device=cuda)
    ctx.bind_tensor("input", x)
    ctx.bind_tensor("output", y, output=True)
    ctx.run()
    assert_close(y.cpu().numpy(), golden["expected"], atol=1e-4, rtol=1e-4, what="stem known answer")
    events = ctx.profile_events()
    assert len(events) == 4 and events[2][1] == 0.0  # Flatten is a view: untimed
    ctx.run()  # repeat (graph replay)
    assert_close(y.cpu().numpy(), golden["expected"], atol=1e-4, rtol=1e-4, what="repeat")
    assert ctx.cached_graph_count() == 1
    rebound = torch.full((1, 1000), float("nan"), device=cuda)
    ctx.bind_tensor("output", rebound, output=True)
    ctx.run()
    assert_close(rebound.cpu().numpy(), golden["expected"], atol=1e-4, rtol=1e-4, what="rebound")
    assert ctx.cached_graph_count() == 2
    stream = torch.cuda.Stream()
    ctx.run_async(stream.cuda_stream)
    ctx.synchronize()
    with pytest.raises(ct.CutritonError) as err:
        ctx.run_async(None)
        ctx.run_async(None)
    assert err.value.code == ct.RUNTIME_ERROR
    ctx.synchronize()


def test_dynamic_profile_graph_lru(cuda):
    import torch

    golden = np.load(GOLDEN / "stem_known_answer.npz")
    model = stem_model(golden["conv_weight"], golden["fc_weight"], input_shape=(-1, 3, -1, -1))
    model.add_shape_profile("images", "input", [1, 3, 160, 160], [1, 3, 224, 224], [2, 3, 256, 256])
    engine = ct.build_engine(model, enable_cuda_graph=True, enable_profiling=False, cuda_graph_cache_capacity=2,
                             tuning_mode=ct.TUNING_DISABLED)
    ctx = engine.create_context()
    assert ctx.resolved_desc("output")[1] == (1, 1000)
    with pytest.raises(ct.CutritonError) as err:
        ctx.set_input_shape("input", [1, 3, 300, 300])
    assert err.value.code == ct.SHAPE_ERROR
    keep = []

    def run_shape(shape):
        ctx.set_input_shape("input", shape)
        ctx.resolve_shapes()
        x = torch.from_numpy(stem_input(tuple(shape))).to(cuda)
        out_shape = ctx.resolved_desc("output")[1]
        y = torch.empty(out_shape, device=cuda)
        ctx.bind_tensor("input", x)
        ctx.bind_tensor("output", y, output=True)
        ctx.run()
        assert torch.isfinite(y).all()
        keep.append((x, y))
        return y

    y224 = run_shape([1, 3, 224, 224])
    assert ctx.cached_graph_count() == 1
    assert_close(y224.cpu().numpy(), golden["expected"], atol=1e-4, rtol=1e-4, what="profile opt")
    run_shape([1, 3, 160, 160])
    assert ctx.cached_graph_count() == 2
    y2 = run_shape([2, 3, 256, 256])
    assert ctx.cached_graph_count() == 2  # LRU capacity 2: oldest evicted
    assert y2.shape == (2, 1000)


def test_tuning_cache_written_once(cuda, tmp_path):
    import torch

    golden = np.load(GOLDEN / "stem_known_answer.npz")
    model = stem_model(golden["conv_weight"], golden["fc_weight"])
    engine = ct.build_engine(model, enable_cuda_graph=False, enable_profiling=False,
                             tuning_mode=ct.TUNING_TUNE_ON_MISS, tuning_cache_dir=str(tmp_path),
                             tuning_warmup_iterations=1, tuning_measurement_iterations=3)

    def run():
        ctx = engine.create_context()
        x = torch.from_numpy(stem_input()).to(cuda)
        y = torch.empty(1, 1000, device=cuda)
        ctx.bind_tensor("input", x)
        ctx.bind_tensor("output", y, output=True)
        ctx.run()
        assert_close(y.cpu().numpy(), golden["expected"], atol=1e-4, rtol=1e-4, what="tuned")

    run()
    files = sorted(tmp_path.glob("*.json"))
    assert files
    stamps = {f.name: f.stat().st_mtime_ns for f in files}
    time.sleep(0.05)
    run()
    assert {f.name: f.stat().st_mtime_ns for f in tmp_path.glob("*.json")} == stamps


def test_tuner_skips_a_candidate_that_reports_an_error(cuda, tmp_path):
    """A 1x1 conv whose input is bound 4 bytes past a 16-byte boundary: the
    output-channels-on-M candidate rejects the binding (it reports a shape
    error instead of computing), so TuneOnMiss must leave it out, clear the
    error and run the op on a candidate that handles the binding."""
    import torch

    rng = np.random.default_rng(5)
    n, c, h, k = 2, 64, 8, 128
    x = rng.standard_normal((n, c, h, h)).astype(np.float32)
    w = (rng.standard_normal((k, c, 1, 1)) * 0.1).astype(np.float32)
    bn = [rng.uniform(0.5, 1.5, k).astype(np.float32), (rng.standard_normal(k) * 0.1).astype(np.float32),
          (rng.standard_normal(k) * 0.1).astype(np.float32), rng.uniform(0.5, 1.5, k).astype(np.float32)]
    model = ct.Model()
    model.add_input("x", [n, c, h, h])
    model.add_constant("w", w, layout="OIHW")
    for name, value in zip(("s", "b", "m", "v"), bn):
        model.add_constant(name, value, layout="")
    model.add_node("conv", "FusedConvBatchNormRelu", ["x", "w", "s", "b", "m", "v"], ["y"], strides=[1, 1],
                   pads=[0, 0, 0, 0], dilations=[1, 1], batchnorm_epsilon=1e-5)
    model.add_output("y")
    engine = ct.build_engine(model, enable_cuda_graph=False, tuning_mode=ct.TUNING_TUNE_ON_MISS,
                             tuning_cache_dir=str(tmp_path), tuning_warmup_iterations=1,
                             tuning_measurement_iterations=3)
    assert any("tcgen05_mn" in cand for cand in engine.ops()[0]["candidates"])
    flat = torch.empty(x.size + 1, device=cuda)
    xd = flat[1:].view(n, c, h, h)  # 4 bytes past the allocation's alignment
    xd.copy_(torch.from_numpy(x))
    assert xd.data_ptr() % 16 == 4
    y = torch.empty(n, k, h, h, device=cuda)
    ctx = engine.create_context()
    ctx.bind_tensor("x", xd)
    ctx.bind_tensor("y", y, output=True)
    ctx.run()
    chosen = engine.ops()[0]["candidates"][ctx.selected_candidate(0)]
    assert "tcgen05_mn" not in chosen, chosen
    expected = oracle.conv2d(x, w, bn=bn, relu=True)
    assert_close(y.cpu().numpy(), expected, atol=1e-4, rtol=1e-4, what=f"tuned around the misaligned input ({chosen})")
    ctx.run()  # the error word was cleared: a second run is clean too


def ffn17_model(golden):
    model = ct.Model()
    model.add_input("x", [17, 128], dtype=np.float16, layout="")
    model.add_input("residual", [17, 512], dtype=np.float16, layout="")
    model.add_constant("weight", golden["weight"].astype(np.float16), layout="")
    model.add_constant("scale", golden["scale"].astype(np.float16), layout="")
    model.add_constant("bias", golden["bias"].astype(np.float16), layout="")
    model.add_node("projection", "Gemm", ["x", "weight"], ["projected"])
    model.add_node("activation", "Gelu", ["projected"], ["activated"])
    model.add_node("residual_add", "Add", ["activated", "residual"], ["sum"])
    model.add_node("output_norm", "LayerNormalization", ["sum", "scale", "bias"], ["output"], axis=-1, epsilon=1e-5)
    model.add_output("output")
    return model


def test_fp16_ffn17_known_answer(cuda):
    golden = np.load(GOLDEN / "ffn17_known_answer.npz")
    model = ffn17_model(golden)
    engine = ct.build_engine(model, enable_cuda_graph=True, tuning_mode=ct.TUNING_DISABLED)
    assert [o["op_type"] for o in engine.ops()] == ["GemmGelu", "SkipLayerNormalization"]
    feeds = {"x": golden["x"].astype(np.float16), "residual": golden["residual"].astype(np.float16)}
    for op_index in (0, 1):
        for cand in range(len(engine.ops()[op_index]["candidates"])):
            out, _ = run_graph(model, feeds, {"output": ((17, 512), np.float16)}, candidate=(op_index, cand),
                               enable_cuda_graph=True)
            assert_close(out["output"], golden["expected"], atol=2e-2, rtol=2e-2,
                         what=f"ffn17 op{op_index} cand{cand}")


@pytest.mark.parametrize("tokens,hidden,inner", [(64, 768, 3072), (17, 256, 1024)])
def test_ffn_block_vs_oracle(cuda, tokens, hidden, inner):
    w = workloads.ffn_weights(hidden, inner, seed=3)
    x = workloads.ffn_input(tokens, hidden, seed=3)
    model = workloads.build_ffn(w, tokens, hidden, inner)
    out, engine = run_graph(model, {"x": x}, {"output": ((tokens, hidden), np.float16)})
    assert [o["op_type"] for o in engine.ops()] == ["GemmGelu", "Gemm", "SkipLayerNormalization"]
    h = oracle.gemm_f16(x, w["w1"], gelu=True)
    y = oracle.gemm_f16(h, w["w2"])
    expected = oracle.layer_norm_f16(y, w["gamma"], w["beta"], residual=x)
    assert_close(out["output"], expected, atol=2e-2, rtol=2e-2, what="FFN block")


def check_logits(actual, expected, what):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    bound = 1e-3 * np.abs(expected).max()
    err = np.abs(actual - expected).max()
    assert err <= bound, f"{what}: max|d|={err:.3e} > 1e-3*max|logit|={bound:.3e}"
    # Top-1 must agree; where the expected logits tie at the maximum (the
    # periodic pattern weights produce ties) any of the tied classes counts.
    rows = np.arange(actual.shape[0])
    picked = expected[rows, actual.argmax(axis=1)]
    assert (picked == expected.max(axis=1)).all(), f"{what}: top-1 differs"


@pytest.mark.parametrize("residual_fusion", [False, True])
def test_resnet50_pattern_weights_vs_reference_model(cuda, residual_fusion):
    golden = np.load(GOLDEN / "resnet50_pattern_bs1.npz")["logits"]
    weights = workloads.resnet50_weights("pattern")
    model = workloads.build_resnet50(weights, batch=1)
    out, _ = run_graph(model, {"input": workloads.resnet50_input(1, mode="pattern")},
                       {"output": ((1, 1000), np.float32)}, enable_residual_fusion=residual_fusion,
                       enable_cuda_graph=True)
    check_logits(out["output"], golden, "ResNet-50 pattern bs1")
    # The reference's own tolerance for this model: allclose 1e-4 / 1e-4.
    assert_close(out["output"], golden, atol=1e-4, rtol=1e-4, what="ResNet-50 pattern allclose")


def test_resnet50_baseline_weights_vs_torch(cuda):
    from oracle import torch_ref

    weights = workloads.resnet50_weights("baseline", seed=0)
    x = workloads.resnet50_input(4, seed=0)
    model = workloads.build_resnet50(weights, batch=4)
    out, _ = run_graph(model, {"input": x}, {"output": ((4, 1000), np.float32)}, enable_residual_fusion=True,
                       enable_cuda_graph=True)
    expected = torch_ref.resnet50_logits(x, weights)
    check_logits(out["output"], expected, "ResNet-50 baseline bs4")


def test_run_host_matches_device_run(cuda):
    import torch

    w = workloads.ffn_weights(256, 1024, seed=5)
    x = workloads.ffn_input(32, 256, seed=5)
    model = workloads.build_ffn(w, 32, 256, 1024)
    engine = ct.build_engine(model, tuning_mode=ct.TUNING_DISABLED)
    ctx = engine.create_context()
    dx = torch.empty(32, 256, dtype=torch.float16, device=cuda)
    dy = torch.empty(32, 256, dtype=torch.float16, device=cuda)
    ctx.bind_tensor("x", dx)
    ctx.bind_tensor("output", dy, output=True)
    host_out = np.zeros((32, 256), np.float16)
    ctx.run_host({"x": x}, {"output": host_out})
    stream = torch.cuda.Stream()
    host_out2 = np.zeros((32, 256), np.float16)
    ctx.run_host({"x": x}, {"output": host_out2}, stream=stream.cuda_stream)
    assert np.array_equal(host_out, host_out2)
    assert np.array_equal(host_out, dy.cpu().numpy())


def test_run_host_async_two_contexts_pipeline(cuda):
    """Two contexts of one engine on two streams, each step enqueued without waiting."""
    import torch

    w = workloads.ffn_weights(256, 1024, seed=6)
    model = workloads.build_ffn(w, 32, 256, 1024)
    engine = ct.build_engine(model, tuning_mode=ct.TUNING_DISABLED)
    ctxs, streams = [], []
    for _ in range(2):
        ctx = engine.create_context()
        ctx.bind_tensor("x", torch.empty(32, 256, dtype=torch.float16, device=cuda))
        ctx.bind_tensor("output", torch.empty(32, 256, dtype=torch.float16, device=cuda), output=True)
        ctxs.append(ctx)
        streams.append(torch.cuda.Stream())
    xs = [torch.from_numpy(workloads.ffn_input(32, 256, seed=10 + i)).pin_memory() for i in range(4)]
    outs = [torch.zeros(32, 256, dtype=torch.float16).pin_memory() for _ in range(4)]
    for i in range(4):
        j = i % 2
        if i >= 2:
            ctxs[j].synchronize()
        ctxs[j].run_host_async({"x": xs[i].numpy()}, {"output": outs[i].numpy()}, streams[j].cuda_stream)
    for ctx in ctxs:
        ctx.synchronize()
    for i in range(4):
        expected = np.zeros((32, 256), np.float16)
        ctxs[0].run_host({"x": xs[i].numpy()}, {"output": expected})
        assert np.array_equal(outs[i].numpy(), expected)
    with pytest.raises(ValueError):
        ctxs[0].run_host_async({"x": xs[0].numpy()}, {"output": outs[0].numpy()}, 0)
