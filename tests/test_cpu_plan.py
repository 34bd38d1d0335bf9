"""Compilation of the benchmark graphs without a GPU (lowering uses the
CUTRITON_ASSUME_COMPUTE_CAPABILITY hook): fused plan structure, candidates
and memory planning."""

from __future__ import annotations

from collections import Counter

import numpy as np
import pytest

import cutriton_b200 as ct
from cutriton_b200 import workloads


@pytest.fixture(autouse=True)
def assume_sm100(monkeypatch):
    monkeypatch.setenv("CUTRITON_ASSUME_COMPUTE_CAPABILITY", "100")


@pytest.fixture(scope="module")
def rn_weights():
    return workloads.resnet50_weights("baseline", seed=0)


def test_resnet50_plan_matches_reference_structure(rn_weights):
    engine = ct.build_engine(workloads.build_resnet50(rn_weights, batch=1))
    ops = engine.ops()
    counts = Counter(o["op_type"] for o in ops)
    # 33 Conv+BN+ReLU, 20 Conv+BN (conv3 + 4 downsample), 16 Add+ReLU,
    # MaxPool, GlobalAveragePool, Flatten (view), Gemm: 73 plan ops.
    assert len(ops) == 73
    assert counts == {"FusedConvBatchNormRelu": 33, "FusedConvBatchNorm": 20, "AddRelu": 16, "MaxPool": 1,
                      "GlobalAveragePool": 1, "Flatten": 1, "Gemm": 1}
    flatten = next(o for o in ops if o["op_type"] == "Flatten")
    assert flatten["candidates"] == ["view:flatten"]
    for o in ops:
        if o["op_type"] in ("FusedConvBatchNormRelu", "FusedConvBatchNorm", "AddRelu"):
            assert any(c.startswith("unfused:") for c in o["candidates"]), o
    assert engine.value_desc("output") == (ct.FLOAT32, (1, 1000))
    assert engine.workspace_bytes() % 256 == 0 and engine.workspace_bytes() > 0


def test_residual_fusion_folds_block_tails(rn_weights):
    engine = ct.build_engine(workloads.build_resnet50(rn_weights, batch=1), enable_residual_fusion=True)
    counts = Counter(o["op_type"] for o in engine.ops())
    assert counts["FusedConvBatchNormAddRelu"] == 16
    assert counts.get("AddRelu", 0) == 0
    assert counts["FusedConvBatchNorm"] == 4  # downsample convs stay
    assert engine.num_ops() == 57
    fused = next(o for o in engine.ops() if o["op_type"] == "FusedConvBatchNormAddRelu")
    assert "unfused:conv_bn_add_relu" in fused["candidates"]


def test_ffn_plan_fuses_gemm_gelu_and_skip_layer_norm():
    w = workloads.ffn_weights(768, 3072)
    engine = ct.build_engine(workloads.build_ffn(w, 64, 768, 3072))
    ops = engine.ops()
    assert [o["op_type"] for o in ops] == ["GemmGelu", "Gemm", "SkipLayerNormalization"]
    assert "unfused:gemm_gelu" in ops[0]["candidates"]
    assert "unfused:add_layer_norm" in ops[2]["candidates"]
    unfused = ct.build_engine(workloads.build_ffn(w, 64, 768, 3072), enable_transformer_fusions=False)
    assert [o["op_type"] for o in unfused.ops()] == ["Gemm", "Gelu", "Gemm", "Add", "LayerNormalization"]


def test_dynamic_profile_plans_at_max():
    weights = workloads.resnet50_weights("pattern")
    model = workloads.build_resnet50(weights, dynamic_batch=True)
    model.add_shape_profile("batch", "input", [1, 3, 224, 224], [32, 3, 224, 224], [128, 3, 224, 224])
    engine = ct.build_engine(model)
    ctx = engine.create_context()
    assert ctx.resolved_desc("output")[1] == (32, 1000)
    ctx.set_input_shape("input", [64, 3, 224, 224])
    ctx.resolve_shapes()
    assert ctx.resolved_desc("output")[1] == (64, 1000)
    with pytest.raises(ct.CutritonError) as err:
        ctx.set_input_shape("input", [129, 3, 224, 224])
    assert err.value.code == ct.SHAPE_ERROR


def test_layer_norm_wider_than_1024_is_unsupported():
    model = ct.Model()
    model.add_input("x", [4, 2048], dtype=np.float16, layout="")
    model.add_constant("g", np.ones(2048, np.float16), layout="")
    model.add_constant("b", np.zeros(2048, np.float16), layout="")
    model.add_node("ln", "LayerNormalization", ["x", "g", "b"], ["y"], axis=-1, epsilon=1e-5)
    model.add_output("y")
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(model)
    assert err.value.code == ct.UNSUPPORTED
