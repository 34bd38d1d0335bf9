"""The Python facade (cutriton_b200.api, the reference's cutriton.compile
shape) and the ONNX reader, on the CPU: files written here (JSON graph IR,
ONNX built byte for byte by tests/onnx_writer.py) are read back exactly and
compile to the expected native plan. Running needs a GPU (test_gpu_api.py)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from cutriton_b200 import api
from cutriton_b200.onnx_import import OnnxFormatError, load_onnx
from tests import onnx_writer as ow


@pytest.fixture()
def assume_sm100(monkeypatch):
    monkeypatch.setenv("CUTRITON_ASSUME_COMPUTE_CAPABILITY", "100")


def test_onnx_reader_recovers_structure_attributes_and_initializers(tmp_path):
    blob, arrays = ow.conv_block_model(np.random.default_rng(1))
    path = tmp_path / "block.onnx"
    path.write_bytes(blob)
    ir = load_onnx(path)
    assert ir["inputs"] == ["x"] and ir["outputs"] == ["y"]
    assert ir["input_shapes"] == {"x": [2, 3, 16, 16]}
    assert [n["op_type"] for n in ir["nodes"]] == ["Conv", "BatchNormalization", "Relu", "MaxPool",
                                                   "GlobalAveragePool", "Flatten", "Gemm"]
    conv = ir["nodes"][0]
    assert conv["attributes"] == {"kernel_shape": [3, 3], "strides": [1, 1], "pads": [1, 1, 1, 1],
                                  "dilations": [1, 1], "group": 1}
    assert ir["nodes"][1]["attributes"]["epsilon"] == pytest.approx(1e-5)
    assert ir["nodes"][6]["attributes"] == {"transB": 1}
    assert set(ir["constants"]) == set(arrays)
    for name, array in arrays.items():
        np.testing.assert_array_equal(ir["constants"][name], array)


def test_onnx_reader_rejects_truncated_files(tmp_path):
    blob, _ = ow.conv_block_model(np.random.default_rng(2))
    path = tmp_path / "cut.onnx"
    path.write_bytes(blob[: len(blob) // 2])
    with pytest.raises(OnnxFormatError):
        load_onnx(path)


def test_onnx_model_compiles_to_the_fused_plan(tmp_path, assume_sm100):
    blob, _ = ow.conv_block_model(np.random.default_rng(3))
    path = tmp_path / "block.onnx"
    path.write_bytes(blob)
    engine = api.compile(path, target="cuda_triton")
    native = engine.native({"x": (2, 3, 16, 16)})
    assert [o["op_type"] for o in native.ops()] == ["FusedConvBatchNormRelu", "MaxPool", "GlobalAveragePool",
                                                    "Flatten", "Gemm"]
    assert native.value_desc("y")[1] == (2, 10)
    assert engine.native({"x": (2, 3, 16, 16)}) is native  # cached per input shapes
    with pytest.raises(ValueError):
        engine.native({"x": (2, 3, 8, 16)})  # the file fixes H = 16


def test_json_graph_ir_like_the_reference_facade(tmp_path, assume_sm100):
    path = tmp_path / "relu_graph.json"
    path.write_text(json.dumps({"inputs": ["x"], "outputs": ["y"],
                                "nodes": [{"name": "relu", "op_type": "Relu", "inputs": ["x"], "outputs": ["y"]}]}))
    engine = api.compile(path)
    native = engine.native({"x": (3,)})
    assert [o["op_type"] for o in native.ops()] == ["Relu"]


def test_facade_errors(tmp_path):
    path = tmp_path / "g.json"
    path.write_text(json.dumps({"inputs": ["x"], "outputs": ["y"],
                                "nodes": [{"op_type": "Erf", "inputs": ["x"], "outputs": ["y"]}]}))
    with pytest.raises(api.UnsupportedModelError, match="Erf"):
        api.compile(path)
    with pytest.raises(api.UnsupportedModelError):
        api.compile(path, target="cpu_reference")
    with pytest.raises(ValueError):
        api.compile(path, target="rocm")
    with pytest.raises(FileNotFoundError):
        api.compile(tmp_path / "missing.json")
    other = tmp_path / "g.txt"
    other.write_text("{}")
    with pytest.raises(ValueError):
        api.compile(other)
