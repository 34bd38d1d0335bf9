"""The Python facade end to end on the GPU: an ONNX model (built byte for
byte by tests/onnx_writer.py) and JSON graph-IR models compiled by
cutriton_b200.api and run through the native sm_100a engine, against the C
oracle."""

from __future__ import annotations

import json

import numpy as np
import pytest

from cutriton_b200 import api
from oracle import ops as oracle
from tests import onnx_writer as ow
from tests.helpers import assert_bitexact, assert_close

pytestmark = pytest.mark.gpu


def test_onnx_conv_block_runs_on_the_engine(cuda, tmp_path):
    rng = np.random.default_rng(7)
    blob, w = ow.conv_block_model(rng)
    path = tmp_path / "block.onnx"
    path.write_bytes(blob)
    ctx = api.compile(path).create_context()
    x = rng.standard_normal((2, 3, 16, 16)).astype(np.float32)
    for _ in range(2):  # the second run reuses the built engine and bound buffers
        y = ctx.run({"x": x})["y"]
        h = oracle.conv2d(x, w["w"], pads=(1, 1, 1, 1), bn=[w["gamma"], w["beta"], w["mean"], w["var"]], relu=True)
        h = oracle.global_average_pool(oracle.max_pool(h)).reshape(2, -1)
        expected = oracle.gemm_f32(h, np.ascontiguousarray(w["fc"].T))
        assert_close(y, expected, atol=1e-4, rtol=1e-4, what="ONNX conv block")


def test_json_graphs_run_on_the_engine(cuda, tmp_path):
    path = tmp_path / "relu.json"
    path.write_text(json.dumps({"inputs": ["x"], "outputs": ["y"],
                                "nodes": [{"name": "relu", "op_type": "Relu", "inputs": ["x"], "outputs": ["y"]}]}))
    out = api.compile(path).create_context().run({"x": [-1.0, 0.0, 1.0, 2.5]})
    assert_bitexact(out["y"], np.array([0.0, 0.0, 1.0, 2.5], np.float32), "Relu")
    path = tmp_path / "gelu.json"
    path.write_text(json.dumps({"inputs": ["x"], "outputs": ["y"], "input_dtypes": {"x": "float16"},
                                "nodes": [{"name": "gelu", "op_type": "Gelu", "inputs": ["x"], "outputs": ["y"]}]}))
    x = np.linspace(-4, 4, 96, dtype=np.float16).reshape(3, 32)
    y = api.compile(path).create_context().run({"x": x})["y"]
    assert_close(y, oracle.gelu_f16(x), atol=1e-3, rtol=1e-3, what="Gelu")
