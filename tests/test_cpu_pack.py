"""Kernel Pack loader and SDK: schema/ABI/SHA/SM/grid validation (negative
cases of the reference's tests/cpp/test_cuda.cpp:488-552 and
tests/python/test_kernel_sdk.py:45-107), exercised without a GPU."""

from __future__ import annotations

import json
import shutil
from pathlib import Path

import numpy as np
import pytest

import cutriton_b200 as ct
from cutriton_b200 import kernel_sdk, kernel_specs


@pytest.fixture()
def relu_model():
    model = ct.Model()
    model.add_input("x", [1, 4, 5, 5])
    model.add_node("relu", "Relu", ["x"], ["y"])
    model.add_output("y")
    return model


@pytest.fixture()
def assume_sm100(monkeypatch):
    monkeypatch.setenv("CUTRITON_ASSUME_COMPUTE_CAPABILITY", "100")


def copy_pack(tmp_path: Path) -> Path:
    dst = tmp_path / "pack"
    shutil.copytree(ct.PACK_DIR, dst, ignore=shutil.ignore_patterns("tuning"))
    return dst


def test_builtin_pack_compiles_graph(relu_model, assume_sm100):
    engine = ct.build_engine(relu_model)
    ops = engine.ops()
    assert [o["op_type"] for o in ops] == ["Relu"]
    assert ops[0]["candidates"][ops[0]["default"]].startswith("cutriton_sm100:relu.fp32")


def test_missing_pack_is_not_found(relu_model, assume_sm100, tmp_path):
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(tmp_path / "missing"))
    assert err.value.code == ct.NOT_FOUND


def test_schema_v1_is_rejected(relu_model, assume_sm100, tmp_path):
    pack = copy_pack(tmp_path)
    doc = json.loads((pack / "pack.json").read_text())
    doc["schema_version"] = 1
    (pack / "pack.json").write_text(json.dumps(doc))
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert err.value.code == ct.INVALID_ARGUMENT


def test_sha_mismatch_is_rejected(relu_model, assume_sm100, tmp_path):
    pack = copy_pack(tmp_path)
    cubin = next((pack / "kernels").rglob("*.cubin"))
    with open(cubin, "ab") as f:
        f.write(b"\0")
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert err.value.code == ct.INVALID_ARGUMENT
    assert "SHA-256" in str(err.value)


def test_sm_mismatch_is_unsupported(relu_model, assume_sm100, tmp_path):
    pack = copy_pack(tmp_path)
    doc = json.loads((pack / "pack.json").read_text())
    for k in doc["kernels"]:
        k["min_compute_capability"] = 999
    (pack / "pack.json").write_text(json.dumps(doc))
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert err.value.code == ct.UNSUPPORTED


@pytest.mark.parametrize("mutation", [
    lambda k: k.__setitem__("grid", [{"kind": "python", "expression": "unsafe"}]),
    lambda k: k["arguments"].pop(),                                  # reserved tail broken
    lambda k: k.__setitem__("binary", "../escape.cubin"),
    lambda k: k["constraints"].append({"kind": "lambda", "value": 1}),
    lambda k: k["arguments"][0]["source"].__setitem__("kind", "eval"),
    lambda k: k.__setitem__("binary_format", "elf"),
])
def test_unsafe_manifest_entries_are_rejected(relu_model, assume_sm100, tmp_path, mutation):
    pack = copy_pack(tmp_path)
    doc = json.loads((pack / "pack.json").read_text())
    mutation(doc["kernels"][0])
    (pack / "pack.json").write_text(json.dumps(doc))
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert err.value.code == ct.INVALID_ARGUMENT


@pytest.mark.parametrize("swizzle,atom", [(128, 64), (64, 32)])
def test_tensor_map_swizzle_atom_is_validated(relu_model, assume_sm100, tmp_path, swizzle, atom):
    """swizzle_atom (32-byte atoms of the 128-byte swizzle) is accepted only
    as 32 with a 128-byte swizzle; anything else fails the pack load."""
    pack = copy_pack(tmp_path)
    doc = json.loads((pack / "pack.json").read_text())
    maps = [a["source"] for k in doc["kernels"] for a in k["arguments"] if a["source"]["kind"] == "tensor_map"]
    assert any(m.get("swizzle_atom") == 32 and m.get("swizzle") == 128 for m in maps)
    maps[0]["swizzle"] = swizzle
    maps[0]["swizzle_atom"] = atom
    (pack / "pack.json").write_text(json.dumps(doc))
    with pytest.raises(ct.CutritonError) as err:
        ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert err.value.code == ct.INVALID_ARGUMENT


def test_abi_v1_grid_is_accepted(relu_model, assume_sm100, tmp_path):
    pack = copy_pack(tmp_path)
    doc = json.loads((pack / "pack.json").read_text())
    doc["abi_schema_version"] = 1
    for k in doc["kernels"]:
        k["grid"] = {"op": "ceil_div", "value": {"kind": "output_numel", "index": 0}, "divisor": 4096}
    (pack / "pack.json").write_text(json.dumps(doc))
    engine = ct.build_engine(relu_model, kernel_artifact_dir=str(pack))
    assert engine.num_ops() == 1


def test_sdk_validates_specs():
    specs = kernel_specs.all_specs()
    for spec in specs:
        spec.validate()
    base = next(s for s in specs if s.kernel_id == "relu.fp32")

    def variant(**kw):
        return kernel_sdk.Variant(**{"variant_id": "v", "num_warps": 8, "meta": {"CHUNK": 4096}, "default": True, **kw})

    with pytest.raises(ValueError):  # an op without a default variant
        kernel_sdk.validate_pack([kernel_sdk.KernelSpec(**{**base.__dict__, "variants": (variant(default=False),)})])
    kernel_sdk.validate_pack(specs)
    bad = [
        kernel_sdk.KernelSpec(**{**base.__dict__, "variants": (variant(), variant())}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "arguments": base.arguments[:-1]}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "arguments": (kernel_sdk.Arg("x", "*fp32", {"kind": "eval"}),)
                                 + base.arguments[1:]}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "grid": ({"kind": "python"},)}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "variants": (variant(meta={}),)}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "constraints": ({"kind": "lambda"},)}),
        kernel_sdk.KernelSpec(**{**base.__dict__, "arguments": (kernel_sdk.Arg(
            "x", "*fp32", {"kind": "input", "index": 0, "prepack": "unknown"}),) + base.arguments[1:]}),
        # 32-byte swizzle atoms exist only for the 128-byte swizzle.
        kernel_sdk.KernelSpec(**{**base.__dict__, "arguments": (kernel_sdk.Arg(
            "m", "tensormap", {"kind": "tensor_map", "tensor": "input", "index": 0, "box": [32, 32],
                               "swizzle": 64, "swizzle_atom": 32}),) + base.arguments[1:]}),
    ]
    for spec in bad:
        with pytest.raises(ValueError):
            spec.validate()


def test_pack_entries_are_cubins_for_sm100():
    doc = json.loads((ct.PACK_DIR / "pack.json").read_text())
    assert doc["schema_version"] == 2 and doc["abi_schema_version"] == 2
    for k in doc["kernels"]:
        assert k["binary_format"] == "cubin"
        assert k["min_compute_capability"] == 100
        data = (ct.PACK_DIR / k["binary"]).read_bytes()
        assert data[:4] == b"\x7fELF"
    op_defaults = {}
    for k in doc["kernels"]:
        op_defaults.setdefault((k["op_type"], k["dtype"]), []).append(k["default"])
    for key, flags in op_defaults.items():
        assert sum(flags) == 1, key


def _kernel_constant(source: str, name: str) -> int:
    import re

    match = re.search(rf"constexpr (?:int|uint32_t) {name} = (\d+)u?;", source)
    assert match, f"{name} not found"
    return int(match.group(1))


def test_launch_shapes_match_the_kernels():
    """The launcher takes block size, shared memory and tensor-map boxes from
    the pack; each must agree with what the kernel was compiled to expect."""
    from cutriton_b200 import kernel_specs
    from cutriton_b200.kernel_sdk import _variant_arguments

    kernels = Path(kernel_specs.__file__).resolve().parent / "csrc" / "kernels"
    checked = set()
    for spec in kernel_specs.all_specs():
        for variant in spec.variants:
            args = {a["name"]: a["source"] for a in _variant_arguments(spec, variant)}
            if spec.source in ("gemm_f16_tp.cu", "gemm_f16_2sm.cu"):
                gemm = (kernels / spec.source).read_text()
                epilogue_warps = _kernel_constant(gemm, "kEpilogueWarps")
                chunk = _kernel_constant(gemm, "kChunk")
                # producer + issuer + epilogue warps; 32 x chunk FP16 store box, swizzle = its row bytes
                assert variant.num_warps == 2 + epilogue_warps, spec.kernel_id
                assert args["tma_out"]["box"] == [chunk, 32], spec.kernel_id
                assert args["tma_out"]["swizzle"] == 2 * chunk, spec.kernel_id
                # stage ring + store staging + barriers + 1 KB alignment slack
                ring = _kernel_constant(gemm, "kRingBytes")
                need = ring + epilogue_warps * 32 * chunk * 2 + 1024
                assert need < variant.shared_memory_bytes <= 232448, spec.kernel_id
                checked.add(spec.source)
            if spec.source == "gemm_f16_2sm.cu":
                # A: 128 rows per CTA; B^T: half of each tile width (256, 192, 128) per CTA
                assert args["tma_a"]["box"] == [64, 128], spec.kernel_id
                for rows in (128, 96, 64):
                    assert args[f"tma_b{rows}"]["box"] == [64, rows], spec.kernel_id
                    assert args[f"tma_b{rows}"]["prepack"] == "transpose_2d", spec.kernel_id
            if spec.source == "conv_tm.cu":
                d = variant.defines
                warps = 2 + int(d["CTB_TM_EPI_WARPS"]) + 4 * int(d["CTB_TM_GATHER_GROUPS"])
                assert variant.num_warps == warps, (spec.kernel_id, variant.variant_id)
                # weight stages + barriers + chunk table + staging ring + activation ring + windows + alignment
                stages = max(int(d["CTB_TM_STAGES_N128"]) * 32768, int(d["CTB_TM_STAGES_N64"]) * 16384)
                need = stages + 512 + 1024 + int(d["CTB_TM_SLOTS"]) * 16384 + 1024
                if d["CTB_TM_A_TMA"] == "1":
                    need += 4 * 16384
                if d.get("CTB_TM_WINDOW") == "1":
                    need += 2 * 232 * 11 * 4 * 4
                assert need <= variant.shared_memory_bytes <= 232448, (spec.kernel_id, variant.variant_id)
                checked.add(spec.source)
    assert checked == {"gemm_f16_tp.cu", "gemm_f16_2sm.cu", "conv_tm.cu"}


def test_conv1x1_mn_shared_memory_matches_the_kernel():
    """The output-channels-on-M 1x1 kernel: 10 warps, and shared memory for
    its stages (three without a residual, two with one; 64 KB each) and the
    epilogue boxes (two output boxes per warp, plus four residual slots)."""
    from cutriton_b200 import kernel_specs

    source = (Path(kernel_specs.__file__).resolve().parent / "csrc" / "kernels" / "conv1x1_mn.cu").read_text()
    assert "kStages = kResidual ? 2 : 3" in source
    assert _kernel_constant(source, "kMaxResSlots") == 4 and _kernel_constant(source, "kOutSlots") == 2
    assert _kernel_constant(source, "kEpiWarps") == 4
    specs = [s for s in kernel_specs.all_specs() if s.source == "conv1x1_mn.cu"]
    assert len(specs) == 4
    for spec in specs:
        residual = spec.op_type.endswith("AddRelu")
        stage = 2 * (128 * 32 * 4) + 2 * (4 * 32 * 32 * 4)  # W_hi, W_lo, X_hi, X_lo
        epilogue = 4 * ((4 if residual else 0) + 2) * 32 * 32 * 4
        need = (2 if residual else 3) * stage + epilogue + 1024
        (variant,) = spec.variants
        assert variant.num_warps == 10
        assert need < variant.shared_memory_bytes <= 232448, spec.kernel_id


def test_window_variant_keeps_its_full_window_box():
    """The stem's input-window variant loads {232 columns, 11 rows, 4
    channels, 1 image} per tile and waits for exactly that many bytes; the
    other variants of its family bind the window map with a tiny unused box.
    A variant that loads windows must never get the tiny box."""
    import json

    from cutriton_b200 import _build

    pack = json.loads((_build.PACK_DIR / "pack.json").read_text())  # built by the session fixture
    window = [k for k in pack["kernels"] if k["variant_id"].endswith("_window")]
    assert window
    for entry in window:
        boxes = [a["source"]["box"] for a in entry["arguments"] if a["name"] == "tma_xwin"]
        assert boxes == [[232, 11, 4, 1]], (entry["kernel_id"], boxes)
