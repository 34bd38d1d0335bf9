"""Python facade over the native engine, in the shape of the reference's
``cutriton.compile`` (python/cutriton/api.py:51-99).

``compile(path, target)`` reads a model file — the reference's lightweight
JSON graph IR (``{"inputs", "outputs", "nodes": [{"name", "op_type",
"inputs", "outputs", ...attributes}], "constants"?}``) or an ONNX file (read by
:mod:`cutriton_b200.onnx_import`, no ``onnx`` package needed) — and returns an
:class:`Engine`. ``Engine.create_context().run({name: array})`` returns the
graph outputs as numpy arrays.

Unlike the reference's facade, which runs numpy reference operators, every
run goes through the compiled sm_100a engine on the GPU: the first run with a
given set of input shapes builds a native Engine for those shapes (cached),
copies the inputs to the device, runs and copies the outputs back. The
``cpu_reference`` target is rejected, as the native ``cpu_reference`` backend
has no kernels (and the reference's returns Unsupported too).

ONNX operators map onto the engine's op set: Conv (group 1, no bias), BatchNormalization, Relu, Add,
MaxPool, GlobalAveragePool, Flatten (axis 1), Gemm / MatMul (2-D, no bias;
a constant B with transB = 1 is transposed at import), Gelu, LayerNormalization
(last axis), Softmax (last axis), SkipLayerNormalization. Anything else raises
:class:`UnsupportedModelError` naming the node.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Mapping

import numpy as np

from . import FLOAT16, Model, build_engine
from .onnx_import import load_onnx

SUPPORTED_TARGETS = {"cuda_sm100", "cuda_triton", "cpu_reference"}
_RESERVED_NODE_KEYS = {"name", "op_type", "inputs", "outputs", "attributes", "domain"}


class UnsupportedModelError(ValueError):
    pass


def compile(model_path: str | Path, target: str = "cuda_sm100", **options: Any) -> "Engine":  # noqa: A001
    """Reads `model_path` (.json graph IR or .onnx) for `target`; `options`
    are CompileOptions fields passed to every native build."""
    if target not in SUPPORTED_TARGETS:
        raise ValueError(f"unknown target {target!r}; choose one of {sorted(SUPPORTED_TARGETS)}")
    if target == "cpu_reference":
        raise UnsupportedModelError("the cpu_reference backend has no kernels; use target 'cuda_sm100'")
    path = Path(model_path)
    if not path.exists():
        raise FileNotFoundError(path)
    suffix = path.suffix.lower()
    if suffix == ".json":
        ir = _normalise_json(json.loads(path.read_text(encoding="utf-8")), path.stem)
    elif suffix == ".onnx":
        ir = load_onnx(path)
    else:
        raise ValueError("model files are .json (graph IR) or .onnx")
    _check_ops(ir)
    return Engine(model_path=path, target=target, plan=ir, options=dict(options))


def _normalise_json(doc: dict[str, Any], default_name: str) -> dict[str, Any]:
    nodes = []
    for index, node in enumerate(doc.get("nodes", [])):
        attrs = dict(node.get("attributes") or {})
        attrs.update({k: v for k, v in node.items() if k not in _RESERVED_NODE_KEYS})
        nodes.append({"name": node.get("name") or f"{node['op_type']}_{index}", "op_type": node["op_type"],
                      "inputs": list(node.get("inputs", [])), "outputs": list(node.get("outputs", [])),
                      "attributes": attrs, "domain": node.get("domain", "")})
    constants = {}
    for name, spec in (doc.get("constants") or {}).items():
        if isinstance(spec, dict):
            constants[name] = np.asarray(spec["data"], dtype=spec.get("dtype", "float32")).reshape(spec["shape"])
        else:
            constants[name] = np.asarray(spec, dtype=np.float32)
    return {"name": doc.get("name", default_name), "inputs": list(doc.get("inputs", [])),
            "outputs": list(doc.get("outputs", [])), "input_shapes": dict(doc.get("input_shapes") or {}),
            "input_dtypes": dict(doc.get("input_dtypes") or {}), "nodes": nodes, "constants": constants}


_SIMPLE = {"Relu", "Add", "GlobalAveragePool", "Gelu", "SkipLayerNormalization"}
_KNOWN = _SIMPLE | {"Conv", "BatchNormalization", "MaxPool", "Flatten", "Gemm", "MatMul", "LayerNormalization",
                    "Softmax"}


def _check_ops(ir: dict[str, Any]) -> None:
    for node in ir["nodes"]:
        if node["op_type"] not in _KNOWN:
            raise UnsupportedModelError(f"node {node['name']!r}: op {node['op_type']} is not supported by cuda_sm100")


def _layout(rank: int) -> str:
    return "NCHW" if rank == 4 else ""


def _to_model(ir: dict[str, Any], shapes: dict[str, tuple[int, ...]], dtypes: dict[str, np.dtype]) -> Model:
    """The IR at concrete input shapes as a native Model."""
    model = Model()
    for name in ir["inputs"]:
        model.add_input(name, list(shapes[name]), dtype=dtypes[name], layout=_layout(len(shapes[name])))
    constants = dict(ir["constants"])
    conv_weights = {n["inputs"][1] for n in ir["nodes"] if n["op_type"] == "Conv" and len(n["inputs"]) > 1}
    used: set[str] = set()
    nodes = []
    for node in ir["nodes"]:
        op, attrs, ins = node["op_type"], dict(node["attributes"]), list(node["inputs"])
        where = f"node {node['name']!r} ({op})"
        if op == "Conv":
            if int(attrs.get("group", 1)) != 1 or len(ins) != 2:
                raise UnsupportedModelError(f"{where}: grouped or biased convolutions are not supported")
            out = {"strides": attrs.get("strides", [1, 1]), "pads": attrs.get("pads", [0, 0, 0, 0]),
                   "dilations": attrs.get("dilations", [1, 1])}
        elif op == "BatchNormalization":
            out = {"epsilon": float(attrs.get("epsilon", 1e-5))}
        elif op == "MaxPool":
            if int(attrs.get("ceil_mode", 0)) != 0:
                raise UnsupportedModelError(f"{where}: ceil_mode is not supported")
            out = {"kernel_shape": attrs["kernel_shape"], "strides": attrs.get("strides", [1, 1]),
                   "pads": attrs.get("pads", [0, 0, 0, 0]), "dilations": attrs.get("dilations", [1, 1])}
        elif op == "Flatten":
            if int(attrs.get("axis", 1)) != 1:
                raise UnsupportedModelError(f"{where}: only axis 1 is supported")
            out = {}
        elif op in ("Gemm", "MatMul"):
            if len(ins) != 2:
                raise UnsupportedModelError(f"{where}: a bias input is not supported (add it as a separate node)")
            if float(attrs.get("alpha", 1.0)) != 1.0 or int(attrs.get("transA", 0)) != 0:
                raise UnsupportedModelError(f"{where}: alpha != 1 and transA are not supported")
            if int(attrs.get("transB", 0)) == 1:
                if ins[1] not in constants:
                    raise UnsupportedModelError(f"{where}: transB needs a constant B")
                transposed = ins[1] + "::transposed"
                constants[transposed] = np.ascontiguousarray(np.asarray(constants[ins[1]]).T)
                ins[1] = transposed
            op, out = "Gemm", {}
        elif op in ("LayerNormalization", "Softmax"):
            # The pack's row kernels normalise the last axis of [rows, cols].
            if int(attrs.get("axis", -1)) not in (-1, 1):
                raise UnsupportedModelError(f"{where}: only the last axis of a 2-D tensor is supported")
            out = {"axis": -1}
            if op == "LayerNormalization":
                out["epsilon"] = float(attrs.get("epsilon", 1e-5))
        elif op == "Gelu":
            if attrs.get("approximate", "none") not in ("none", ""):
                raise UnsupportedModelError(f"{where}: only the exact (erf) GELU is supported")
            out = {}
        else:
            out = {}
        used.update(ins)
        nodes.append((node["name"], op, ins, list(node["outputs"]), out))
    for name, array in constants.items():
        if name not in used:
            continue
        array = np.asarray(array)
        if array.dtype == np.float64:
            array = array.astype(np.float32)
        if array.dtype not in (np.float32, np.float16):
            raise UnsupportedModelError(f"constant {name!r}: dtype {array.dtype} is not supported")
        model.add_constant(name, array, layout="OIHW" if name in conv_weights else "")
    for name, op, ins, outs, attrs in nodes:
        model.add_node(name, op, ins, outs, **attrs)
    for name in ir["outputs"]:
        model.add_output(name)
    return model


@dataclass
class Engine:
    """A model read for a target; native engines are built per input shapes."""

    model_path: Path
    target: str
    plan: dict[str, Any] = field(default_factory=dict)
    options: dict[str, Any] = field(default_factory=dict)
    _built: dict[tuple, Any] = field(default_factory=dict, repr=False)

    def create_context(self) -> "ExecutionContext":
        return ExecutionContext(self)

    def native(self, shapes: Mapping[str, tuple[int, ...]], dtypes: Mapping[str, Any] | None = None):
        """The native Engine for these input shapes (built once, then cached)."""
        dtypes = {n: np.dtype((dtypes or {}).get(n, self.plan["input_dtypes"].get(n, "float32")))
                  for n in self.plan["inputs"]}
        shapes = {n: tuple(int(d) for d in shapes[n]) for n in self.plan["inputs"]}
        for name, declared in self.plan["input_shapes"].items():
            got = shapes.get(name)
            if got is not None and (len(declared) != len(got)
                                    or any(d > 0 and d != g for d, g in zip(declared, got))):
                raise ValueError(f"input {name!r}: shape {got} does not fit the model's {declared}")
        key = tuple((n, shapes[n], dtypes[n].str) for n in self.plan["inputs"])
        if key not in self._built:
            self._built[key] = build_engine(_to_model(self.plan, shapes, dtypes), **self.options)
        return self._built[key]


class ExecutionContext:
    def __init__(self, engine: Engine):
        self.engine = engine
        self._contexts: dict[int, tuple[Any, dict[str, Any]]] = {}

    def run(self, inputs: Mapping[str, Any]) -> dict[str, np.ndarray]:
        """Copies `inputs` to the GPU, runs the compiled engine and returns
        every graph output as a host array."""
        import torch

        plan = self.engine.plan
        missing = [n for n in plan["inputs"] if n not in inputs]
        if missing:
            raise ValueError(f"missing inputs: {missing}")
        arrays = {n: np.ascontiguousarray(np.asarray(
            inputs[n], dtype=plan["input_dtypes"].get(n, getattr(inputs[n], "dtype", np.float32))))
            for n in plan["inputs"]}
        native = self.engine.native({n: a.shape for n, a in arrays.items()}, {n: a.dtype for n, a in arrays.items()})
        entry = self._contexts.get(id(native))
        if entry is None:
            ctx = native.create_context()
            device: dict[str, Any] = {}
            for n, a in arrays.items():
                device[n] = torch.empty(a.shape, dtype=getattr(torch, a.dtype.name), device="cuda")
                ctx.bind_tensor(n, device[n])
            for n in plan["outputs"]:
                code, shape = native.value_desc(n)
                dtype = np.float16 if code == FLOAT16 else np.float32
                device[n] = torch.empty(shape, dtype=getattr(torch, np.dtype(dtype).name), device="cuda")
                ctx.bind_tensor(n, device[n], output=True)
            entry = (ctx, device)
            self._contexts[id(native)] = entry
        ctx, device = entry
        outputs = {n: np.empty(tuple(device[n].shape), dtype=np.float16 if device[n].dtype == torch.float16
                               else np.float32) for n in plan["outputs"]}
        ctx.run_host(arrays, outputs)
        return outputs
