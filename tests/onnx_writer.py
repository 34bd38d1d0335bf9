"""Minimal ONNX protobuf writer for tests (the onnx package is not
installed): enough of ModelProto / GraphProto / NodeProto / AttributeProto /
TensorProto / ValueInfoProto, with onnx.proto's field numbers, to build small
models byte for byte."""

from __future__ import annotations

import struct

import numpy as np

FLOAT, INT64, FLOAT16 = 1, 7, 10


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(number: int, wire: int) -> bytes:
    return _varint((number << 3) | wire)


def field_bytes(number: int, payload: bytes) -> bytes:
    return _key(number, 2) + _varint(len(payload)) + payload


def field_str(number: int, text: str) -> bytes:
    return field_bytes(number, text.encode())


def field_int(number: int, value: int) -> bytes:
    return _key(number, 0) + _varint(value)


def field_float(number: int, value: float) -> bytes:
    return _key(number, 5) + struct.pack("<f", value)


def attribute(name: str, value) -> bytes:
    body = field_str(1, name)
    if isinstance(value, float):
        body += field_float(2, value) + field_int(20, 1)
    elif isinstance(value, int):
        body += field_int(3, value) + field_int(20, 2)
    elif isinstance(value, str):
        body += field_bytes(4, value.encode()) + field_int(20, 3)
    else:  # list of ints, packed
        body += field_bytes(8, b"".join(_varint(int(v)) for v in value)) + field_int(20, 7)
    return body


def tensor(name: str, array: np.ndarray) -> bytes:
    array = np.ascontiguousarray(array)
    dtype = {np.dtype(np.float32): FLOAT, np.dtype(np.float16): FLOAT16, np.dtype(np.int64): INT64}[array.dtype]
    body = b"".join(field_int(1, d) for d in array.shape) + field_int(2, dtype) + field_str(8, name)
    return body + field_bytes(9, array.astype(array.dtype.newbyteorder("<")).tobytes())


def value_info(name: str, shape, elem: int = FLOAT) -> bytes:
    dims = b"".join(field_bytes(1, field_int(1, d) if d >= 0 else field_str(2, "N")) for d in shape)
    tensor_type = field_int(1, elem) + field_bytes(2, dims)
    return field_str(1, name) + field_bytes(2, field_bytes(1, tensor_type))


def node(op_type: str, inputs, outputs, name: str = "", **attrs) -> bytes:
    body = b"".join(field_str(1, i) for i in inputs) + b"".join(field_str(2, o) for o in outputs)
    if name:
        body += field_str(3, name)
    body += field_str(4, op_type)
    body += b"".join(field_bytes(5, attribute(k, v)) for k, v in attrs.items())
    return body


def model(nodes, inputs, outputs, initializers=(), name: str = "g") -> bytes:
    graph = b"".join(field_bytes(1, n) for n in nodes) + field_str(2, name)
    graph += b"".join(field_bytes(5, t) for t in initializers)
    graph += b"".join(field_bytes(11, v) for v in inputs) + b"".join(field_bytes(12, v) for v in outputs)
    opset = field_str(1, "") + field_int(2, 17)
    return field_int(1, 8) + field_str(2, "cutriton_b200-tests") + field_bytes(7, graph) + field_bytes(8, opset)


def conv_block_model(rng: np.random.Generator, n: int = 2, c: int = 3, h: int = 16, k: int = 8,
                     classes: int = 10) -> tuple[bytes, dict[str, np.ndarray]]:
    """Conv 3x3 -> BatchNormalization -> Relu -> MaxPool -> GlobalAveragePool
    -> Flatten -> Gemm(transB=1): a PyTorch-export-shaped ResNet stem + head."""
    w = (rng.standard_normal((k, c, 3, 3)) * 0.2).astype(np.float32)
    bn = [rng.uniform(0.5, 1.5, k).astype(np.float32), (rng.standard_normal(k) * 0.1).astype(np.float32),
          (rng.standard_normal(k) * 0.1).astype(np.float32), rng.uniform(0.5, 1.5, k).astype(np.float32)]
    fc = (rng.standard_normal((classes, k)) * 0.1).astype(np.float32)  # [N, K]: used with transB = 1
    names = ["w", "gamma", "beta", "mean", "var", "fc"]
    arrays = dict(zip(names, [w, *bn, fc]))
    nodes = [
        node("Conv", ["x", "w"], ["c"], "conv", kernel_shape=[3, 3], strides=[1, 1], pads=[1, 1, 1, 1],
             dilations=[1, 1], group=1),
        node("BatchNormalization", ["c", "gamma", "beta", "mean", "var"], ["b"], "bn", epsilon=1e-5),
        node("Relu", ["b"], ["r"], "relu"),
        node("MaxPool", ["r"], ["p"], "pool", kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1]),
        node("GlobalAveragePool", ["p"], ["g"], "gap"),
        node("Flatten", ["g"], ["f"], "flat", axis=1),
        node("Gemm", ["f", "fc"], ["y"], "fc_node", transB=1),
    ]
    blob = model(nodes, [value_info("x", [n, c, h, h])], [value_info("y", [n, classes])],
                 [tensor(nm, arr) for nm, arr in arrays.items()])
    return blob, arrays
