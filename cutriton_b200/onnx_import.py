"""ONNX model files -> the graph IR of :mod:`cutriton_b200.api`.

The `onnx` package is not needed: this module reads the protobuf wire format
of the ONNX messages it uses directly (field numbers of onnx.proto):

* ModelProto      graph = 7
* GraphProto      node = 1, name = 2, initializer = 5, input = 11, output = 12
* NodeProto       input = 1, output = 2, name = 3, op_type = 4, attribute = 5, domain = 7
* AttributeProto  name = 1, f = 2, i = 3, s = 4, t = 5, floats = 7, ints = 8, type = 20
* TensorProto     dims = 1, data_type = 2, float_data = 4, int32_data = 5,
                  int64_data = 7, name = 8, raw_data = 9, double_data = 10
* ValueInfoProto  name = 1, type = 2 -> TypeProto.tensor_type = 1 ->
                  elem_type = 1, shape = 2 -> dim = 1 -> dim_value = 1 / dim_param = 2

Besides the structure the reference's facade extracts (python/cutriton/api.py:
77-99: names, op types, inputs, outputs, attribute names), it keeps attribute
values, initializers (FLOAT / FLOAT16 / INT64 tensors) and input shapes, so the
imported graph compiles to a native engine.
"""

from __future__ import annotations

import struct
from pathlib import Path
from typing import Any

import numpy as np

# TensorProto.DataType values used here.
FLOAT, INT64, FLOAT16, DOUBLE, INT32 = 1, 7, 10, 11, 6
_NUMPY = {FLOAT: np.float32, FLOAT16: np.float16, INT64: np.int64, DOUBLE: np.float64, INT32: np.int32}


class OnnxFormatError(ValueError):
    pass


def _varint(buf: bytes, pos: int) -> tuple[int, int]:
    value = shift = 0
    while True:
        if pos >= len(buf):
            raise OnnxFormatError("truncated varint")
        byte = buf[pos]
        pos += 1
        value |= (byte & 0x7F) << shift
        if byte < 0x80:
            return value, pos
        shift += 7
        if shift > 63:
            raise OnnxFormatError("varint too long")


def _fields(buf: bytes):
    """Yields (field number, wire type, value) of one message; length-delimited
    values are bytes, varints ints, fixed32/64 raw bytes."""
    pos = 0
    while pos < len(buf):
        key, pos = _varint(buf, pos)
        number, wire = key >> 3, key & 7
        if wire == 0:
            value, pos = _varint(buf, pos)
        elif wire == 1:
            value, pos = buf[pos:pos + 8], pos + 8
        elif wire == 2:
            length, pos = _varint(buf, pos)
            value, pos = buf[pos:pos + length], pos + length
        elif wire == 5:
            value, pos = buf[pos:pos + 4], pos + 4
        else:
            raise OnnxFormatError(f"unsupported wire type {wire}")
        if pos > len(buf):
            raise OnnxFormatError("truncated field")
        yield number, wire, value


def _signed64(value: int) -> int:
    return value - (1 << 64) if value >= 1 << 63 else value


def _packed_varints(value: Any, wire: int) -> list[int]:
    if wire == 0:
        return [_signed64(value)]
    out, pos = [], 0
    while pos < len(value):
        v, pos = _varint(value, pos)
        out.append(_signed64(v))
    return out


def _floats(value: Any, wire: int) -> list[float]:
    if wire == 5:
        return [struct.unpack("<f", value)[0]]
    return list(struct.unpack(f"<{len(value) // 4}f", value))


def _tensor(buf: bytes) -> tuple[str, np.ndarray]:
    dims: list[int] = []
    dtype = 0
    name = ""
    raw = None
    floats: list[float] = []
    ints: list[int] = []
    for number, wire, value in _fields(buf):
        if number == 1:
            dims += _packed_varints(value, wire)
        elif number == 2:
            dtype = value
        elif number == 4:
            floats += _floats(value, wire)
        elif number in (5, 7):
            ints += _packed_varints(value, wire)
        elif number == 8:
            name = value.decode()
        elif number == 9:
            raw = value
    if dtype not in _NUMPY:
        raise OnnxFormatError(f"initializer {name!r}: data type {dtype} is not supported")
    np_dtype = _NUMPY[dtype]
    if raw is not None:
        array = np.frombuffer(raw, dtype=np.dtype(np_dtype).newbyteorder("<")).astype(np_dtype)
    elif dtype == FLOAT16:
        array = np.array(ints, dtype=np.uint16).view(np.float16)  # int32_data holds the bit patterns
    elif dtype in (FLOAT, DOUBLE):
        array = np.array(floats, dtype=np_dtype)
    else:
        array = np.array(ints, dtype=np_dtype)
    count = int(np.prod(dims)) if dims else 1
    if array.size != count:
        raise OnnxFormatError(f"initializer {name!r}: {array.size} values for shape {dims}")
    return name, array.reshape(dims)


def _attribute(buf: bytes) -> tuple[str, Any]:
    name = ""
    f = i = s = t = None
    floats: list[float] = []
    ints: list[int] = []
    kind = None
    for number, wire, value in _fields(buf):
        if number == 1:
            name = value.decode()
        elif number == 2:
            f = struct.unpack("<f", value)[0]
        elif number == 3:
            i = _signed64(value)
        elif number == 4:
            s = value.decode(errors="replace")
        elif number == 5:
            t = _tensor(value)[1]
        elif number == 7:
            floats += _floats(value, wire)
        elif number == 8:
            ints += _packed_varints(value, wire)
        elif number == 20:
            kind = value
    # AttributeType: FLOAT 1, INT 2, STRING 3, TENSOR 4, FLOATS 6, INTS 7.
    if kind == 7 or (kind is None and ints):
        return name, ints
    if kind == 6 or (kind is None and floats):
        return name, floats
    if kind == 1 or (kind is None and f is not None):
        return name, float(f if f is not None else 0.0)
    if kind == 2 or (kind is None and i is not None):
        return name, int(i if i is not None else 0)
    if kind == 3 or (kind is None and s is not None):
        return name, s or ""
    if kind == 4 or t is not None:
        return name, t
    return name, None


def _value_info(buf: bytes) -> tuple[str, list[int] | None, int]:
    name, shape, elem = "", None, FLOAT
    for number, _, value in _fields(buf):
        if number == 1:
            name = value.decode()
        elif number == 2:
            for tn, _, tv in _fields(value):
                if tn != 1:
                    continue
                for fn, _, fv in _fields(tv):
                    if fn == 1:
                        elem = fv
                    elif fn == 2:
                        shape = []
                        for dn, _, dv in _fields(fv):
                            if dn != 1:
                                continue
                            size = -1
                            for kn, _, kv in _fields(dv):
                                if kn == 1:
                                    size = _signed64(kv)
                            shape.append(size)
    return name, shape, elem


def _node(buf: bytes, index: int) -> dict[str, Any]:
    node: dict[str, Any] = {"inputs": [], "outputs": [], "attributes": {}, "name": "", "op_type": "", "domain": ""}
    for number, _, value in _fields(buf):
        if number == 1:
            node["inputs"].append(value.decode())
        elif number == 2:
            node["outputs"].append(value.decode())
        elif number == 3:
            node["name"] = value.decode()
        elif number == 4:
            node["op_type"] = value.decode()
        elif number == 5:
            key, attr = _attribute(value)
            node["attributes"][key] = attr
        elif number == 7:
            node["domain"] = value.decode()
    node["name"] = node["name"] or f"{node['op_type']}_{index}"
    return node


def load_onnx(path: str | Path) -> dict[str, Any]:
    """Reads an ONNX file into the IR dict of :func:`cutriton_b200.api.compile`:
    ``{"name", "inputs", "outputs", "input_shapes", "input_dtypes", "nodes",
    "constants"}``; graph inputs that are initializers are constants."""
    data = Path(path).read_bytes()
    graph = None
    for number, _, value in _fields(data):
        if number == 7:
            graph = value
    if graph is None:
        raise OnnxFormatError(f"{path}: no graph in the model")
    name = Path(path).stem
    nodes, constants, inputs, outputs = [], {}, [], []
    shapes: dict[str, list[int]] = {}
    dtypes: dict[str, str] = {}
    for number, _, value in _fields(graph):
        if number == 1:
            nodes.append(_node(value, len(nodes)))
        elif number == 2:
            name = value.decode() or name
        elif number == 5:
            tname, array = _tensor(value)
            constants[tname] = array
        elif number == 11:
            vname, shape, elem = _value_info(value)
            inputs.append(vname)
            if shape is not None:
                shapes[vname] = shape
            dtypes[vname] = "float16" if elem == FLOAT16 else "float32"
        elif number == 12:
            outputs.append(_value_info(value)[0])
    inputs = [n for n in inputs if n not in constants]
    return {"name": name, "inputs": inputs, "outputs": outputs, "input_shapes": shapes, "input_dtypes": dtypes,
            "nodes": nodes, "constants": constants}
