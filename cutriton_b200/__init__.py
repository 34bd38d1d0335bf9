"""Host-side mirror of the CUTriton C++ API over ``libcutriton_b200.so``.

Python callers build a :class:`Model` (graph + constants), compile it with
:func:`build_engine` into an :class:`Engine` and run it through an
:class:`ExecutionContext` — the same objects and call order as the C++ API
(reference include/cutriton/{ir/graph.h, compiler/compiler.h,
runtime/engine.h}). Every call goes through the C ABI of
``include/cutriton_b200.h``; errors raise :class:`CutritonError` carrying the
C++ ``ErrorCode``. There is no compute in Python and no fallback: without the
built library or a GPU the calls fail.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "lib" / "libcutriton_b200.so"
PACK_DIR = PACKAGE_DIR / "pack"

OK, INVALID_ARGUMENT, NOT_FOUND, ALREADY_EXISTS, UNSUPPORTED, SHAPE_ERROR, RUNTIME_ERROR, INTERNAL = range(8)
ERROR_NAMES = ["OK", "InvalidArgument", "NotFound", "AlreadyExists", "Unsupported", "ShapeError",
               "RuntimeError", "Internal"]
FLOAT32, FLOAT16, INT32, INT64 = 1, 2, 3, 4
TUNING_DISABLED, TUNING_USE_CACHE, TUNING_TUNE_ON_MISS, TUNING_FORCE_RETUNE = range(4)
MAX_RANK = 8

_NUMPY_DTYPES = {FLOAT32: np.float32, FLOAT16: np.float16, INT32: np.int32, INT64: np.int64}
_DTYPE_OF_NUMPY = {np.dtype(v): k for k, v in _NUMPY_DTYPES.items()}


class CutritonError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES[code] if 0 <= code < len(ERROR_NAMES) else code}: {message}")
        self.code = code


class CompileOptions(ctypes.Structure):
    """Layout of ``ctb_compile_options``."""

    _fields_ = [
        ("target", ctypes.c_char_p),
        ("device_id", ctypes.c_int),
        ("enable_cuda_graph", ctypes.c_int),
        ("enable_profiling", ctypes.c_int),
        ("enable_transformer_fusions", ctypes.c_int),
        ("enable_residual_fusion", ctypes.c_int),
        ("kernel_artifact_dir", ctypes.c_char_p),
        ("tuning_cache_dir", ctypes.c_char_p),
        ("tuning_mode", ctypes.c_int),
        ("tuning_warmup_iterations", ctypes.c_int),
        ("tuning_measurement_iterations", ctypes.c_int),
        ("cuda_graph_cache_capacity", ctypes.c_size_t),
    ]


_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)
_CHARPP = ctypes.POINTER(ctypes.c_char_p)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ctb_last_error": (ctypes.c_char_p, []),
    "ctb_abi_version": (ctypes.c_int, []),
    "ctb_model_create": (ctypes.c_int, [ctypes.POINTER(_P)]),
    "ctb_model_destroy": (None, [_P]),
    "ctb_graph_add_input": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _I64P, ctypes.c_char_p]),
    "ctb_graph_add_output": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "ctb_graph_add_node": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _CHARPP, ctypes.c_int, _CHARPP]),
    "ctb_node_set_attr_int": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int64]),
    "ctb_node_set_attr_float": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_double]),
    "ctb_node_set_attr_ints": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _I64P]),
    "ctb_model_add_constant": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _I64P, ctypes.c_char_p, _P, ctypes.c_size_t]),
    "ctb_compile_options_init": (None, [ctypes.POINTER(CompileOptions)]),
    "ctb_model_add_shape_profile": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _I64P, _I64P, _I64P]),
    "ctb_engine_build": (ctypes.c_int, [_P, ctypes.POINTER(CompileOptions), ctypes.POINTER(_P)]),
    "ctb_engine_destroy": (None, [_P]),
    "ctb_engine_num_ops": (ctypes.c_int, [_P]),
    "ctb_engine_op_info": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "ctb_engine_candidate_id": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]),
    "ctb_engine_value_desc": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), _I64P]),
    "ctb_engine_workspace_bytes": (ctypes.c_size_t, [_P]),
    "ctb_context_create": (ctypes.c_int, [_P, ctypes.POINTER(_P)]),
    "ctb_context_destroy": (None, [_P]),
    "ctb_context_bind_input": (ctypes.c_int, [_P, ctypes.c_char_p, _P, ctypes.c_size_t]),
    "ctb_context_bind_output": (ctypes.c_int, [_P, ctypes.c_char_p, _P, ctypes.c_size_t]),
    "ctb_context_select_profile": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "ctb_context_set_input_shape": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_int, _I64P]),
    "ctb_context_resolve_shapes": (ctypes.c_int, [_P]),
    "ctb_context_resolved_desc": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), _I64P]),
    "ctb_context_run": (ctypes.c_int, [_P]),
    "ctb_context_run_async": (ctypes.c_int, [_P, _P]),
    "ctb_context_synchronize": (ctypes.c_int, [_P]),
    "ctb_context_profile_event_count": (ctypes.c_int, [_P]),
    "ctb_context_profile_event": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_double)]),
    "ctb_context_cached_graph_count": (ctypes.c_size_t, [_P]),
    "ctb_context_loaded_module_count": (ctypes.c_size_t, [_P]),
    "ctb_context_selected_candidate": (ctypes.c_int, [_P, ctypes.c_int]),
    "ctb_context_select_candidate": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int]),
    "ctb_context_run_host": (ctypes.c_int, [_P, ctypes.c_int, _CHARPP, ctypes.POINTER(_P), ctypes.c_int, _CHARPP, ctypes.POINTER(_P), _P]),
    "ctb_context_run_host_async": (ctypes.c_int, [_P, ctypes.c_int, _CHARPP, ctypes.POINTER(_P), ctypes.c_int, _CHARPP, ctypes.POINTER(_P), _P]),
}

_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Loads ``libcutriton_b200.so`` (in-tree build) once; raises if missing."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("CUTRITON_B200_LIBRARY", LIBRARY_PATH))
        if not path.exists():
            raise CutritonError(NOT_FOUND, f"{path} is not built; run __graft_entry__.build()")
        lib = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def _check(code: int) -> None:
    if code != OK:
        raise CutritonError(code, library().ctb_last_error().decode(errors="replace"))


def _i64(values: Sequence[int]):
    arr = (ctypes.c_int64 * max(1, len(values)))(*values)
    return arr


def _strings(values: Sequence[str]):
    return (ctypes.c_char_p * max(1, len(values)))(*[v.encode() for v in values])


def dtype_code(dtype) -> int:
    return _DTYPE_OF_NUMPY[np.dtype(dtype)]


class Model:
    """cutriton::Model: a Graph plus host-resident constants."""

    def __init__(self) -> None:
        handle = _P()
        _check(library().ctb_model_create(ctypes.byref(handle)))
        self._h = handle

    def __del__(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            try:
                _lib.ctb_model_destroy(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def add_input(self, name: str, shape: Sequence[int], dtype=np.float32, layout: str = "NCHW") -> None:
        _check(library().ctb_graph_add_input(self._h, name.encode(), dtype_code(dtype), len(shape), _i64(shape),
                                             layout.encode()))

    def add_output(self, name: str) -> None:
        _check(library().ctb_graph_add_output(self._h, name.encode()))

    def add_node(self, name: str, op_type: str, inputs: Sequence[str], outputs: Sequence[str], **attrs) -> None:
        _check(library().ctb_graph_add_node(self._h, name.encode(), op_type.encode(), len(inputs), _strings(inputs),
                                            len(outputs), _strings(outputs)))
        for key, value in attrs.items():
            self.set_attr(name, key, value)

    def set_attr(self, node: str, key: str, value) -> None:
        lib = library()
        if isinstance(value, bool) or isinstance(value, (int, np.integer)):
            _check(lib.ctb_node_set_attr_int(self._h, node.encode(), key.encode(), int(value)))
        elif isinstance(value, (float, np.floating)):
            _check(lib.ctb_node_set_attr_float(self._h, node.encode(), key.encode(), float(value)))
        else:
            values = [int(v) for v in value]
            _check(lib.ctb_node_set_attr_ints(self._h, node.encode(), key.encode(), len(values), _i64(values)))

    def add_constant(self, name: str, array: np.ndarray, layout: str = "NCHW") -> None:
        data = np.ascontiguousarray(array)
        _check(library().ctb_model_add_constant(self._h, name.encode(), dtype_code(data.dtype), data.ndim,
                                                _i64(data.shape), layout.encode(), data.ctypes.data_as(_P),
                                                data.nbytes))

    def add_shape_profile(self, profile: str, input_name: str, min_shape: Sequence[int], opt_shape: Sequence[int],
                          max_shape: Sequence[int]) -> None:
        _check(library().ctb_model_add_shape_profile(self._h, profile.encode(), input_name.encode(), len(min_shape),
                                                     _i64(min_shape), _i64(opt_shape), _i64(max_shape)))


def compile_options(**overrides) -> CompileOptions:
    options = CompileOptions()
    library().ctb_compile_options_init(ctypes.byref(options))
    options.kernel_artifact_dir = str(PACK_DIR).encode()
    for key, value in overrides.items():
        if isinstance(value, str):
            value = value.encode()
        elif isinstance(value, bool):
            value = int(value)
        setattr(options, key, value)
    return options


class Engine:
    """cutriton::Engine (compiled plan + shared constants)."""

    def __init__(self, handle: ctypes.c_void_p) -> None:
        self._h = handle

    def __del__(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            try:
                _lib.ctb_engine_destroy(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def num_ops(self) -> int:
        return library().ctb_engine_num_ops(self._h)

    def op(self, index: int) -> dict:
        op_type = ctypes.create_string_buffer(128)
        node = ctypes.create_string_buffer(256)
        count = ctypes.c_int()
        default = ctypes.c_int()
        _check(library().ctb_engine_op_info(self._h, index, op_type, 128, node, 256, ctypes.byref(count),
                                            ctypes.byref(default)))
        ids = []
        for c in range(count.value):
            buf = ctypes.create_string_buffer(512)
            _check(library().ctb_engine_candidate_id(self._h, index, c, buf, 512))
            ids.append(buf.value.decode())
        return {"op_type": op_type.value.decode(), "node": node.value.decode(), "candidates": ids,
                "default": default.value}

    def ops(self) -> list[dict]:
        return [self.op(i) for i in range(self.num_ops())]

    def value_desc(self, name: str) -> tuple[int, tuple[int, ...]]:
        dtype = ctypes.c_int()
        rank = ctypes.c_int()
        shape = (ctypes.c_int64 * MAX_RANK)()
        _check(library().ctb_engine_value_desc(self._h, name.encode(), ctypes.byref(dtype), ctypes.byref(rank), shape))
        return dtype.value, tuple(shape[i] for i in range(rank.value))

    def workspace_bytes(self) -> int:
        return int(library().ctb_engine_workspace_bytes(self._h))

    def create_context(self) -> "ExecutionContext":
        handle = _P()
        _check(library().ctb_context_create(self._h, ctypes.byref(handle)))
        return ExecutionContext(handle, self)


def build_engine(model: Model, **options) -> Engine:
    opts = compile_options(**options)
    handle = _P()
    _check(library().ctb_engine_build(model._h, ctypes.byref(opts), ctypes.byref(handle)))
    return Engine(handle)


class ExecutionContext:
    """cutriton::ExecutionContext. Device buffers are bound by address."""

    def __init__(self, handle: ctypes.c_void_p, engine: Engine) -> None:
        self._h = handle
        self._engine = engine  # keeps plan inspection alive; the C++ context does not need it
        # Tensors bound through bind_tensor, by name: the context holds only
        # their addresses, so it keeps them alive until rebound or destroyed
        # (a freed tensor's memory would be handed to the next allocation).
        self._bound: dict[str, object] = {}

    def __del__(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            try:
                _lib.ctb_context_destroy(self._h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def bind_input(self, name: str, device_ptr: int, nbytes: int) -> None:
        """Binds device memory by address; the caller keeps it alive."""
        _check(library().ctb_context_bind_input(self._h, name.encode(), _P(device_ptr), nbytes))
        self._bound.pop(name, None)

    def bind_output(self, name: str, device_ptr: int, nbytes: int) -> None:
        """Binds device memory by address; the caller keeps it alive."""
        _check(library().ctb_context_bind_output(self._h, name.encode(), _P(device_ptr), nbytes))
        self._bound.pop(name, None)

    def bind_tensor(self, name: str, tensor, output: bool = False) -> None:
        """Binds a CUDA torch tensor (contiguous) by its data pointer and keeps
        a reference to it for as long as it is bound."""
        nbytes = tensor.numel() * tensor.element_size()
        (self.bind_output if output else self.bind_input)(name, tensor.data_ptr(), nbytes)
        self._bound[name] = tensor

    def select_profile(self, name: str) -> None:
        _check(library().ctb_context_select_profile(self._h, name.encode()))

    def set_input_shape(self, name: str, shape: Sequence[int]) -> None:
        _check(library().ctb_context_set_input_shape(self._h, name.encode(), len(shape), _i64(shape)))

    def resolve_shapes(self) -> None:
        _check(library().ctb_context_resolve_shapes(self._h))

    def resolved_desc(self, name: str) -> tuple[int, tuple[int, ...]]:
        dtype = ctypes.c_int()
        rank = ctypes.c_int()
        shape = (ctypes.c_int64 * MAX_RANK)()
        _check(library().ctb_context_resolved_desc(self._h, name.encode(), ctypes.byref(dtype), ctypes.byref(rank),
                                                   shape))
        return dtype.value, tuple(shape[i] for i in range(rank.value))

    def run(self) -> None:
        _check(library().ctb_context_run(self._h))

    def run_async(self, stream: int | None = None) -> None:
        _check(library().ctb_context_run_async(self._h, _P(stream or 0)))

    def synchronize(self) -> None:
        _check(library().ctb_context_synchronize(self._h))

    def profile_events(self) -> list[tuple[str, float]]:
        lib = library()
        out = []
        for i in range(lib.ctb_context_profile_event_count(self._h)):
            name = ctypes.create_string_buffer(256)
            ms = ctypes.c_double()
            _check(lib.ctb_context_profile_event(self._h, i, name, 256, ctypes.byref(ms)))
            out.append((name.value.decode(), ms.value))
        return out

    def cached_graph_count(self) -> int:
        return int(library().ctb_context_cached_graph_count(self._h))

    def loaded_module_count(self) -> int:
        return int(library().ctb_context_loaded_module_count(self._h))

    def selected_candidate(self, op: int) -> int:
        return library().ctb_context_selected_candidate(self._h, op)

    def select_candidate(self, op: int, candidate: int) -> None:
        _check(library().ctb_context_select_candidate(self._h, op, candidate))

    def run_host(self, inputs: dict[str, np.ndarray], outputs: dict[str, np.ndarray], stream: int | None = None) -> None:
        """Host -> device copies, run, device -> host copies in one call."""
        self._run_host(library().ctb_context_run_host, inputs, outputs, stream or 0)

    def run_host_async(self, inputs: dict[str, np.ndarray], outputs: dict[str, np.ndarray], stream: int) -> None:
        """The same copies and run enqueued on `stream`; returns without waiting.

        The arrays must stay alive (and pinned, for the copies to overlap) until
        synchronize().
        """
        if not stream:
            raise ValueError("run_host_async needs a stream")
        self._run_host(library().ctb_context_run_host_async, inputs, outputs, stream)

    def _run_host(self, fn, inputs: dict[str, np.ndarray], outputs: dict[str, np.ndarray], stream: int) -> None:
        for name, arr in list(inputs.items()) + list(outputs.items()):
            if not arr.flags["C_CONTIGUOUS"]:
                raise ValueError(f"host buffer {name!r} must be C-contiguous")
        in_names = list(inputs)
        out_names = list(outputs)
        in_ptrs = (_P * max(1, len(in_names)))(*[inputs[n].ctypes.data for n in in_names])
        out_ptrs = (_P * max(1, len(out_names)))(*[outputs[n].ctypes.data for n in out_names])
        _check(fn(self._h, len(in_names), _strings(in_names), in_ptrs, len(out_names), _strings(out_names), out_ptrs,
                  _P(stream)))


def exported_symbols() -> Iterable[str]:
    return SIGNATURES.keys()
