"""ctb_gemm_f16_noalloc (include/cutriton_b200_noalloc.h): the persistent FP16
GEMM through a C entry point that allocates nothing, its scratch in a static
device array. Compared with the engine's Gemm / GemmGelu (the existing C-ABI
path) on two calls in a row; rejected shapes return an error without a launch.
Collected last on purpose: it must also pass after everything else ran.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest

import cutriton_b200 as ct
from tests.helpers import run_graph

LIB = Path(__file__).resolve().parents[1] / "cutriton_b200" / "lib" / "libcutriton_b200_noalloc.so"
INVALID_ARGUMENT = 1


def load():
    lib = ctypes.CDLL(str(LIB))
    fn = lib.ctb_gemm_f16_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_library_exports_entry_point():
    assert LIB.exists()
    assert hasattr(ctypes.CDLL(str(LIB)), "ctb_gemm_f16_noalloc")


def engine_gemm(a: np.ndarray, b: np.ndarray, op: str) -> np.ndarray:
    model = ct.Model()
    model.add_input("a", list(a.shape), dtype=np.float16, layout="")
    model.add_constant("b", b, layout="")
    model.add_node("proj", op, ["a", "b"], ["y"])
    model.add_output("y")
    out, _ = run_graph(model, {"a": a}, {"y": ((a.shape[0], b.shape[1]), np.float16)})
    return out["y"]


@pytest.mark.gpu
@pytest.mark.parametrize("mnk,op", [((1280, 2560, 64), "Gemm"), ((4096, 3072, 768), "GemmGelu"),
                                    ((33, 200, 72), "Gemm")])
def test_noalloc_matches_engine_twice(cuda, mnk, op):
    import torch

    m, n, k = mnk
    rng = np.random.default_rng(11)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = (rng.standard_normal((k, n)) * 0.02).astype(np.float16)
    expected = engine_gemm(a, b, op).astype(np.float32)

    fn = load()
    a_d = torch.from_numpy(a).cuda()
    bt_d = torch.from_numpy(np.ascontiguousarray(b.T)).cuda()
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        c_d = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        rc = fn(a_d.data_ptr(), bt_d.data_ptr(), c_d.data_ptr(), m, n, k, int(op == "GemmGelu"), stream, err, 256)
        assert rc == 0, err.value.decode()
        got = c_d.float().cpu().numpy()
        np.testing.assert_allclose(got, expected, atol=2e-2, rtol=2e-2, err_msg=f"{op} {mnk} call {call}")


@pytest.mark.gpu
def test_noalloc_rejects_unsupported_shape(cuda):
    import torch

    fn = load()
    a = torch.zeros(16, 12, dtype=torch.float16, device="cuda")
    bt = torch.zeros(16, 12, dtype=torch.float16, device="cuda")
    c = torch.zeros(16, 16, dtype=torch.float16, device="cuda")
    err = ctypes.create_string_buffer(256)
    rc = fn(a.data_ptr(), bt.data_ptr(), c.data_ptr(), 16, 16, 12, 0, None, err, 256)
    assert rc == INVALID_ARGUMENT
    assert b"multiples of 8" in err.value
