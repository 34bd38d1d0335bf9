"""ctb_gemm_f16_noalloc (include/cutriton_b200_noalloc.h): the persistent FP16
GEMM through a C entry point that allocates nothing, for callers that cannot
allocate device memory on their call path. Its scratch lives in a static
device array of the library.

Each case calls the entry point twice in a row through the C ABI and
compares both results with the C oracle (oracle/ops.c: FP32 accumulation,
erf-GELU on the accumulator, RNE FP16 store) within the FP16 bar of the other
GEMM tests (2e-2 abs + 2e-2 rel), and with the engine's own Gemm/GemmGelu
(the existing C-ABI path). All buffers exist before the second call; the
device's free memory must be the same after it. Rejected shapes and a stream
of the wrong device return an error without a launch.

Collected last on purpose: it must pass after everything else ran as well as
alone in a fresh process.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest

import cutriton_b200 as ct
from oracle import ops as oracle
from tests.helpers import assert_close, run_graph

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
def test_noalloc_matches_oracle_twice(cuda, mnk, op):
    import torch

    m, n, k = mnk
    rng = np.random.default_rng(11)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = (rng.standard_normal((k, n)) * 0.02).astype(np.float16)
    # Oracle on a row sample (rows are independent): first and last 64 rows
    # and 64 seeded rows in between.
    rows = np.unique(np.concatenate([np.arange(min(64, m)), np.arange(max(0, m - 64), m),
                                     rng.integers(0, m, 64)]))
    expected = oracle.gemm_f16(np.ascontiguousarray(a[rows]), b, gelu=(op == "GemmGelu")).astype(np.float32)
    engine_out = engine_gemm(a, b, op).astype(np.float32)

    fn = load()
    a_d = torch.from_numpy(a).cuda()
    bt_d = torch.from_numpy(np.ascontiguousarray(b.T)).cuda()
    outs = [torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda") for _ in range(2)]
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    free_after = []
    for call in range(2):
        rc = fn(a_d.data_ptr(), bt_d.data_ptr(), outs[call].data_ptr(), m, n, k, int(op == "GemmGelu"), stream,
                err, 256)
        assert rc == 0, err.value.decode()
        torch.cuda.synchronize()
        free_after.append(torch.cuda.mem_get_info()[0])
    # The first call may load the library's module on this device; the
    # second must not allocate anything.
    assert free_after[1] == free_after[0], f"free memory changed by {free_after[0] - free_after[1]} bytes"
    for call in range(2):
        got = outs[call].float().cpu().numpy()
        assert_close(got[rows], expected, atol=2e-2, rtol=2e-2, what=f"{op} {mnk} call {call} vs oracle")
        assert_close(got, engine_out, atol=2e-2, rtol=2e-2, what=f"{op} {mnk} call {call} vs engine")


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


@pytest.mark.gpu
def test_noalloc_rejects_stream_of_other_device(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible devices")
    fn = load()
    a = torch.zeros(16, 16, dtype=torch.float16, device="cuda:0")
    c = torch.zeros(16, 16, dtype=torch.float16, device="cuda:0")
    other = torch.cuda.Stream(device=1)
    err = ctypes.create_string_buffer(256)
    torch.cuda.set_device(0)
    rc = fn(a.data_ptr(), a.data_ptr(), c.data_ptr(), 16, 16, 16, 0, other.cuda_stream, err, 256)
    assert rc == INVALID_ARGUMENT
    assert b"stream belongs to device 1" in err.value
