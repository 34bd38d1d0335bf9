"""Failure detection on the GPU without a fault: a kernel wait that can never
be satisfied gives up after a short limit, records the error in the engine's
device-mapped error block and returns; the host reports it at Synchronize and
the context (and the device) stay usable.

The probe op ("BoundedWaitProbe", kernels/diag.cu) waits on an mbarrier that
nothing arrives on, through the same bounded-wait routine the tensor-core
pipeline kernels use for their TMA / MMA / epilogue handshakes.
"""

import numpy as np
import pytest

import cutriton_b200 as ct
from tests.helpers import run_graph

RNG = np.random.default_rng(7)


def probe_model(n: int, limit_us: int) -> ct.Model:
    model = ct.Model()
    model.add_input("x", [n])
    model.add_node("probe", "BoundedWaitProbe", ["x"], ["y"], limit_us=limit_us)
    model.add_output("y")
    return model


@pytest.mark.gpu
def test_expired_wait_is_reported_and_context_stays_usable(cuda):
    import torch

    n = 4096
    engine = ct.build_engine(probe_model(n, limit_us=20000), enable_cuda_graph=False)
    ctx = engine.create_context()
    x = torch.from_numpy(RNG.standard_normal(n).astype(np.float32)).cuda()
    y = torch.zeros(n, device="cuda")
    ctx.bind_tensor("x", x)
    ctx.bind_tensor("y", y, output=True)
    for _ in range(2):  # the error block is cleared after each report
        with pytest.raises(ct.CutritonError, match=r"abandoned a bounded wait \(code 1, site 90"):
            ctx.run()
        # The kernel itself completed: the copy after the abandoned wait is there.
        assert torch.equal(y, x)
        y.zero_()

    # The device and the runtime still work: an ordinary graph runs correctly.
    relu = ct.Model()
    relu.add_input("a", [2, 8, 4, 4])
    relu.add_node("r", "Relu", ["a"], ["b"])
    relu.add_output("b")
    a = RNG.standard_normal((2, 8, 4, 4)).astype(np.float32)
    out, _ = run_graph(relu, {"a": a}, {"b": ((2, 8, 4, 4), np.float32)})
    np.testing.assert_array_equal(out["b"], np.maximum(a, 0.0))
