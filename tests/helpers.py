"""Shared helpers: single-node graphs run through the engine (C ABI) with
torch CUDA tensors, and tolerance checks."""

from __future__ import annotations

import numpy as np

import cutriton_b200 as ct


def run_graph(model: ct.Model, inputs: dict[str, np.ndarray], outputs: dict[str, tuple[tuple[int, ...], np.dtype]],
              candidate: tuple[int, int] | None = None, **options) -> tuple[dict[str, np.ndarray], ct.Engine]:
    """Compiles `model`, binds CUDA copies of `inputs`, runs once and returns
    host copies of `outputs`. `candidate` = (op, index) pins a candidate."""
    import torch

    options.setdefault("enable_cuda_graph", False)
    options.setdefault("tuning_mode", ct.TUNING_DISABLED)
    engine = ct.build_engine(model, **options)
    context = engine.create_context()
    device = torch.device("cuda:0")
    keep = []
    for name, array in inputs.items():
        t = torch.from_numpy(np.ascontiguousarray(array)).to(device)
        keep.append(t)
        context.bind_tensor(name, t)
    out_tensors = {}
    for name, (shape, dtype) in outputs.items():
        t = torch.full(shape, float("nan"), dtype=getattr(torch, np.dtype(dtype).name), device=device)
        out_tensors[name] = t
        context.bind_tensor(name, t, output=True)
    if candidate is not None:
        context.select_candidate(*candidate)
    context.run()
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out_tensors.items()}, engine


def assert_close(actual: np.ndarray, expected: np.ndarray, atol: float, rtol: float, what: str = "") -> None:
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    assert np.all(np.isfinite(actual)), f"{what}: non-finite values"
    err = np.abs(actual - expected)
    tol = atol + rtol * np.abs(expected)
    bad = err > tol
    if bad.any():
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} outside tolerance; worst at {i}: "
                             f"{actual[i]} vs {expected[i]} (max abs err {err.max():.3e})")


def assert_bitexact(actual: np.ndarray, expected: np.ndarray, what: str = "") -> None:
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    a = np.ascontiguousarray(actual)
    e = np.ascontiguousarray(expected)
    diff = a.view(np.uint8) != e.view(np.uint8)
    assert not diff.any(), f"{what}: {int(diff.sum())} differing bytes"
