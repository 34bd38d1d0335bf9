"""Drop-in check with the reference's own C++ callers.

The reference's core test program (tests/cpp/test_core.cpp of the CUTriton
checkout) is compiled unchanged against this repository's include/ tree and
linked against libcutriton_b200.so, then run: it exercises Status/Tensor/
Buffer, Model constants, the fusion passes, the memory planner's alignment,
reuse and Flatten aliasing, the registries, shape profiles, the pack loader
and the engine with a mock CPU backend. Its own assertions are the
acceptance test of the C++17 surface.

The checkout is looked up in $CUTRITON_REFERENCE_CHECKOUT, else beside this
repository (../reference); without one the test is skipped. Nothing is copied
from it into the repository.

Also here: planner cases of this repository (reuse, overlapping lifetimes,
view chains, a dynamic shape) through the C ABI's engine build, so the planner is
pinned even where the reference checkout is absent.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import cutriton_b200 as ct
from cutriton_b200 import _build

REPO = Path(__file__).resolve().parents[1]


def reference_checkout() -> Path | None:
    env = os.environ.get("CUTRITON_REFERENCE_CHECKOUT")
    candidates = [Path(env)] if env else []
    candidates.append(REPO.parent / "reference")
    for path in candidates:
        if (path / "tests" / "cpp" / "test_core.cpp").exists():
            return path
    return None


def test_reference_core_test_program_passes(tmp_path):
    checkout = reference_checkout()
    if checkout is None:
        pytest.skip("no CUTriton checkout beside the repository")
    library = _build.build_library()
    exe = tmp_path / "reference_core_test"
    compile_cmd = ["g++", "-std=c++17", "-O1", f"-I{REPO / 'include'}", str(checkout / "tests" / "cpp" / "test_core.cpp"),
                   f"-L{library.parent}", f"-Wl,-rpath,{library.parent}", "-lcutriton_b200", "-lpthread", "-o", str(exe)]
    built = subprocess.run(compile_cmd, capture_output=True, text=True, timeout=600)
    assert built.returncode == 0, built.stderr[-4000:]
    # The program writes its scratch files under the working directory.
    ran = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600, cwd=tmp_path,
                         env={**os.environ, "CUTRITON_ASSUME_COMPUTE_CAPABILITY": ""})
    assert ran.returncode == 0, (ran.stdout[-2000:], ran.stderr[-2000:])


def relu_chain(sizes: list[int]) -> ct.Model:
    """input -> relu -> relu -> ... ; value i has sizes[i] floats."""
    m = ct.Model()
    m.add_input("v0", [sizes[0]], layout="")
    for i in range(1, len(sizes)):
        m.add_node(f"n{i}", "Relu", [f"v{i - 1}"], [f"v{i}"])
    m.add_output(f"v{len(sizes) - 1}")
    return m


@pytest.fixture()
def assume_sm100(monkeypatch):
    monkeypatch.setenv("CUTRITON_ASSUME_COMPUTE_CAPABILITY", "100")


def test_planner_reuses_ranges_of_finished_values(assume_sm100):
    # Intermediates v1..v4 of a chain: each is alive only while its reader
    # runs, so two slots of the largest size suffice.
    engine = ct.build_engine(relu_chain([1024, 1024, 1024, 1024, 1024, 1024]), tuning_mode=ct.TUNING_DISABLED)
    assert engine.workspace_bytes() == 2 * 4096


def test_planner_keeps_overlapping_lifetimes_apart(assume_sm100):
    # `small` is written first and read last, so it stays alive while `h0`
    # and `h1` come and go: at node c all three are alive, and no more ever.
    m = ct.Model()
    m.add_input("x", [64], layout="")
    m.add_node("a", "Relu", ["x"], ["small"])
    m.add_node("b", "Relu", ["x"], ["h0"])
    m.add_node("c", "Relu", ["h0"], ["h1"])
    m.add_node("d", "Add", ["h1", "x"], ["mix"])
    m.add_node("e", "Add", ["small", "x"], ["y"])
    m.add_output("y")
    m.add_output("mix")
    engine = ct.build_engine(m, tuning_mode=ct.TUNING_DISABLED)
    assert engine.workspace_bytes() == 3 * 256


def test_planner_rejects_unresolved_dynamic_shape(assume_sm100):
    m = ct.Model()
    m.add_input("x", [-1, 8], layout="")
    m.add_node("a", "Relu", ["x"], ["h"])
    m.add_node("b", "Relu", ["h"], ["y"])
    m.add_output("y")
    with pytest.raises(ct.CutritonError):
        ct.build_engine(m, tuning_mode=ct.TUNING_DISABLED)


def test_planner_view_of_view_shares_the_root_range(assume_sm100):
    m = ct.Model()
    m.add_input("x", [2, 8, 1, 1])
    m.add_node("r", "Relu", ["x"], ["h"])
    m.add_node("f1", "Flatten", ["h"], ["flat"])
    m.add_node("out", "Relu", ["flat"], ["y"])
    m.add_output("y")
    engine = ct.build_engine(m, tuning_mode=ct.TUNING_DISABLED)
    ops = engine.ops()
    assert [o["op_type"] for o in ops] == ["Relu", "Flatten", "Relu"]
    assert ops[1]["candidates"] == ["view:flatten"]
    assert engine.workspace_bytes() == 256
    np.testing.assert_equal(engine.value_desc("flat")[1], (2, 8))
