"""Native build: the runtime shared library and the sm_100a Kernel Pack.

* ``libcutriton_b200.so`` — the C++17 runtime (IR, passes, pack loader,
  compiler, planner, launcher, engine) plus the C ABI of
  ``include/cutriton_b200.h``. It loads the CUDA driver lazily, so it links
  and loads on hosts without a GPU.
* ``pack/`` — one cubin per kernel source built with
  ``nvcc -gencode arch=compute_100a,code=sm_100a``, and ``pack.json`` (schema
  v2) emitted by :mod:`cutriton_b200.kernel_sdk` from the kernel specs.

Outputs stay inside the package directory (in-tree, git-ignored) so they
travel with a snapshot of the repository. Steps are skipped when outputs are
newer than their inputs.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = REPO / "include"
BUILD = PACKAGE / "_build"
LIB_DIR = PACKAGE / "lib"
LIBRARY = LIB_DIR / "libcutriton_b200.so"
PACK_DIR = PACKAGE / "pack"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = CUDA_HOME / "bin" / "nvcc"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

RUNTIME_SOURCES = [
    "cuda_driver.cpp",
    "capi.cpp",
    "core/status.cpp",
    "core/tensor.cpp",
    "core/buffer.cpp",
    "ir/graph.cpp",
    "ir/op_schema.cpp",
    "ir/fusion.cpp",
    "ir/pass.cpp",
    "backend/kernel_artifact.cpp",
    "backend/backend.cpp",
    "backend/cuda_launcher.cpp",
    "backend/prepack.cpp",
    "compiler/compiler.cpp",
    "runtime/memory_planner.cpp",
    "runtime/profiler.cpp",
    "runtime/device_session.cpp",
    "runtime/tuner.cpp",
    "runtime/engine.cpp",
]

CXXFLAGS = [
    "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-fvisibility=default",
    f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}",
]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(output: Path, inputs: list[Path]) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in inputs if p.exists())


def _headers() -> list[Path]:
    return sorted(INCLUDE.rglob("*.h")) + sorted(CSRC.rglob("*.h"))


def build_library(jobs: int = 8) -> Path:
    """Compiles the runtime sources and links ``libcutriton_b200.so``."""
    obj_dir = BUILD / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objects: list[Path] = []
    work: list[list[str]] = []
    for rel in RUNTIME_SOURCES:
        src = CSRC / rel
        obj = obj_dir / (rel.replace("/", "_") + ".o")
        objects.append(obj)
        if _stale(obj, [src, *headers]):
            work.append(["g++", *CXXFLAGS, "-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        for fut in [pool.submit(_run, cmd) for cmd in work]:
            fut.result()
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if work or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        _run(["g++", "-shared", "-o", str(tmp), *map(str, objects), "-ldl", "-lpthread",
              "-Wl,--no-undefined"])
        os.replace(tmp, LIBRARY)
    return LIBRARY


def compile_cubin(source: Path, output: Path, defines: dict[str, str] | None = None) -> Path:
    """``nvcc -cubin`` for sm_100a (with -lineinfo for profiler attribution)."""
    output.parent.mkdir(parents=True, exist_ok=True)
    deps = [source, *sorted((CSRC / "kernels").glob("*.cuh"))]
    flags = [f"-D{k}={v}" for k, v in sorted((defines or {}).items())]
    # The defines are part of the cubin's identity: a change rebuilds it.
    stamp = output.with_suffix(".flags")
    if _stale(output, deps) or not stamp.exists() or stamp.read_text() != " ".join(flags):
        tmp = output.with_suffix(".cubin.tmp")
        _run([str(NVCC), "-cubin", *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
              f"-I{CSRC / 'kernels'}", *flags, str(source), "-o", str(tmp)])
        os.replace(tmp, output)
        stamp.write_text(" ".join(flags))
    return output


def build_pack(jobs: int = 8) -> Path:
    """Builds every cubin named by the kernel specs and writes pack.json."""
    from . import kernel_sdk

    return kernel_sdk.build_pack(PACK_DIR, compile_cubin, jobs=jobs)


NOALLOC_SOURCE = CSRC / "noalloc" / "gemm_f16_noalloc.cu"
NOALLOC_LIBRARY = LIB_DIR / "libcutriton_b200_noalloc.so"


def build_noalloc_library() -> Path:
    """``libcutriton_b200_noalloc.so``: the no-allocation FP16 GEMM entry point
    (CUDA runtime, static cudart; the kernel comes from kernels/gemm_f16_tp.cu)."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    deps = [NOALLOC_SOURCE, CSRC / "kernels" / "gemm_f16_tp.cu", INCLUDE / "cutriton_b200_noalloc.h",
            *sorted((CSRC / "kernels").glob("*.cuh"))]
    if _stale(NOALLOC_LIBRARY, deps):
        tmp = NOALLOC_LIBRARY.with_suffix(".so.tmp")
        _run([str(NVCC), "-shared", "-Xcompiler", "-fPIC", *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
              "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC / 'kernels'}", str(NOALLOC_SOURCE), "-o", str(tmp)])
        os.replace(tmp, NOALLOC_LIBRARY)
    return NOALLOC_LIBRARY


def build_all(jobs: int | None = None) -> None:
    jobs = jobs or min(16, os.cpu_count() or 4)
    build_library(jobs)
    build_pack(jobs)
    build_noalloc_library()


if __name__ == "__main__":
    build_all()
    print(f"built {LIBRARY} and {PACK_DIR / 'pack.json'}", file=sys.stderr)
