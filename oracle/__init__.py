"""CPU oracle for parity checks — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only
as the checker or the timed CPU baseline; the product path never calls it.

* :mod:`oracle.ops` — ctypes bindings of ``ops.c``, the plain-C restatement
  of the reference kernels (python/cutriton/triton_kernels/*.py).
* :mod:`oracle.torch_ref` — PyTorch-eager CPU restatement of the reference's
  comparison models (benchmarks/resnet50_compare.py:18-141,
  transformer_ffn_compare.py:52-60), used for whole-network checks and as
  the CPU baseline.

Parity is pinned: tests/test_oracle_golden.py checks these against the golden
vectors of tests/golden/ (made by tests/golden/make_golden.py from the
reference's own PyTorch model and the known-answer formulas of its
tests/cpp/test_cuda.cpp).
"""
