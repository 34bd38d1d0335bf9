"""ExecutionContext.bind_tensor keeps the bound tensor alive (CPU only).

The C++ context stores only the address of a bound buffer. If the Python
object owning that buffer were freed while bound, torch's caching allocator
would hand the same memory to the next tensor of that size: two bindings of
one context (or of two contexts) would then share memory and results would
depend on timing. The wrapper therefore holds each bound tensor until the name
is rebound or the context goes away. The C calls are replaced by a recorder.
"""

from __future__ import annotations

import gc
import weakref

import cutriton_b200 as ct


class FakeTensor:
    def __init__(self, ptr: int, numel: int = 16, element_size: int = 4):
        self._ptr, self._numel, self._size = ptr, numel, element_size

    def data_ptr(self) -> int:
        return self._ptr

    def numel(self) -> int:
        return self._numel

    def element_size(self) -> int:
        return self._size


def make_context(calls):
    ctx = ct.ExecutionContext.__new__(ct.ExecutionContext)
    ctx._h = None
    ctx._engine = None
    ctx._bound = {}

    def record(kind):
        def bind(name, ptr, nbytes):
            calls.append((kind, name, ptr, nbytes))
            ctx._bound.pop(name, None)
        return bind

    ctx.bind_input = record("in")
    ctx.bind_output = record("out")
    return ctx


def test_bound_tensor_lives_while_bound_and_is_released_on_rebind():
    calls = []
    ctx = make_context(calls)
    ctx.bind_tensor("x", FakeTensor(0x1000))
    ctx.bind_tensor("y", FakeTensor(0x2000, numel=8, element_size=2), output=True)
    assert calls == [("in", "x", 0x1000, 64), ("out", "y", 0x2000, 16)]
    held = weakref.ref(ctx._bound["x"])
    gc.collect()
    assert held() is not None  # no other reference exists: the context keeps it
    ctx.bind_tensor("x", FakeTensor(0x3000))
    gc.collect()
    assert held() is None  # rebinding the name releases the old tensor
    assert ctx._bound["x"].data_ptr() == 0x3000
