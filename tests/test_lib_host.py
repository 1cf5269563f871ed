"""Host logic of nebula_b200/lib.py without a GPU: buffers released while a thread
records a graph are freed only when that capture ends (a cudaFree inside a capture
invalidates it), whether it ends by qg_graph_end or by destroying the graph still
recording; other threads free at once. The library is replaced by a fake that
records the calls."""
import ctypes as C
import threading

import pytest

from nebula_b200 import lib


class FakeLib:
    """The qg_* entry points Device and the capture calls use."""

    def __init__(self, end_code=0):
        self.freed, self.destroyed, self.next_ptr, self.end_code = [], [], 0x1000, end_code

    def qg_alloc(self, n):
        self.next_ptr += 0x100
        return self.next_ptr

    def qg_free(self, p):
        self.freed.append(p)

    def qg_write(self, d, s, n):
        return 0

    def qg_graph_begin(self, ref):
        target = getattr(ref, "_obj", None)  # C.byref(g); C.pointer(g) has .contents
        if target is None:
            target = ref.contents
        target.value = 0xABC0
        return 0

    def qg_graph_end(self, g):
        return self.end_code

    def qg_graph_destroy(self, g):
        self.destroyed.append(g)

    def qg_error(self, code):
        return b"fake error"


@pytest.fixture
def fake(monkeypatch):
    f = FakeLib()
    monkeypatch.setattr(lib, "_LIB", f)
    yield f
    lib._capture.__dict__.clear()


def test_free_outside_a_capture_is_immediate(fake):
    d = lib.Device(nbytes=64)
    p = d.p
    d.free()
    assert fake.freed == [p] and d.p is None
    d.free()  # a second free does nothing
    assert fake.freed == [p]


def test_frees_wait_for_graph_end(fake):
    g = C.c_void_p()
    lib.call("graph_begin", C.byref(g))
    a, b = lib.Device(nbytes=8), lib.Device(nbytes=8)
    pa, pb = a.p, b.p
    a.free()
    del b  # finalized during the capture
    assert fake.freed == []
    lib.call("graph_end", g)
    assert sorted(fake.freed) == sorted([pa, pb])
    c = lib.Device(nbytes=8)
    pc = c.p
    c.free()
    assert fake.freed[-1] == pc  # immediate again


def test_failed_graph_end_still_frees_and_raises(monkeypatch):
    f = FakeLib(end_code=900)
    monkeypatch.setattr(lib, "_LIB", f)
    try:
        g = C.c_void_p()
        lib.call("graph_begin", C.pointer(g))
        d = lib.Device(nbytes=8)
        p = d.p
        d.free()
        with pytest.raises(lib.CudaError):
            lib.call("graph_end", g)
        assert f.freed == [p]
        assert lib._deferring() is None
    finally:
        lib._capture.__dict__.clear()


def test_destroying_the_recording_graph_ends_the_deferral(fake):
    g = C.c_void_p()
    lib.call("graph_begin", C.byref(g))
    d = lib.Device(nbytes=8)
    p = d.p
    d.free()
    lib.graph_destroy(C.c_void_p(0x1234))  # another graph: the capture goes on
    assert fake.freed == [] and lib._deferring() == [p]
    lib.graph_destroy(g)  # the one recording: abandoned, frees run
    assert fake.destroyed[-1] == 0xABC0 and fake.freed == [p] and lib._deferring() is None


def test_other_threads_free_at_once(fake):
    g = C.c_void_p()
    lib.call("graph_begin", C.byref(g))
    d = lib.Device(nbytes=8)
    p = d.p
    t = threading.Thread(target=d.free)
    t.start()
    t.join()
    assert fake.freed == [p]
    lib.call("graph_end", g)
    assert fake.freed == [p]
