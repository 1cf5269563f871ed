"""ctypes binding of ``libqwen_gpu.so`` - the same shape as the reference's
own binding (qwen/test_gpu.py:12-61: a SIGNATURES table over ``qg_*``, a
``call`` that raises on a non-zero cudaError_t, and a ``Device`` buffer).

The library is the product; there is no fallback. ``load()`` raises when the
built library is missing instead of substituting anything else.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libqwen_gpu.so"

P, I, F, Z, D = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_double
U64 = C.c_uint64

# name (without qg_ prefix) -> (argtypes, restype); one line per declaration in include/gpu.h
SIGNATURES = {
    "alloc": ([Z], P), "free": ([P], None), "write": ([P, P, Z], I), "read": ([P, P, Z], I),
    "copy": ([P, P, Z], I), "zero": ([P, Z], I), "sync": ([], I),
    "graph_begin": ([C.POINTER(P)], I), "graph_end": ([P], I), "graph_launch": ([P], I), "graph_destroy": ([P], None),
    "memory": ([C.POINTER(Z), C.POINTER(Z)], I), "error": ([I], C.c_char_p),
    "tensor_bytes": ([I, C.POINTER(U64), C.POINTER(U64)], I),
    "upload_create": ([Z], P), "upload_destroy": ([P], None),
    "upload_expert": ([P, P, P, Z, P, Z, P, Z], I), "upload_seconds": ([P], D),
    "matmul": ([P, P, I, I, I, P, I], I), "gather": ([P, P, I, I, I], I),
    "unary": ([P, P, I, I, F], I), "binary": ([P, P, P, I, I], I),
    "dequant": ([P, P, I, I, I], I), "shared_add": ([P, P, P, I], I),
    "route": ([P, P, P, I], I), "prune_routes": ([P, P, P, I, D, P], I),
    "moe_map": ([P, P, I], I), "moe_gather": ([P, P, P, I], I),
    "moe_scatter": ([P, P, P, P, P, I, I], I), "moe_reduce": ([P, P, I], I),
    "mtp_moe": ([P, P, P, P, P, P, I, P, I, P, I, I], I),
    "moe_workspace_bytes": ([I, I, I, C.POINTER(Z)], I),
    "moe_routed": ([P, P, P, P, I, P, I, P, I, P, I, I, I, P], I),
    "moe_routed_static": ([P, P, P, P, I, P, I, P, I, P, I, I, I], I),
    "moe_layer": ([P, P, P, P, I, P, P, P, I, P, I, P, I, P, I, P, I, P, I, P, I, I, P], I),
    "ep_workspace_bytes": ([I, I, I, C.POINTER(Z)], I), "ep_ipc_handle": ([P, P], I),
    "ep_ipc_open": ([P, C.POINTER(P)], I), "ep_ipc_close": ([P], I),
    "moe_layer_ep": ([P, P, P, P, I, P, P, P, I, P, I, P, I, I, P, P, I, P, I, P, I, P, I, I, I, I, I, P], I),
    "moe_status": ([P, C.POINTER(I), C.POINTER(I), C.POINTER(I)], I),
    "moe_profile": ([I], I), "moe_profile_read": ([I, C.POINTER(D), C.POINTER(I)], I),
    "synth_weights": ([P, I, I, I, U64, F], I), "synth_normal": ([P, Z, U64, F], I),
    "index_open": ([C.c_char_p, C.POINTER(P), C.c_char_p, Z], I), "index_close": ([P], None),
    "index_tensor": ([P, C.c_char_p, C.POINTER(P), C.POINTER(I), C.POINTER(U64), C.POINTER(U64)], I),
    "upload_experts": ([P, P, P, Z, P, I], I),
    "route_trace_open": ([C.c_char_p, C.POINTER(P)], I),
    "route_trace_next": ([P, C.POINTER(I), C.POINTER(I), C.POINTER(I), P, P, I], I),
    "route_trace_close": ([P], None),
}

_LIB = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load the built library (once) and bind every signature."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is not built; run nebula_b200/build.py (or __graft_entry__.build())")
    lib = C.CDLL(str(p))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, "qg_" + name)
        fn.argtypes, fn.restype = args, res
    if path is None:
        _LIB = lib
    return lib


class CudaError(RuntimeError):
    def __init__(self, name: str, code: int, text: str):
        super().__init__(f"qg_{name}: {text} (cudaError {code})")
        self.code = code


# Buffers released while this thread records a graph (qg_graph_begin .. qg_graph_end, or
# qg_graph_destroy of the graph still recording, which abandons the capture): a cudaFree
# then would invalidate the capture, and Python may finalize a buffer at any point
# (reference cycles are collected whenever the interpreter allocates), so their frees wait
# until the capture ends.
_capture = threading.local()


def _deferring() -> list | None:
    return getattr(_capture, "pending", None)


def _handle_written(arg):
    """The graph handle qg_graph_begin wrote through C.byref(g) or C.pointer(g)."""
    obj = getattr(arg, "_obj", None)
    if obj is None:
        obj = getattr(arg, "contents", None)
    return getattr(obj, "value", None)


def _end_capture(lib) -> None:
    pending, _capture.pending, _capture.graph = _deferring() or [], None, None
    for p in pending:
        lib.qg_free(p)


def call(name: str, *args) -> None:
    """Call ``qg_<name>`` and raise on a non-zero cudaError_t."""
    lib = load()
    code = getattr(lib, "qg_" + name)(*args)
    if name == "graph_begin" and not code:
        _capture.pending = []
        _capture.graph = _handle_written(args[0])
    elif name == "graph_end":
        _end_capture(lib)
    if code:
        raise CudaError(name, code, lib.qg_error(code).decode())


def graph_destroy(graph) -> None:
    """qg_graph_destroy (a ``c_void_p`` or an int handle). Destroying the graph this
    thread is still recording ends that capture, and the frees it deferred run."""
    lib = load()
    h = graph.value if isinstance(graph, C.c_void_p) else graph
    lib.qg_graph_destroy(h)
    if _deferring() is not None and h is not None and getattr(_capture, "graph", None) == h:
        _end_capture(lib)


def code(name: str, *args) -> int:
    """Call ``qg_<name>`` and return its cudaError_t."""
    return getattr(load(), "qg_" + name)(*args)


class Device:
    """A device buffer (qwen/test_gpu.py:45-61): from a numpy array (copied in),
    or empty with a numpy shape/dtype (``like``) or a raw byte count. No host
    mirror is kept; ``get`` reads the device copy back."""

    def __init__(self, x=None, nbytes: int | None = None, like: np.ndarray | None = None):
        lib = load()
        if x is not None:
            x = np.ascontiguousarray(x)
            self.shape, self.dtype = x.shape, x.dtype
        elif like is not None:
            self.shape, self.dtype = like.shape, like.dtype
        else:
            self.shape, self.dtype = (int(nbytes),), np.dtype(np.uint8)
        self.nbytes = int(np.prod(self.shape)) * np.dtype(self.dtype).itemsize
        self.p = lib.qg_alloc(max(self.nbytes, 1))
        if not self.p:
            raise MemoryError(f"qg_alloc({self.nbytes})")
        if x is not None:
            call("write", self.p, x.ctypes.data, self.nbytes)

    @classmethod
    def empty(cls, shape, dtype) -> "Device":
        return cls(like=np.empty(shape, dtype))

    def get(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        call("read", out.ctypes.data, self.p, out.nbytes)
        return out

    def set(self, x: np.ndarray) -> None:
        x = np.ascontiguousarray(x, dtype=self.dtype)
        assert x.nbytes == self.nbytes
        call("write", self.p, x.ctypes.data, x.nbytes)

    def free(self) -> None:
        if getattr(self, "p", None):
            pending = _deferring()
            if pending is not None:  # this thread is recording a graph
                pending.append(self.p)
            else:
                load().qg_free(self.p)
            self.p = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def workspace_bytes(tokens: int, hidden: int, ffn: int) -> int:
    n = Z(0)
    call("moe_workspace_bytes", tokens, hidden, ffn, C.byref(n))
    return n.value


def workspace(tokens: int, hidden: int, ffn: int) -> Device:
    """A zero-filled MoE workspace (qg_moe_routed / qg_moe_layer need zeros once)."""
    ws = Device(nbytes=workspace_bytes(tokens, hidden, ffn))
    call("zero", ws.p, ws.nbytes)
    return ws


def status(ws) -> tuple[int, int, int]:
    """(invalid_tokens, selected pairs, distinct experts) of the last MoE call on ws."""
    a, b, c = I(0), I(0), I(0)
    call("moe_status", ws if isinstance(ws, int) else ws.p, C.byref(a), C.byref(b), C.byref(c))
    return a.value, b.value, c.value


def row_bytes(typ: int, cols: int) -> int:
    n = U64(0)
    dims = (U64 * 4)(cols, 1, 1, 1)
    call("tensor_bytes", typ, dims, C.byref(n))
    return n.value


def synth_weights(typ: int, rows: int, cols: int, seed: int, stddev: float = 0.02) -> Device:
    buf = Device(nbytes=rows * row_bytes(typ, cols))
    call("synth_weights", buf.p, typ, rows, cols, seed, stddev)
    return buf


def synth_normal(count: int, seed: int, stddev: float = 1.0) -> Device:
    buf = Device(like=np.empty(count, np.float32))
    call("synth_normal", buf.p, count, seed, stddev)
    return buf
