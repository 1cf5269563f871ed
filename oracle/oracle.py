"""TEST INFRASTRUCTURE ONLY - Python face of the CPU checker.

Wraps two libraries built by ``oracle/build.py``:

* the reference's own CPU MoE (``qwen/cpu.c``, ``qwen/cpu_dispatch.c``)
  compiled unmodified into ``oracle/_ref`` - ``qc_matmul`` / ``qc_moe`` /
  ``qc_weight_at`` with the signatures of ``qwen/cpu.h:5-16``;
* ``oracle/restate.c`` - C restatements of the reference's device routing
  steps (``qwen/gpu.cu:456-527,552``).

``moe_layer`` composes them exactly as the reference host does for one MoE
layer (``qwen/qwen.c:714-735``): router GEMV, top-10 routing, routed experts
with the rank-order combine, then the sigmoid-gated shared expert
(``qwen/qwen.c:708-713``).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

from . import build as _build

P, I, F = C.c_void_p, C.c_int, C.c_float
TOP = 10
EXPERTS = 512


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def host_threads() -> int:
    """Threads for the reference CPU MoE: min(28, usable cores) (``qwen/cpu.c:150,164`` cap)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        n = os.cpu_count() or 1
    return max(1, min(28, n))


class RefCPU:
    """The reference CPU MoE library at one compiled shape (``qwen/cpu.c:11``)."""

    def __init__(self, hidden: int = 2048, ffn: int = 512):
        path = _build.ref_path(hidden, ffn)
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run oracle/build.py where the reference tree exists")
        self.hidden, self.ffn = hidden, ffn
        self.lib = lib = C.CDLL(str(path))
        sig = {
            "qc_backend_name": ([], C.c_char_p),
            "qc_backend_available": ([C.c_char_p], I),
            "qc_create": ([I, I], P),
            "qc_destroy": ([P], None),
            "qc_row_bytes": ([I, I], C.c_size_t),
            "qc_weight_at": ([P, I, I], F),
            "qc_matmul": ([P, P, I, I, I, P, I, I], I),
            "qc_moe": ([P, P, P, P, P, I, P, I, P, I, P, I], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res
        self._ws = None
        self._ws_key = None

    def backend(self) -> str:
        return self.lib.qc_backend_name().decode()

    def row_bytes(self, typ: int, cols: int) -> int:
        return int(self.lib.qc_row_bytes(typ, cols))

    def variant(self, prefix: str, name: str):
        """A specific ISA variant's entry point (prefix qcs_, qc2_ or qc5_)."""
        return getattr(self.lib, prefix + name)

    def matmul(self, w: np.ndarray, typ: int, rows: int, cols: int, x: np.ndarray,
               threads: int | None = None) -> np.ndarray:
        """``qc_matmul`` (``qwen/cpu.c:119-148``): out[t][row] with the 32-lane order."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        nt = x.shape[0]
        out = np.empty((nt, rows), np.float32)
        rc = self.lib.qc_matmul(_ptr(out), _ptr(w), typ, rows, cols, _ptr(x), nt, threads or host_threads())
        if rc:
            raise ValueError(f"qc_matmul rejected its arguments (rc={rc})")
        return out

    def _workspace(self, capacity: int, threads: int):
        key = (capacity, threads)
        if self._ws_key != key:
            if self._ws:
                self.lib.qc_destroy(self._ws)
            self._ws = self.lib.qc_create(capacity, threads)
            if not self._ws:
                raise MemoryError("qc_create failed")
            self._ws_key = key
        return self._ws

    def moe(self, x: np.ndarray, ids: np.ndarray, weights: np.ndarray,
            gate: np.ndarray, gt: int, up: np.ndarray, ut: int, down: np.ndarray, dt: int,
            threads: int | None = None, check: bool = True) -> np.ndarray | int:
        """``qc_moe`` (``qwen/cpu.c:235-261``). Returns out [nt][hidden], or the rc when check=False."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        nt = x.shape[0]
        ws = self._workspace(max(nt, 18), threads or host_threads())
        out = np.zeros((nt, self.hidden), np.float32)
        rc = self.lib.qc_moe(ws, _ptr(out), _ptr(x), _ptr(ids), _ptr(weights), nt,
                             _ptr(gate), gt, _ptr(up), ut, _ptr(down), dt)
        if not check:
            return rc
        if rc:
            raise ValueError(f"qc_moe rejected its arguments (rc={rc})")
        return out

    def close(self) -> None:
        if self._ws:
            self.lib.qc_destroy(self._ws)
            self._ws = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PruneStats(C.Structure):
    """``qg_prune_stats`` (``qwen/gpu.h:63-66``)."""
    _fields_ = [("token_layers", C.c_uint64), ("missing_selections", C.c_uint64),
                ("skipped_selections", C.c_uint64), ("avoided_token_handoffs", C.c_uint64),
                ("skipped_mass", C.c_double)]


class Restate:
    """C restatements in ``oracle/restate.c``."""

    def __init__(self):
        path = _build.build_restate() if not _build.restate_path().exists() else _build.restate_path()
        self.lib = lib = C.CDLL(str(path))
        sig = {
            "or_route": ([P, P, P, I], I),
            "or_prune": ([P, P, P, I, C.c_double, P], I),
            "or_moe_map": ([P, P, P, I], I),
            "or_swiglu": ([P, P, P, C.c_size_t], None),
            "or_shared_add": ([P, P, P, I, I], None),
            "or_moe_reduce": ([P, P, I, I], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res

    def route(self, logits: np.ndarray):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        nt = logits.shape[0]
        ids = np.zeros((nt, TOP), np.int32)
        w = np.zeros((nt, TOP), np.float32)
        if self.lib.or_route(_ptr(ids), _ptr(w), _ptr(logits), nt):
            raise ValueError("or_route")
        return ids, w

    def prune(self, ids: np.ndarray, weights: np.ndarray, resident: np.ndarray, threshold: float,
              stats: PruneStats | None = None):
        ids = np.ascontiguousarray(ids, dtype=np.int32).copy()
        weights = np.ascontiguousarray(weights, dtype=np.float32).copy()
        resident = np.ascontiguousarray(resident, dtype=np.uint8)
        stats = stats or PruneStats()
        rc = self.lib.or_prune(_ptr(ids), _ptr(weights), _ptr(resident), ids.shape[0], threshold,
                               C.addressof(stats))
        return rc, ids, weights, stats

    def moe_map(self, ids: np.ndarray):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        nt = ids.shape[0]
        m = np.zeros((EXPERTS, nt), np.int32)
        counts = np.zeros(EXPERTS, np.int32)
        if self.lib.or_moe_map(_ptr(m), _ptr(counts), _ptr(ids), nt):
            raise ValueError("or_moe_map")
        return m, counts

    def swiglu(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, dtype=np.float32)
        u = np.ascontiguousarray(u, dtype=np.float32)
        mid = np.empty_like(g)
        self.lib.or_swiglu(_ptr(mid), _ptr(g), _ptr(u), g.size)
        return mid

    def shared_add(self, out: np.ndarray, shared: np.ndarray, gate: np.ndarray) -> None:
        gate = np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
        shared = np.ascontiguousarray(shared, dtype=np.float32)
        self.lib.or_shared_add(_ptr(out), _ptr(shared), _ptr(gate), out.shape[0], out.shape[1])

    def moe_reduce(self, slots: np.ndarray) -> np.ndarray:
        slots = np.ascontiguousarray(slots, dtype=np.float32)
        nt, _, width = slots.shape
        out = np.empty((nt, width), np.float32)
        self.lib.or_moe_reduce(_ptr(out), _ptr(slots), nt, width)
        return out


def moe_layer(ref: RefCPU, rs: Restate, x: np.ndarray, router: np.ndarray,
              gate: np.ndarray, gt: int, up: np.ndarray, ut: int, down: np.ndarray, dt: int,
              shared: tuple | None = None, logits: np.ndarray | None = None,
              threads: int | None = None):
    """One routed-MoE layer as ``qwen/qwen.c:714-735`` runs it, on the CPU.

    router: F32 [512][hidden] (``ffn_gate_inp``); shared = (sg, sgt, su, sut, sd, sdt,
    s_router F32 [hidden]) or None. ``logits`` overrides the router GEMV (config 4 feeds
    logits directly). Returns (out [nt][hidden], ids, weights, logits).
    """
    H, Fd = ref.hidden, ref.ffn
    if logits is None:
        logits = ref.matmul(router, 0, EXPERTS, H, x, threads)
    ids, w = rs.route(logits)
    out = ref.moe(x, ids, w, gate, gt, up, ut, down, dt, threads)
    if shared is not None:
        sg, sgt, su, sut, sd, sdt, sr = shared
        g = ref.matmul(sg, sgt, Fd, H, x, threads)
        u = ref.matmul(su, sut, Fd, H, x, threads)
        mid = rs.swiglu(g, u)
        sh = ref.matmul(sd, sdt, H, Fd, mid, threads)
        sgate = ref.matmul(sr, 0, 1, H, x, threads)
        rs.shared_add(out, sh, sgate)
    return out, ids, w, logits


class Synth:
    """``oracle/synth.c``: the library's synthetic generator restated on the host,
    bit for bit (``qg_synth_weights`` / ``qg_synth_normal``)."""

    def __init__(self):
        path = _build.build_synth() if not _build.synth_path().exists() else _build.synth_path()
        self.lib = lib = C.CDLL(str(path))
        lib.or_synth_normal.argtypes = [P, C.c_uint64, C.c_uint64, C.c_uint64, F]
        lib.or_synth_normal.restype = None
        lib.or_synth_weights.argtypes = [P, I, I, C.c_uint64, F, C.c_int64, C.c_int64]
        lib.or_synth_weights.restype = I

    @staticmethod
    def row_bytes(typ: int, cols: int) -> int:
        return {0: cols * 4, 12: cols // 256 * 144, 20: cols // 32 * 18}[typ]

    def weights(self, typ: int, rows: int, cols: int, seed: int, stddev: float = 0.02,
                out: np.ndarray | None = None, row0: int = 0, nrows: int | None = None) -> np.ndarray:
        """Rows [row0, row0+nrows) of the rows x cols matrix into ``out`` (a flat uint8
        array of the whole matrix; allocated when None, untouched outside those rows)."""
        rb = self.row_bytes(typ, cols)
        if out is None:
            out = np.empty(rows * rb, np.uint8)
        nrows = rows - row0 if nrows is None else nrows
        if row0 < 0 or nrows < 0 or row0 + nrows > rows or out.nbytes < rows * rb:
            raise ValueError("row range outside the matrix")
        if self.lib.or_synth_weights(out.ctypes.data + row0 * rb, typ, cols, seed, stddev, row0, nrows):
            raise ValueError("or_synth_weights")
        return out

    def normal(self, count: int, seed: int, stddev: float = 1.0) -> np.ndarray:
        out = np.empty(count, np.float32)
        self.lib.or_synth_normal(out.ctypes.data, 0, count, seed, stddev)
        return out
