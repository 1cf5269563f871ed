"""Replay of the reference's QROUTE1 route traces through the routed MoE.

The reference's route profiler (``qwen_profile_routes``, qwen/qwen.c:87-94 and
:638-646) records, for every routed layer call, the layer, the target
position, the token count and the ids and weights of every token's ten
routes. ``records`` reads such a file through the library's C reader
(``qg_route_trace_open/next/close``); ``replay`` feeds every record's routing
to ``qg_moe_routed`` on the caller's resident experts of that layer, so the
experts run with recorded (realistic) routing instead of synthetic logits.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Iterator

import numpy as np

from . import lib as L

TOP = 10


def records(path: str, capacity: int = 8192) -> Iterator[tuple[int, int, np.ndarray, np.ndarray]]:
    """(layer, position, ids [tokens][10] int32, weights [tokens][10] float32) per record."""
    lib = L.load()
    tr = C.c_void_p()
    L.call("route_trace_open", str(path).encode(), C.byref(tr))
    try:
        ids = np.empty((capacity, TOP), np.int32)
        w = np.empty((capacity, TOP), np.float32)
        while True:
            layer, pos, nt = C.c_int(), C.c_int(), C.c_int()
            L.call("route_trace_next", tr, C.byref(layer), C.byref(pos), C.byref(nt), ids.ctypes.data,
                   w.ctypes.data, capacity)
            if nt.value == 0:
                return
            yield layer.value, pos.value, ids[:nt.value].copy(), w[:nt.value].copy()
    finally:
        lib.qg_route_trace_close(tr)


def replay(path: str, experts: Callable[[int], tuple], x: Callable[[int, int], "L.Device"], hidden: int, ffn: int,
           capacity: int = 8192) -> Iterator[tuple[int, int, "L.Device", "L.Device"]]:
    """Runs every record of a trace through qg_moe_routed.

    experts(layer) -> (gate, gate_type, up, up_type, down, down_type) device buffers
    of that layer's resident experts; x(layer, tokens) -> the record's input
    activations on the device. Yields (layer, position, out, workspace) per record
    (out [tokens][hidden]; the workspace holds the call's status words)."""
    ws = L.workspace(min(capacity, 8192), hidden, ffn)
    for layer, pos, ids, w in records(path, capacity):
        nt = ids.shape[0]
        gate, gt, up, ut, down, dt = experts(layer)
        di, dw = L.Device(ids), L.Device(w)
        out = L.Device.empty((nt, hidden), np.float32)
        L.call("moe_routed", out.p, x(layer, nt).p, di.p, dw.p, nt, gate.p, gt, up.p, ut, down.p, dt, hidden, ffn,
               ws.p)
        yield layer, pos, out, ws
