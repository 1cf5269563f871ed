"""Host side of expert parallelism (qg_moe_layer_ep): expert placement, the
per-rank expert buffers, and the exchange of workspace IPC handles.

Placement follows the hot-expert ranking of a layer: experts sorted from
hottest to coldest are dealt across the ranks in snake order (0,1,..,N-1,N-1,
..,1,0,0,1,..), so every rank gets a similar share of hot experts and of
experts. The router and the shared expert stay replicated; one rank per layer
(layer % N) computes the shared expert.

The handle exchange needs only a ``torch.distributed`` process group
(``all_gather_object``), so it works over gloo as well as NCCL.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lib as L

E = 512
Q4K = 12
IPC_HANDLE_BYTES = 64


def snake_owner(ranking: np.ndarray, world: int) -> np.ndarray:
    """owner[e] for experts listed hottest first in `ranking` (a permutation of 0..511)."""
    ranking = np.asarray(ranking, dtype=np.int64)
    if world < 1 or sorted(ranking.tolist()) != list(range(E)):
        raise ValueError("ranking must be a permutation of the 512 experts and world >= 1")
    owner = np.empty(E, np.int32)
    for r, e in enumerate(ranking):
        rnd, pos = divmod(r, world)
        owner[e] = pos if rnd % 2 == 0 else world - 1 - pos
    return owner


def local_map(owner: np.ndarray, rank: int) -> tuple[np.ndarray, list[int]]:
    """expert_local[512] (index on `rank` or -1) and the rank's experts in local order."""
    experts = [int(e) for e in np.flatnonzero(owner == rank)]
    loc = np.full(E, -1, np.int32)
    loc[experts] = np.arange(len(experts), dtype=np.int32)
    return loc, experts


def extract_experts(src: "L.Device", experts: list[int], rows_per_expert: int, row_bytes: int) -> "L.Device":
    """Device copy of the listed experts' rows (gate, up or down of one layer), in that order."""
    per = rows_per_expert * row_bytes
    dst = L.Device(nbytes=len(experts) * per)
    for i, e in enumerate(experts):
        L.call("copy", C.c_void_p(dst.p + i * per), C.c_void_p(src.p + e * per), per)
    return dst


def exchange_handles(handle: bytes, world: int, group=None) -> list[bytes]:
    """Every rank's 64-byte workspace handle, in rank order."""
    import torch.distributed as dist
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle is 64 bytes")
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    if any(not isinstance(h, bytes) or len(h) != IPC_HANDLE_BYTES for h in handles):
        raise RuntimeError("a rank sent no valid workspace handle")
    return handles


class EpGroup:
    """This rank's EP workspace plus every peer's, mapped into this process."""

    def __init__(self, tokens: int, hidden: int, ffn: int, rank: int, world: int, group=None):
        self.rank, self.world = rank, world
        nbytes = C.c_size_t(0)
        L.call("ep_workspace_bytes", tokens, hidden, ffn, C.byref(nbytes))
        self.ws = L.Device(nbytes=nbytes.value)
        L.call("zero", self.ws.p, nbytes.value)
        L.call("sync")
        handle = (C.c_ubyte * IPC_HANDLE_BYTES)()
        L.call("ep_ipc_handle", self.ws.p, handle)
        handles = exchange_handles(bytes(handle), world, group)
        self.mapped = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(self.ws.p)
                continue
            p = C.c_void_p()
            L.call("ep_ipc_open", (C.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(h), C.byref(p))
            self.mapped.append(p.value)
            ptrs.append(p.value)
        self.ptrs = (C.c_void_p * world)(*ptrs)

    def close(self) -> None:
        for p in self.mapped:
            L.call("ep_ipc_close", C.c_void_p(p))
        self.mapped = []
