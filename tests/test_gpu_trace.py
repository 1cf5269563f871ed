"""Replay of a QROUTE1 route trace (the reference's route profiler format,
qwen/qwen.c:87-94,638-646) through qg_moe_routed: every record's recorded
routing - including omitted routes (-e-2 with weight 0, as qg_prune_routes
writes them) and an invalid token - gives the reference CPU MoE's output for
those routes within the path's tolerance, and the invalid token a NaN row."""
import struct

import numpy as np
import pytest

from conftest import assert_parity
from test_gpu_moe import Layer

pytestmark = pytest.mark.gpu
H, F = 2048, 512


def write_trace(path, recs):
    blob = bytearray(b"QROUTE1\n")
    for layer, pos, ids, w in recs:
        blob += struct.pack("<3I", layer, pos, ids.shape[0])
        blob += np.ascontiguousarray(ids, "<i4").tobytes() + np.ascontiguousarray(w, "<f4").tobytes()
    path.write_bytes(bytes(blob))


def test_trace_replay_matches_reference(gpu_lib, ref2048, tmp_path):
    from nebula_b200 import lib as L
    from nebula_b200 import trace
    layers = [Layer(L, H, F, 12, 12, seed=80 + l) for l in range(2)]
    rng = np.random.default_rng(42)
    recs, xs = [], {}
    for i, (layer, nt) in enumerate(((0, 17), (1, 5), (0, 1), (1, 64))):
        ids = np.stack([rng.choice(512, 10, replace=False) for _ in range(nt)]).astype(np.int32)
        w = rng.uniform(0.01, 0.3, (nt, 10)).astype(np.float32)
        w /= w.sum(1, keepdims=True)
        for t in range(0, nt, 4):  # omitted routes
            ids[t, 9] = -ids[t, 9] - 2
            w[t, 9] = 0.0
        if nt > 2:  # one invalid token (duplicate id)
            ids[1, 3] = ids[1, 2]
        recs.append((layer, 17 * i, ids, w))
        xs[i] = rng.normal(0, 1, (nt, H)).astype(np.float32)
    write_trace(tmp_path / "routes.bin", recs)
    order = iter(range(len(recs)))
    dx = {}

    def x_of(layer, nt):
        i = next(order)
        dx[i] = L.Device(xs[i])
        return dx[i]

    def experts_of(layer):
        lay = layers[layer]
        return lay.gate, 12, lay.up, 12, lay.down, 12

    seen = 0
    for i, (layer, pos, out, ws) in enumerate(trace.replay(str(tmp_path / "routes.bin"), experts_of, x_of, H, F)):
        rl, rpos, ids, w = recs[i]
        assert (layer, pos) == (rl, rpos)
        lay = layers[layer]
        o = out.get()
        bad = np.zeros(ids.shape[0], bool)
        if ids.shape[0] > 2:
            bad[1] = True
        ok_ids = ids.copy()
        ok_ids[bad] = np.arange(10)  # any valid routes for the rows the reference would reject
        ref = ref2048.moe(xs[i], ok_ids, w, lay.hgate, 12, lay.hup, 12, lay.hdown, 12)
        assert np.isnan(o[bad]).all(), f"record {i}: the invalid token's row is not NaN"
        assert_parity(o[~bad], ref[~bad], f"record {i} (layer {layer}, {ids.shape[0]} tokens)")
        assert L.status(ws)[0] == int(bad.sum())
        seen += 1
    assert seen == len(recs)
