"""GPU parity of the reference-ABI primitives (qwen/gpu.h) against the CPU
checker: the reference's own CPU code (oracle/_ref), the C restatements of its
device routing steps (oracle/restate.c), and the golden fixtures. Ports the
MoE-path cases of qwen/test_gpu.py."""
import ctypes as C

import numpy as np
import pytest

import make_golden as mg
from oracle.blocks import dequant64, random_blocks

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(gpu_lib):
    from nebula_b200 import lib
    return lib


def test_dequant_matches_reference_decoder_bitwise(L):
    formats = np.load(mg.OUT / "formats.npz")
    for typ in mg.TYPES:
        packed, values = formats[f"packed_{typ}"], formats[f"values_{typ}"]
        rows, cols = values.shape
        dp = L.Device(packed)
        out = L.Device.empty((rows, cols), np.float32)
        L.call("dequant", out.p, dp.p, typ, rows, cols)
        np.testing.assert_array_equal(out.get(), values, err_msg=f"type {typ}")
        row = L.Device.empty((cols,), np.float32)
        L.call("gather", row.p, dp.p, typ, cols, rows - 1)
        np.testing.assert_array_equal(row.get(), values[-1], err_msg=f"gather type {typ}")


@pytest.mark.parametrize("typ", (0, 12, 20))
@pytest.mark.parametrize("shape", mg.MATMUL_SHAPES)
def test_matmul_bitwise_vs_golden(L, typ, shape):
    gold = np.load(mg.OUT / "matmul.npz")
    rows, cols = shape
    w, xs = mg.matmul_case_inputs(typ, rows, cols)
    dw = L.Device(w)
    for nt, x in zip(mg.MATMUL_TOKENS, xs):
        dx = L.Device(x)
        out = L.Device.empty((nt, rows), np.float32)
        L.call("matmul", out.p, dw.p, typ, rows, cols, dx.p, nt)
        np.testing.assert_array_equal(out.get(), gold[f"out_{typ}_{cols}_{nt}"], err_msg=f"type {typ} nt {nt}")


@pytest.mark.parametrize("typ", (0, 1, 30, 2, 6, 7, 8, 12, 13, 14, 20))
def test_matmul_bitwise_vs_qc_matmul(L, ref2048, typ):
    """qwen/test_gpu.py:110-162 shapes and batch tails; bit-exact against qc_matmul."""
    rng = np.random.default_rng(812603 + typ)
    for cols in ((256, 768) if typ in (12, 13, 14) else (320, 640)):
        rows = 13
        w = random_blocks(rng, typ, rows, cols, d=0.002, dmin=0.001)
        dw = L.Device(w)
        for nt in (1, 2, 4, 5, 8, 9, 16, 17, 18, 19, 33, 512, 2048):
            x = (rng.normal(size=(nt, cols)) * 0.2).astype(np.float32)
            dx = L.Device(x)
            out = L.Device.empty((nt, rows), np.float32)
            L.call("matmul", out.p, dw.p, typ, rows, cols, dx.p, nt)
            ref = ref2048.matmul(w, typ, rows, cols, x)
            np.testing.assert_array_equal(out.get(), ref, err_msg=f"type {typ} cols {cols} nt {nt}")


@pytest.mark.parametrize("nt", (17, 2048))
def test_router_gemv_bitwise_at_model_shape(L, ref2048, nt):
    """The router of a verify batch (one warp per row) and of a prefill batch
    (tiled kernel), both bitwise equal to qc_matmul."""
    rng = np.random.default_rng(0)
    router = rng.normal(0, 0.02, (512, 2048)).astype(np.float32)
    x = rng.normal(0, 1, (nt, 2048)).astype(np.float32)
    dr, dx = L.Device(router), L.Device(x)
    out = L.Device.empty((nt, 512), np.float32)
    L.call("matmul", out.p, dr.p, 0, 512, 2048, dx.p, nt)
    np.testing.assert_array_equal(out.get(), ref2048.matmul(router.view(np.uint8), 0, 512, 2048, x))


@pytest.mark.parametrize("rows,nt", ((1, 2048), (1, 100), (48, 100), (40, 77)))
def test_tiled_gemv_ragged_shapes_bitwise(L, ref2048, rows, nt):
    """The tiled fp32 kernel on a shared-gate row (8 x 16 tiles) and on row and
    token counts that leave partial tiles (32 x 32 tiles), bitwise qc_matmul."""
    rng = np.random.default_rng(rows * 1000 + nt)
    w = rng.normal(0, 0.02, (rows, 2048)).astype(np.float32)
    x = rng.normal(0, 1, (nt, 2048)).astype(np.float32)
    dw, dx = L.Device(w), L.Device(x)
    out = L.Device.empty((nt, rows), np.float32)
    L.call("matmul", out.p, dw.p, 0, rows, 2048, dx.p, nt)
    np.testing.assert_array_equal(out.get(), ref2048.matmul(w.view(np.uint8), 0, rows, 2048, x))


def test_route_matches_restatement(L, restate):
    rng = np.random.default_rng(812603)
    nt = 2048
    logits = (rng.normal(size=(nt, 512))).astype(np.float32)
    logits[0] = 0
    logits[1, ::5] = 3.0  # ties at the top
    logits[2, 7] = np.nan
    logits[3, 300] = -np.inf
    dl = L.Device(logits)
    ids, w = L.Device.empty((nt, 10), np.int32), L.Device.empty((nt, 10), np.float32)
    L.call("route", ids.p, w.p, dl.p, nt)
    rid, rw = restate.route(logits)
    np.testing.assert_array_equal(ids.get(), rid)
    np.testing.assert_allclose(w.get(), rw, rtol=1e-6, atol=0)  # CUDA vs host expf: a few ulp
    sel = np.argsort(-logits[4:], axis=1, kind="stable")[:, :10]
    np.testing.assert_array_equal(ids.get()[4:], sel)
    assert (ids.get()[2] == -1).all() and (ids.get()[3] == -1).all()


def test_prune_known_answer(L, restate):
    """qwen/test_gpu.py:84-95."""
    class Counters(C.Structure):
        _fields_ = [(k, C.c_uint64) for k in ("token_layers", "missing", "skipped", "avoided")] + [("mass", C.c_double)]
    ids = np.tile(np.arange(10, dtype=np.int32), (5, 1))
    weights = np.full((5, 10), .1, np.float32)
    resident = np.zeros(512, np.uint8)
    resident[:8] = 1
    weights[0, 8:] = .04
    weights[1, 8:] = .05
    weights[2, 8:] = .06
    weights[3, 8:] = 0
    weights[4, 8:] = [.01, .10]
    di, dw, dr = L.Device(ids), L.Device(weights), L.Device(resident)
    dc = L.Device(np.zeros(C.sizeof(Counters), np.uint8))
    L.call("prune_routes", di.p, dw.p, dr.p, 5, .10, dc.p)
    rc, rids, rw, st = restate.prune(ids, weights, resident, .10)
    np.testing.assert_array_equal(di.get(), rids)
    np.testing.assert_array_equal(dw.get(), rw)
    got = Counters.from_buffer_copy(dc.get())
    assert (got.token_layers, got.missing, got.skipped, got.avoided) == (5, 10, 4, 2)
    assert got.mass == pytest.approx(st.skipped_mass, rel=1e-12)


def test_moe_map_matches_restatement(L, restate):
    """qwen/test_gpu.py:352-359 and the 8192 case of qwen/test_large_profiles.py."""
    rng = np.random.default_rng(44)
    for nt in (1, 17, 511, 513, 1025, 2048, 8192):
        ids = np.stack([rng.choice(512, 10, replace=False) for _ in range(nt)]).astype(np.int32)
        dids = L.Device(ids)
        m = L.Device(np.full((512, nt), -7, np.int32))
        L.call("moe_map", m.p, dids.p, nt)
        rm, counts = restate.moe_map(ids)
        got = m.get()
        for e in range(512):
            np.testing.assert_array_equal(got[e, :counts[e]], rm[e, :counts[e]], err_msg=f"nt {nt} e {e}")


def test_gather_scatter_reduce_replay_independent(L):
    """qwen/test_gpu.py:361-384: two expert orders give bitwise-equal reductions."""
    rng = np.random.default_rng(812603)
    nt = 4
    ids = np.stack([rng.choice(27, 10, replace=False) for _ in range(nt)]).astype(np.int32)
    weights = np.exp(rng.normal(size=(nt, 10)) * .2).astype(np.float32)
    weights /= weights.sum(1, keepdims=True)
    values = (rng.normal(size=(27, nt, 2560)) * 6).astype(np.float32)
    dids, dw = L.Device(ids), L.Device(weights)
    mapping = L.Device(np.zeros((512, nt), np.int32))
    L.call("moe_map", mapping.p, dids.p, nt)
    slots = L.Device(np.zeros((nt, 10, 2560), np.float32))
    out = L.Device(np.zeros((nt, 2560), np.float32))
    expected = np.zeros((nt, 2560), np.float32)
    for k in range(10):
        expected += values[ids[:, k], np.arange(nt)] * weights[:, k, None]
    results = []
    for order in (np.unique(ids), rng.permutation(np.unique(ids))):
        L.call("zero", slots.p, slots.nbytes)
        for expert in order:
            selected = (ids == expert).any(1)
            dx = L.Device(values[expert])
            compact = L.Device(np.zeros_like(values[expert]))
            token_map = mapping.p + int(expert) * nt * 4
            L.call("moe_gather", compact.p, dx.p, token_map, int(selected.sum()))
            np.testing.assert_array_equal(compact.get()[:selected.sum()], values[expert, selected])
            L.call("moe_scatter", slots.p, compact.p, dw.p, dids.p, token_map, int(expert), int(selected.sum()))
        L.call("moe_reduce", out.p, slots.p, nt)
        results.append(out.get())
    np.testing.assert_array_equal(results[0], results[1])
    np.testing.assert_allclose(results[0], expected, rtol=2e-5, atol=2e-5)


def test_mtp_moe_seventeen_rows(L):
    """qwen/test_gpu.py:164-187: Q4_K/Q4_K/IQ4_NL at 2560/640 vs float64 NumPy; 18 rows rejected."""
    rng = np.random.default_rng(812603)
    mats, dev = [], []
    for typ, rows, cols in ((12, 640, 2560), (12, 640, 2560), (20, 2560, 640)):
        packed = random_blocks(rng, typ, 2 * rows, cols, d=.0002, dmin=.0001)
        mats.append(dequant64(packed, typ, 2 * rows, cols).reshape(2, rows, cols))
        dev.append(L.Device(packed))
    nt = 17
    x = (rng.normal(size=(nt, 2560)) * .2).astype(np.float32)
    ids = rng.integers(0, 2, (nt, 10), dtype=np.int32)
    scales = rng.uniform(.01, .2, (nt, 10)).astype(np.float32)
    dx, di, dw = L.Device(x), L.Device(ids), L.Device(scales)
    mid = L.Device(np.zeros((nt, 10, 640), np.float32))
    slots = L.Device(np.zeros((nt, 10, 2560), np.float32))
    L.call("mtp_moe", slots.p, mid.p, dx.p, di.p, dw.p, dev[0].p, 12, dev[1].p, 12, dev[2].p, 20, nt)
    sig = lambda v: 1 / (1 + np.exp(-v))
    expected = np.empty((nt, 10, 2560))
    for e in range(2):
        g = x.astype(np.float64) @ mats[0][e].T
        u = x.astype(np.float64) @ mats[1][e].T
        y = ((g * sig(g)) * u) @ mats[2][e].T
        for t, k in zip(*np.nonzero(ids == e)):
            expected[t, k] = y[t] * scales[t, k]
    np.testing.assert_allclose(slots.get(), expected, atol=2e-5, rtol=5e-5)
    assert L.code("mtp_moe", slots.p, mid.p, dx.p, di.p, dw.p, dev[0].p, 12, dev[1].p, 12, dev[2].p, 20, 18) != 0
    bad = ids.copy()
    bad[3, 4] = -1
    di.set(bad)
    L.call("mtp_moe", slots.p, mid.p, dx.p, di.p, dw.p, dev[0].p, 12, dev[1].p, 12, dev[2].p, 20, nt)
    assert np.isnan(slots.get()[3, 4]).all() and np.isfinite(slots.get()[3, 3]).all()


def test_elementwise_ops(L, restate):
    rng = np.random.default_rng(1)
    n = 4 * 2560
    a = rng.normal(size=n).astype(np.float32) * 3
    b = rng.normal(size=n).astype(np.float32)
    da, db, do = L.Device(a), L.Device(b), L.Device.empty((n,), np.float32)
    L.call("unary", do.p, da.p, n, 0, 1.0)
    np.testing.assert_allclose(do.get(), restate.swiglu(a, np.ones_like(a)), rtol=3e-7, atol=1e-30)
    L.call("unary", do.p, da.p, n, 1, 0.5)
    np.testing.assert_allclose(do.get(), 1 / (1 + np.exp(-(a * 0.5).astype(np.float64))), rtol=1e-6)
    L.call("binary", do.p, da.p, db.p, n, 0)
    np.testing.assert_array_equal(do.get(), a + b)
    L.call("binary", do.p, da.p, db.p, n, 1)
    np.testing.assert_array_equal(do.get(), a * b)
    base = rng.normal(size=(4, 2560)).astype(np.float32)
    gate = rng.normal(size=4).astype(np.float32)
    dbase, dg = L.Device(base), L.Device(gate)
    L.call("shared_add", dbase.p, da.p, dg.p, 4)
    expected = base.copy()
    restate.shared_add(expected, a.reshape(4, 2560), gate)
    np.testing.assert_allclose(dbase.get(), expected, rtol=3e-7, atol=1e-6)


def test_graph_replay_equals_eager(L, ref2048):
    rng = np.random.default_rng(2)
    w = random_blocks(rng, 12, 64, 2048)
    x = rng.normal(size=(5, 2048)).astype(np.float32)
    dw, dx = L.Device(w), L.Device(x)
    out = L.Device(np.zeros((5, 64), np.float32))
    g = C.c_void_p()
    L.call("graph_begin", C.byref(g))
    try:
        L.call("matmul", out.p, dw.p, 12, 64, 2048, dx.p, 5)
        L.call("graph_end", g)
        for _ in range(2):
            L.call("zero", out.p, out.nbytes)
            L.call("graph_launch", g)
            np.testing.assert_array_equal(out.get(), ref2048.matmul(w, 12, 64, 2048, x))
    finally:
        L.load().qg_graph_destroy(g)


def test_buffer_collected_during_capture_is_freed_after_it(L, ref2048):
    """A device buffer that Python finalizes while this thread records a graph (a
    reference cycle collected mid-capture) is freed at qg_graph_end, not during the
    capture, whose cudaFree would invalidate it."""
    import gc

    class Cycle:
        pass

    rng = np.random.default_rng(3)
    w = random_blocks(rng, 12, 32, 512)
    x = rng.normal(size=(3, 512)).astype(np.float32)
    dw, dx = L.Device(w), L.Device(x)
    out = L.Device(np.zeros((3, 32), np.float32))
    c = Cycle()
    c.me, c.buf = c, L.Device(nbytes=1 << 20)
    del c
    g = C.c_void_p()
    gc.disable()
    L.call("graph_begin", C.byref(g))
    try:
        gc.collect()  # finalizes the cycle's buffer inside the capture
        L.call("matmul", out.p, dw.p, 12, 32, 512, dx.p, 3)
        L.call("graph_end", g)
        L.call("graph_launch", g)
        np.testing.assert_array_equal(out.get(), ref2048.matmul(w, 12, 32, 512, x))
    finally:
        gc.enable()
        L.load().qg_graph_destroy(g)


def test_upload_expert_packs_gate_up_down(L):
    rng = np.random.default_rng(3)
    parts = [rng.integers(0, 256, n, dtype=np.uint8) for n in (1152 * 8, 1152 * 8, 288 * 32)]
    total = sum(p.size for p in parts)
    up = L.load().qg_upload_create(total)
    assert up
    dst = L.Device(np.zeros(total, np.uint8))
    try:
        L.call("upload_expert", up, dst.p, parts[0].ctypes.data, parts[0].size, parts[1].ctypes.data,
               parts[1].size, parts[2].ctypes.data, parts[2].size)
        L.call("sync")
        np.testing.assert_array_equal(dst.get(), np.concatenate(parts))
        assert L.load().qg_upload_seconds(up) >= 0
        assert L.code("upload_expert", up, dst.p, parts[0].ctypes.data, total + 1, None, 0, None, 0) != 0
    finally:
        L.load().qg_upload_destroy(up)


@pytest.mark.parametrize("typ,rows,cols,seed,std", ((12, 640, 2048, 901, 0.02), (20, 300, 2048, 17, 0.02),
                                                   (0, 512, 2048, 904, 0.02), (12, 2048, 512, 3, 0.02),
                                                   (20, 2560, 640, 8, 0.5)))
def test_host_synth_restatement_matches_device_bytes(L, typ, rows, cols, seed, std):
    """oracle/synth.c gives the device generator's bytes bit for bit, so the CPU
    baselines can run on the GPU arm's exact layers."""
    from oracle.oracle import Synth
    dev = L.synth_weights(typ, rows, cols, seed, std).get()
    host = Synth().weights(typ, rows, cols, seed, std)
    np.testing.assert_array_equal(dev, host)
    # a row range alone, as the CPU baselines generate the experts they need
    part = np.zeros_like(host)
    Synth().weights(typ, rows, cols, seed, std, out=part, row0=rows // 3, nrows=rows // 4)
    rb = host.nbytes // rows
    lo, hi = rows // 3 * rb, (rows // 3 + rows // 4) * rb
    np.testing.assert_array_equal(part[lo:hi], host[lo:hi])
    x = L.synth_normal(100_003, seed + 1).get()
    np.testing.assert_array_equal(x, Synth().normal(100_003, seed + 1))
