"""GPU parity of the fused routed-MoE entry points (qg_moe_routed,
qg_moe_layer) against the reference CPU MoE (qc_moe / qc_matmul from
oracle/_ref plus the restated routing and shared expert), on the shapes and
formats of the benchmark configurations.

Tolerance (floating point): rel-L2 <= 1e-5 and max-abs <= 1e-4 * max|ref|.
Expert ids must be bit-exact."""
import ctypes as C

import numpy as np
import pytest

import make_golden as mg
from conftest import assert_parity, rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(gpu_lib):
    from nebula_b200 import lib
    return lib


class Layer:
    """One layer of 512 synthetic experts on the device plus host copies."""

    def __init__(self, L, H, F, gt, dt, seed, shared=False, experts=512):
        self.L, self.H, self.F, self.gt, self.dt = L, H, F, gt, dt
        rows = experts * F
        self.gate = L.synth_weights(gt, rows, H, seed * 10 + 1)
        self.up = L.synth_weights(gt, rows, H, seed * 10 + 2)
        self.down = L.synth_weights(dt, experts * H, F, seed * 10 + 3)
        self.router = L.synth_weights(0, 512, H, seed * 10 + 4)
        self.hgate, self.hup, self.hdown = self.gate.get(), self.up.get(), self.down.get()
        self.hrouter = self.router.get().view(np.float32).reshape(512, H)
        self.shared = None
        if shared:
            self.sg = L.synth_weights(gt, F, H, seed * 10 + 5)
            self.su = L.synth_weights(gt, F, H, seed * 10 + 6)
            self.sd = L.synth_weights(dt, H, F, seed * 10 + 7)
            self.sr = L.synth_weights(0, 1, H, seed * 10 + 8)
            self.shared = (self.sg.get(), gt, self.su.get(), gt, self.sd.get(), dt,
                           self.sr.get().view(np.float32).reshape(1, H))

    def routed(self, x, ids, w):
        L = self.L
        T = x.shape[0]
        dx, di, dw = L.Device(x), L.Device(ids), L.Device(w)
        out = L.Device.empty((T, self.H), np.float32)
        ws = L.workspace(T, self.H, self.F)
        L.call("moe_routed", out.p, dx.p, di.p, dw.p, T, self.gate.p, self.gt, self.up.p, self.gt,
               self.down.p, self.dt, self.H, self.F, ws.p)
        return out.get(), ws

    def layer(self, x, bias=None, ws=None):
        L = self.L
        T = x.shape[0]
        dx = L.Device(x)
        out = L.Device.empty((T, self.H), np.float32)
        ids, w = L.Device.empty((T, 10), np.int32), L.Device.empty((T, 10), np.float32)
        ws = ws if ws is not None else L.workspace(T, self.H, self.F)
        db = L.Device(bias) if bias is not None else None
        sh = (self.sg.p, self.gt, self.su.p, self.gt, self.sd.p, self.dt, self.sr.p) if self.shared else \
            (None, 0, None, 0, None, 0, None)
        L.call("moe_layer", out.p, ids.p, w.p, dx.p, T, self.router.p, db.p if db else None,
               self.gate.p, self.gt, self.up.p, self.gt, self.down.p, self.dt, *sh, self.H, self.F, ws.p)
        return out.get(), ids.get(), w.get(), ws


def oracle_routed(ref, layer, x, ids, w):
    return ref.moe(x, ids, w, layer.hgate, layer.gt, layer.hup, layer.gt, layer.hdown, layer.dt)


@pytest.fixture(scope="module")
def q4k_2048(L):
    return Layer(L, 2048, 512, 12, 12, seed=0, shared=True)


@pytest.fixture(scope="module")
def iq4_2048(L):
    return Layer(L, 2048, 512, 20, 20, seed=1, shared=True)


@pytest.fixture(scope="module")
def prod_2560(L):
    return Layer(L, 2560, 640, 12, 20, seed=2, shared=True)


def random_routes(rng, T, experts=512):
    ids = np.stack([rng.choice(experts, 10, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.01, 0.3, (T, 10)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    return ids, w


@pytest.mark.parametrize("T", (1, 4, 17))
def test_routed_q4k_2048(L, ref2048, q4k_2048, T):
    rng = np.random.default_rng(T)
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    ids, w = random_routes(rng, T)
    out, ws = q4k_2048.routed(x, ids, w)
    assert_parity(out, oracle_routed(ref2048, q4k_2048, x, ids, w), f"Q4_K T={T}")
    inv, sel, used = L.status(ws)
    assert inv == 0 and sel == T * 10 and used == len(np.unique(ids))


@pytest.mark.parametrize("T", (1, 17, 18))
def test_routed_iq4nl_2048(L, ref2048, iq4_2048, T):
    rng = np.random.default_rng(100 + T)
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    ids, w = random_routes(rng, T)
    out, _ = iq4_2048.routed(x, ids, w)
    assert_parity(out, oracle_routed(ref2048, iq4_2048, x, ids, w), f"IQ4_NL T={T}")


@pytest.mark.parametrize("T", (1, 17, 30, 33))
def test_layer_iq4nl_with_shared_expert(L, ref2048, restate, iq4_2048, T):
    """All-IQ4_NL experts (config 2's format) through the whole layer with an
    IQ4_NL shared expert: 24- and 32-token decode tiles on the tensor cores, and
    a batch above 32 on the general path."""
    rng = np.random.default_rng(500 + T)
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    out, ids, w, ws = iq4_2048.layer(x)
    e_out, e_ids, e_w, _ = orc.moe_layer(ref2048, restate, x, iq4_2048.hrouter, iq4_2048.hgate, 20,
                                         iq4_2048.hup, 20, iq4_2048.hdown, 20, shared=iq4_2048.shared)
    np.testing.assert_array_equal(ids, e_ids)
    assert_parity(out, e_out, f"IQ4_NL layer T={T}")
    inv, sel, used = L.status(ws)
    assert inv == 0 and sel == T * 10 and used == len(np.unique(e_ids))


@pytest.mark.parametrize("T", (1, 5, 17, 33))
def test_routed_product_shape_2560(L, ref2560, prod_2560, T):
    """Nebula's production mix: Q4_K gate/up, IQ4_NL down, hidden 2560, ffn 640."""
    rng = np.random.default_rng(200 + T)
    x = rng.normal(0, 1, (T, 2560)).astype(np.float32)
    ids, w = random_routes(rng, T)
    out, _ = prod_2560.routed(x, ids, w)
    assert_parity(out, oracle_routed(ref2560, prod_2560, x, ids, w), f"2560 T={T}")


@pytest.mark.parametrize("case", mg.MOE_CASES, ids=lambda c: f"{c[0]}x{c[1]}_t{c[2]}_{c[3]}")
def test_routed_on_golden_inputs(L, case):
    """The golden qc_moe inputs (random legal blocks, omitted routes every third token)."""
    hidden, ffn, gt, dt, seed = case
    ref = orc.RefCPU(hidden, ffn)
    gate, up, down, x, ids, w = mg.moe_case_inputs(*case)
    # pad the 12 experts to a 512-expert layout is unnecessary: ids < 12
    dg, du, dd = L.Device(gate), L.Device(up), L.Device(down)
    for nt in mg.MOE_TOKENS:
        dx, di, dw = L.Device(x[:nt]), L.Device(ids[:nt]), L.Device(w[:nt])
        out = L.Device.empty((nt, hidden), np.float32)
        ws = L.workspace(nt, hidden, ffn)
        L.call("moe_routed", out.p, dx.p, di.p, dw.p, nt, dg.p, gt, du.p, gt, dd.p, dt, hidden, ffn, ws.p)
        expected = ref.moe(x[:nt], ids[:nt], w[:nt], gate, gt, up, gt, down, dt)
        assert_parity(out.get(), expected, f"golden {case} nt={nt}")


def test_invalid_and_omitted_routes(L, ref2048, q4k_2048):
    rng = np.random.default_rng(7)
    T = 9
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    ids, w = random_routes(rng, T)
    # omitted routes (qg_prune_routes encoding): contribute nothing
    ids[0, 9], w[0, 9] = -ids[0, 9] - 2, 0.0
    ids[5, 3], w[5, 3] = -ids[5, 3] - 2, 0.0
    bad = ids.copy()
    bad_w = w.copy()
    bad[1, :] = -1          # router's invalid-distribution sentinel
    bad[2, 4] = bad[2, 3]   # duplicate id
    bad_w[3, 0] = np.nan    # non-finite weight
    bad_w[4, 1] = -0.1      # negative weight
    out, ws = q4k_2048.routed(x, bad, bad_w)
    good = [0, 5, 6, 7, 8]
    expected = oracle_routed(ref2048, q4k_2048, x[good], ids[good], w[good])
    assert_parity(out[good], expected, "valid rows next to invalid ones")
    assert np.isnan(out[[1, 2, 3, 4]]).all()
    inv, sel, _ = L.status(ws)
    assert inv == 4 and sel == 5 * 10 - 2


def test_invalid_and_omitted_routes_large_batch(L, ref2048, q4k_2048):
    """A batch planned by several CTAs (chunks of 128 tokens, the last one
    ragged), with invalid and omitted routes in different chunks."""
    rng = np.random.default_rng(17)
    T = 300
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    ids, w = random_routes(rng, T)
    for t, k in ((0, 9), (200, 3), (299, 0)):
        ids[t, k], w[t, k] = -ids[t, k] - 2, 0.0
    bad, bad_w = ids.copy(), w.copy()
    bad[1, :] = -1
    bad[130, 4] = bad[130, 3]
    bad_w[257, 0] = np.nan
    bad_w[298, 1] = -0.1
    out, ws = q4k_2048.routed(x, bad, bad_w)
    good = [t for t in range(T) if t not in (1, 130, 257, 298)]
    expected = oracle_routed(ref2048, q4k_2048, x[good], ids[good], w[good])
    assert_parity(out[good], expected, "large batch: valid rows next to invalid ones")
    assert np.isnan(out[[1, 130, 257, 298]]).all()
    inv, sel, used = L.status(ws)
    assert inv == 4 and sel == len(good) * 10 - 3
    assert used == len(np.unique(ids[good][ids[good] >= 0]))


def test_workspace_reuse_across_paths(L, ref2048, q4k_2048):
    """One zeroed workspace serves many calls: decode-path calls (T <= 17) leave
    their counters at zero, and large-batch calls in between do not disturb them."""
    rng = np.random.default_rng(21)
    ws = L.workspace(40, 2048, 512)
    lay = q4k_2048
    for T in (17, 3, 40, 1, 17, 40, 9):
        x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
        ids, w = random_routes(rng, T)
        dx, di, dw = L.Device(x), L.Device(ids), L.Device(w)
        out = L.Device.empty((T, 2048), np.float32)
        L.call("moe_routed", out.p, dx.p, di.p, dw.p, T, lay.gate.p, 12, lay.up.p, 12, lay.down.p, 12, 2048, 512, ws.p)
        assert_parity(out.get(), oracle_routed(ref2048, lay, x, ids, w), f"reuse T={T}")
        inv, sel, used = L.status(ws)
        assert (inv, sel, used) == (0, T * 10, len(np.unique(ids)))


def test_replay_is_deterministic(L, q4k_2048):
    rng = np.random.default_rng(8)
    x = rng.normal(0, 1, (17, 2048)).astype(np.float32)
    ids, w = random_routes(rng, 17)
    a, _ = q4k_2048.routed(x, ids, w)
    b, _ = q4k_2048.routed(x, ids, w)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("T", (1, 4, 17))
def test_layer_with_shared_expert(L, ref2048, restate, q4k_2048, T):
    """Config 1/3 shape: router GEMV + top-10 + routed experts + gated shared expert."""
    rng = np.random.default_rng(300 + T)
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    out, ids, w, ws = q4k_2048.layer(x)
    e_out, e_ids, e_w, _ = orc.moe_layer(ref2048, restate, x, q4k_2048.hrouter, q4k_2048.hgate, 12,
                                         q4k_2048.hup, 12, q4k_2048.hdown, 12, shared=q4k_2048.shared)
    np.testing.assert_array_equal(ids, e_ids)
    np.testing.assert_allclose(w, e_w, rtol=1e-6, atol=0)
    assert_parity(out, e_out, f"layer T={T}")


@pytest.mark.parametrize("T", (1, 2, 3, 4, 17, 300))
def test_layer_product_shape_with_shared_expert(L, ref2560, restate, prod_2560, T):
    """The production mix at 2560/640 (Q4_K gate/up, IQ4_NL down, IQ4_NL shared
    down) through the whole layer: the single-kernel layer (1 to 4 tokens), the
    tensor-core decode path (T <= 32) and the large-batch path."""
    rng = np.random.default_rng(400 + T)
    x = rng.normal(0, 1, (T, 2560)).astype(np.float32)
    out, ids, w, ws = prod_2560.layer(x)
    e_out, e_ids, e_w, _ = orc.moe_layer(ref2560, restate, x, prod_2560.hrouter, prod_2560.hgate, 12,
                                         prod_2560.hup, 12, prod_2560.hdown, 20, shared=prod_2560.shared)
    np.testing.assert_array_equal(ids, e_ids)
    assert_parity(out, e_out, f"product layer T={T}")
    inv, sel, used = L.status(ws)
    assert inv == 0 and sel == T * 10 and used == len(np.unique(e_ids))


def test_layer_product_small_batches_share_one_workspace(L, ref2560, restate, prod_2560):
    """The production mix's single-kernel layer has a 2-token and a 4-token
    instance; both advance the same grid-barrier counter of the workspace. Calls
    of T = 1, 3, 2, 4, 4, 1 on one workspace (a non-finite token in the fifth)
    each match the reference: ids bit-exact, outputs within tolerance, status
    words of that call."""
    rng = np.random.default_rng(700)
    ws = L.workspace(4, 2560, 640)
    for call, T in enumerate((1, 3, 2, 4, 4, 1)):
        x = rng.normal(0, 1, (T, 2560)).astype(np.float32)
        if call == 4:
            x[T - 1, 7] = np.nan
        out, ids, w, _ = prod_2560.layer(x, ws=ws)
        n = T - 1 if call == 4 else T  # the finite tokens come first; the checker takes only those
        e_out, e_ids, e_w, _ = orc.moe_layer(ref2560, restate, x[:n], prod_2560.hrouter, prod_2560.hgate, 12,
                                             prod_2560.hup, 12, prod_2560.hdown, 20, shared=prod_2560.shared)
        np.testing.assert_array_equal(ids[:n], e_ids)
        assert_parity(out[:n], e_out, f"product T={T} call {call}")
        assert L.status(ws) == (T - n, n * 10, len(np.unique(e_ids)))
        if n < T:
            assert np.isnan(out[T - 1]).all() and (ids[T - 1] == -1).all()


def test_prefill_product_shape(L, ref2560, restate, prod_2560):
    """Prefill of the production mix: T=2048, N(0,1) logits to top-10."""
    rng = np.random.default_rng(5)
    T = 2048
    logits = rng.normal(0, 1, (T, 512)).astype(np.float32)
    x = rng.normal(0, 1, (T, 2560)).astype(np.float32)
    e_ids, e_w = restate.route(logits)
    out, ws = prod_2560.routed(x, e_ids, e_w)
    assert_parity(out, oracle_routed(ref2560, prod_2560, x, e_ids, e_w), "product prefill T=2048")
    assert L.status(ws) == (0, T * 10, 512)


@pytest.mark.parametrize("T", (1, 2, 3, 4))
def test_layer_small_batch_single_kernel(L, ref2048, restate, q4k_2048, T):
    """Small batches: 1 or 2 tokens run the whole layer in one kernel (router,
    top-10, gate/up, down and combine), 3 and 4 the tensor-core decode path. Ids
    bit-exact, outputs within tolerance, with the shared expert and a routing
    bias, over three calls on one workspace (the single kernel's grid-barrier
    counter carries over). A token with a non-finite input gets a NaN row and is
    counted as invalid."""
    rng = np.random.default_rng(600 + T)
    bias = np.zeros(512, np.float32)
    bias[rng.permutation(512)] = (-1.1 * np.log(np.arange(512) + 1.0)).astype(np.float32)
    ws = L.workspace(T, 2048, 512)
    for call in range(3):
        x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
        if call == 2:
            x[T - 1, 5] = np.nan
        out, ids, w, _ = q4k_2048.layer(x, bias, ws=ws)
        n = T if call < 2 else T - 1  # the finite tokens come first; the checker takes only those
        if n:
            xg = x[:n]
            logits = ref2048.matmul(q4k_2048.hrouter.view(np.uint8), 0, 512, 2048, xg) + bias
            e_out, e_ids, e_w, _ = orc.moe_layer(ref2048, restate, xg, None, q4k_2048.hgate, 12, q4k_2048.hup, 12,
                                                 q4k_2048.hdown, 12, shared=q4k_2048.shared, logits=logits)
            np.testing.assert_array_equal(ids[:n], e_ids)
            assert_parity(out[:n], e_out, f"T={T} call {call}")
        inv, sel, used = L.status(ws)
        assert (inv, sel, used) == (T - n, n * 10, len(np.unique(ids[:n])))
        if call == 2:
            assert np.isnan(out[T - 1]).all() and (ids[T - 1] == -1).all()


def test_layer_zipf_bias(L, ref2048, restate, q4k_2048):
    """Config 3 routing skew: logits + bias, bias[perm[r]] = -1.1*ln(r+1)."""
    rng = np.random.default_rng(3)
    perm = rng.permutation(512)
    bias = np.zeros(512, np.float32)
    bias[perm] = (-1.1 * np.log(np.arange(512) + 1.0)).astype(np.float32)
    x = rng.normal(0, 1, (17, 2048)).astype(np.float32)
    out, ids, w, _ = q4k_2048.layer(x, bias)
    logits = ref2048.matmul(q4k_2048.hrouter.view(np.uint8), 0, 512, 2048, x) + bias
    e_out, e_ids, e_w, _ = orc.moe_layer(ref2048, restate, x, None, q4k_2048.hgate, 12, q4k_2048.hup, 12,
                                         q4k_2048.hdown, 12, shared=q4k_2048.shared, logits=logits)
    np.testing.assert_array_equal(ids, e_ids)
    assert_parity(out, e_out, "zipf layer")
    assert len(np.unique(ids)) < 100  # the skew concentrates routing


def test_layer_graph_capture_matches_eager(L, q4k_2048):
    rng = np.random.default_rng(4)
    T, H, F = 17, 2048, 512
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    eager, _, _, _ = q4k_2048.layer(x)
    dx = L.Device(x)
    out = L.Device(np.zeros((T, H), np.float32))
    ws = L.workspace(T, H, F)
    lay = q4k_2048
    g = C.c_void_p()
    L.call("graph_begin", C.byref(g))
    try:
        L.call("moe_layer", out.p, None, None, dx.p, T, lay.router.p, None, lay.gate.p, 12, lay.up.p, 12,
               lay.down.p, 12, lay.sg.p, 12, lay.su.p, 12, lay.sd.p, 12, lay.sr.p, H, F, ws.p)
        L.call("graph_end", g)
        L.call("graph_launch", g)
        np.testing.assert_array_equal(out.get(), eager)
    finally:
        L.load().qg_graph_destroy(g)


def test_prefill_2048_tokens(L, ref2048, restate, q4k_2048):
    """Config 4: T=2048, logits N(0,1) fed straight to top-10 (about 40 tokens per expert)."""
    rng = np.random.default_rng(3)
    T = 2048
    logits = rng.normal(0, 1, (T, 512)).astype(np.float32)
    x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
    dl = L.Device(logits)
    di, dw = L.Device.empty((T, 10), np.int32), L.Device.empty((T, 10), np.float32)
    L.call("route", di.p, dw.p, dl.p, T)
    ids, w = di.get(), dw.get()
    e_ids, e_w = restate.route(logits)
    np.testing.assert_array_equal(ids, e_ids)
    out, ws = q4k_2048.routed(x, ids, w)
    expected = oracle_routed(ref2048, q4k_2048, x, e_ids, e_w)
    assert_parity(out, expected, "prefill T=2048")
    inv, sel, used = L.status(ws)
    assert (inv, sel, used) == (0, T * 10, 512)
