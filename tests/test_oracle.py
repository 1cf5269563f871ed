"""Pins the CPU checker (oracle/) before any GPU result is compared with it.

* The reference CPU MoE compiled into oracle/_ref reproduces the golden
  fixtures made by running the reference here (tests/golden/make_golden.py):
  reference NumPy decoder values, qc_matmul outputs, qc_moe digests.
* Its ISA variants agree bitwise, as the reference's own
  qwen/test_cpu_dispatch.py:46-92 requires, including the duplicate-id
  rejection and every fp16 encoding.
* The C restatements of the device routing steps meet the expectations the
  reference's GPU tests state (qwen/test_gpu.py:84-95, 338-346, 352-359,
  361-384).
"""
import hashlib

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.blocks import dequant64, random_blocks
import make_golden as mg

GOLDEN = mg.OUT


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def formats():
    return np.load(GOLDEN / "formats.npz")


@pytest.mark.parametrize("typ", mg.TYPES)
def test_weight_at_matches_reference_numpy_decoder(ref2048, formats, typ):
    packed = formats[f"packed_{typ}"]
    values = formats[f"values_{typ}"]
    rows, cols = values.shape
    rb = packed.shape[1]
    out = np.array([[ref2048.lib.qc_weight_at(packed[r].ctypes.data, typ, i) for i in range(cols)]
                    for r in range(rows)], np.float32)
    np.testing.assert_allclose(out, values, rtol=1e-6, atol=1e-7, err_msg=f"type {typ}")
    assert rb == ref2048.row_bytes(typ, cols)


@pytest.mark.parametrize("typ", (0, 12, 20))
def test_float64_expansion_matches_reference_numpy_decoder(formats, typ):
    packed, values = formats[f"packed_{typ}"], formats[f"values_{typ}"]
    rows, cols = values.shape
    np.testing.assert_allclose(dequant64(packed, typ, rows, cols), values, rtol=1e-6, atol=1e-8)


@pytest.mark.parametrize("typ", (0, 12, 20))
@pytest.mark.parametrize("shape", mg.MATMUL_SHAPES)
def test_qc_matmul_golden(ref2048, typ, shape):
    gold = np.load(GOLDEN / "matmul.npz")
    rows, cols = shape
    w, xs = mg.matmul_case_inputs(typ, rows, cols)
    assert digest(w, *xs) == str(gold[f"sha_{typ}_{cols}"]), "regenerated inputs drifted"
    for nt, x in zip(mg.MATMUL_TOKENS, xs):
        out = ref2048.matmul(w, typ, rows, cols, x, threads=2)
        np.testing.assert_array_equal(out, gold[f"out_{typ}_{cols}_{nt}"])
        # and against an independent float64 expansion
        ref = x.astype(np.float64) @ dequant64(w, typ, rows, cols).T
        np.testing.assert_allclose(out, ref, rtol=4e-5, atol=8e-5)


@pytest.mark.parametrize("case", mg.MOE_CASES, ids=lambda c: f"{c[0]}x{c[1]}_t{c[2]}_{c[3]}")
def test_qc_moe_golden(case):
    hidden, ffn, gt, dt, seed = case
    ref = orc.RefCPU(hidden, ffn)
    gold = np.load(GOLDEN / "moe.npz")
    gate, up, down, x, ids, w = mg.moe_case_inputs(*case)
    key = f"{hidden}_{ffn}_{gt}_{dt}"
    assert digest(gate, up, down, x, ids, w) == str(gold[f"sha_{key}"])
    for nt in mg.MOE_TOKENS:
        out = ref.moe(x[:nt], ids[:nt], w[:nt], gate, gt, up, gt, down, dt, threads=2)
        np.testing.assert_array_equal(out[0], gold[f"row0_{key}_{nt}"])
        assert digest(out) == str(gold[f"outsha_{key}_{nt}"]), f"nt={nt}"


def test_isa_variants_bit_exact(ref2048):
    """qwen/test_cpu_dispatch.py:44-58 on the variants this host supports."""
    lib = ref2048.lib
    variants = [p for n, p in (("scalar", "qcs_"), ("avx2", "qc2_"), ("avx512", "qc5_"))
                if lib.qc_backend_available(n.encode())]
    assert "qcs_" in variants
    import ctypes as C
    rng = np.random.default_rng(91011)
    for typ in (0, 1, 30, 2, 20, 6, 7, 8, 12, 13, 14):
        w = random_blocks(rng, typ, 7, 512)
        for nt in (1, 3, 4, 5, 17, 18):
            x = rng.normal(0, .2, (nt, 512)).astype("f4")
            expected = None
            for prefix in variants:
                fn = getattr(lib, prefix + "matmul")
                fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
                out = np.empty((nt, 7), "f4")
                assert fn(out.ctypes.data, w.ctypes.data, typ, 7, 512, x.ctypes.data, nt, 2) == 0
                if expected is None:
                    expected = out
                else:
                    np.testing.assert_array_equal(out, expected, err_msg=f"{prefix} type {typ} nt {nt}")


def test_all_half_encodings(ref2048):
    """qwen/test_cpu_dispatch.py:59-68."""
    import ctypes as C
    halves = np.arange(65536, dtype="u2")
    fn = ref2048.lib.qc_weight_at
    observed = np.array([fn(halves.ctypes.data, 1, i) for i in range(0, 65536, 7)], "f4")
    with np.errstate(invalid="ignore"):
        expected = halves[::7].view("f2").astype("f4")
    np.testing.assert_array_equal(observed, expected)


def test_qc_moe_rejects_duplicate_ids(ref2560):
    """qwen/test_cpu_dispatch.py:88-90: a repeated id makes qc_moe fail."""
    rng = np.random.default_rng(3)
    gate = random_blocks(rng, 12, 2 * 640, 2560)
    down = random_blocks(rng, 20, 2 * 2560, 640)
    x = rng.normal(0, .05, (5, 2560)).astype("f4")
    ids = np.full((5, 10), -2, np.int32)
    ids[:, 0], ids[:, 1] = 0, 1
    w = np.zeros((5, 10), np.float32)
    w[:, 0], w[:, 1] = .6, .3
    assert ref2560.moe(x, ids, w, gate, 12, gate, 12, down, 20, threads=2, check=False) == 0
    ids[0, 1] = 0
    assert ref2560.moe(x, ids, w, gate, 12, gate, 12, down, 20, threads=2, check=False) == -1


def test_route_restatement(restate):
    """qwen/test_gpu.py:338-346: ids == stable argsort of -logits, softmax over the ten, NaN -> -1."""
    rng = np.random.default_rng(812603)
    logits = (rng.normal(size=(6, 512)) * 0.2).astype(np.float32)
    logits[0] = 0
    logits[2, ::7] = 0.5  # ties among the top values
    ids, w = restate.route(logits)
    sel = np.argsort(-logits, axis=1, kind="stable")[:, :10]
    np.testing.assert_array_equal(ids, sel)
    vals = np.take_along_axis(logits, sel, axis=1).astype(np.float64)
    p = np.exp(vals - vals.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    np.testing.assert_allclose(w, p, rtol=2e-6, atol=1e-7)
    logits[1, 7] = np.nan
    logits[3, 100] = np.inf
    ids, w = restate.route(logits)
    assert (ids[1] == -1).all() and (w[1] == 0).all()
    assert (ids[3] == -1).all()


def test_prune_restatement_known_answer(restate):
    """qwen/test_gpu.py:84-95 known-answer case."""
    ids = np.tile(np.arange(10, dtype=np.int32), (5, 1))
    weights = np.full((5, 10), .1, np.float32)
    resident = np.zeros(512, np.uint8)
    resident[:8] = 1
    weights[0, 8:] = .04
    weights[1, 8:] = .05
    weights[2, 8:] = .06
    weights[3, 8:] = 0
    weights[4, 8:] = [.01, .10]
    rc, out_ids, out_w, st = restate.prune(ids, weights, resident, 0.10)
    assert rc == 0
    assert np.all(out_ids[[0, 3], 8:] <= -2)
    np.testing.assert_array_equal(out_ids[[1, 2, 4]], ids[[1, 2, 4]])
    np.testing.assert_array_equal(out_w[:, :8], weights[:, :8])
    assert (st.token_layers, st.missing_selections, st.skipped_selections, st.avoided_token_handoffs) == (5, 10, 4, 2)
    assert restate.prune(ids, weights, resident, 0.2)[0] != 0  # threshold must be <= 0.1


def test_map_restatement(restate):
    """qwen/test_gpu.py:352-359."""
    rng = np.random.default_rng(5)
    for nt in (1, 17, 511, 513):
        ids = np.stack([rng.choice(512, 10, replace=False) for _ in range(nt)]).astype(np.int32)
        m, counts = restate.moe_map(ids)
        for e in range(0, 512, 7):
            expected = np.flatnonzero((ids == e).any(1))
            assert counts[e] == len(expected)
            np.testing.assert_array_equal(m[e, :len(expected)], expected)


def test_reduce_restatement_is_rank_ordered(restate):
    rng = np.random.default_rng(9)
    slots = rng.normal(size=(3, 10, 64)).astype(np.float32) * 1e3
    out = restate.moe_reduce(slots)
    expected = np.zeros((3, 64), np.float32)
    for k in range(10):
        expected = expected + slots[:, k]
    np.testing.assert_array_equal(out, expected)


def test_moe_layer_oracle_matches_float64(ref2048, restate):
    """The composed CPU layer (router + routing + qc_moe + shared expert) against a float64 NumPy model."""
    rng = np.random.default_rng(11)
    H, F, E = 2048, 512, 16
    router = np.zeros((512, H), np.float32)
    router[:E] = rng.normal(0, .02, (E, H))
    router[E:] = -1.0  # experts >= E are never selected for x > 0 ... keep logits low
    x = np.abs(rng.normal(0, 1, (3, H))).astype(np.float32)
    gate = random_blocks(rng, 12, E * F, H, d=0.0002, dmin=0.0001)
    up = random_blocks(rng, 12, E * F, H, d=0.0002, dmin=0.0001)
    down = random_blocks(rng, 12, E * H, F, d=0.0002, dmin=0.0001)
    sg = random_blocks(rng, 12, F, H, d=0.0002, dmin=0.0001)
    su = random_blocks(rng, 12, F, H, d=0.0002, dmin=0.0001)
    sd = random_blocks(rng, 12, H, F, d=0.0002, dmin=0.0001)
    sr = rng.normal(0, .02, (1, H)).astype(np.float32)
    # pad expert arrays to 512 experts' worth of rows only where selected: ids are < E by construction
    out, ids, w, logits = orc.moe_layer(ref2048, restate, x, router, gate, 12, up, 12, down, 12,
                                        shared=(sg, 12, su, 12, sd, 12, sr), threads=2)
    assert (ids < E).all() and (ids >= 0).all()
    G = dequant64(gate, 12, E * F, H).reshape(E, F, H)
    U = dequant64(up, 12, E * F, H).reshape(E, F, H)
    Dn = dequant64(down, 12, E * H, F).reshape(E, H, F)
    sig = lambda v: 1 / (1 + np.exp(-v))
    x64 = x.astype(np.float64)
    exp = np.zeros((3, H))
    for t in range(3):
        for k in range(10):
            e = ids[t, k]
            g, u = G[e] @ x64[t], U[e] @ x64[t]
            exp[t] += w[t, k] * (Dn[e] @ ((g * sig(g)) * u))
    g = dequant64(sg, 12, F, H) @ x64.T
    u = dequant64(su, 12, F, H) @ x64.T
    sh = (dequant64(sd, 12, H, F) @ ((g * sig(g)) * u)).T
    exp += sh * sig(x64 @ sr[0].astype(np.float64))[:, None]
    np.testing.assert_allclose(out, exp, rtol=2e-4, atol=2e-4 * np.abs(exp).max())
