"""Host-side arithmetic of bench.py (no GPU): the byte counts behind every
roofline figure, the parity bar, the routing skew and the committed traffic
ratios it reads.

Expert sizes follow the reference's row sizes (qwen/cpu.c:22-24: Q4_K 144 bytes
per 256 values, IQ4_NL 18 bytes per 32) and its production mix (qwen/README.md:
Q4_K gate/up, IQ4_NL down)."""
import numpy as np
import pytest

import bench


def test_row_and_expert_bytes():
    assert bench.row_bytes(bench.Q4K, 2048) == 8 * 144
    assert bench.row_bytes(bench.IQ4NL, 640) == 20 * 18
    assert bench.row_bytes(0, 2560) == 2560 * 4
    # hidden 2048 / ffn 512: gate + up rows of 2048 values, down rows of 512
    assert bench.expert_bytes(2048, 512, bench.Q4K, bench.Q4K) == 1_769_472 == bench.EXPERT_BYTES
    assert bench.expert_bytes(2048, 512, bench.IQ4NL, bench.IQ4NL) == 1_769_472
    # Nebula's mix: Q4_K gate/up rows of 1,440 bytes, IQ4_NL down rows of 360
    assert bench.expert_bytes(2560, 640, bench.Q4K, bench.IQ4NL) == 2 * 640 * 1440 + 2560 * 360 == 2_764_800


@pytest.mark.parametrize("h,eb,U,T,weights", [
    (2560, 2_764_800, 10, 1, 35_665_920),   # single-kernel layer, one token
    (2560, 2_764_800, 38, 4, 113_080_320),  # four tokens, 38 distinct experts
    (2048, 1_769_472, 10, 1, 23_666_688),
])
def test_layer_bytes_match_the_profiled_weights(h, eb, U, T, weights):
    """layer_bytes = the used experts, the shared expert, the router with the
    shared-gate row (the weights the ncu summaries count), x in and out, and the
    routing output."""
    lb = bench.layer_bytes(U, T, eb, h, True)
    assert lb - 2 * T * h * 4 - T * bench.K * 8 == weights
    assert bench.layer_bytes(U, T, eb, h, False) == lb - eb - h * 4


def test_parity_bar():
    rng = np.random.default_rng(0)
    ref = rng.normal(0, 1, (4, 64)).astype(np.float32)
    ids = rng.integers(0, 512, (4, 10)).astype(np.int32)
    ok = bench.parity(ref.copy(), ref, ids.copy(), ids)
    assert ok["pass"] and ok["bitwise_equal"] and ok["ids_bitexact"]
    near = ref * np.float32(1 + 1e-7)
    r = bench.parity(near, ref)
    assert r["pass"] and not r["bitwise_equal"] and r["rel_l2"] < 1e-6
    far = ref.copy()
    far[0, 0] += np.float32(1e-2 * np.abs(ref).max())
    assert not bench.parity(far, ref)["pass"]  # max-abs above 1e-4 x max|ref|
    nan = ref.copy()
    nan[1, 3] = np.nan
    assert not bench.parity(nan, ref)["pass"]
    bad_ids = ids.copy()
    bad_ids[2, 5] = (bad_ids[2, 5] + 1) % 512
    r = bench.parity(ref, ref, bad_ids, ids)
    assert not r["pass"] and not r["ids_bitexact"]


def test_zipf_bias_is_the_reference_skew():
    """bias[ranking[r]] = -1.1 ln(r + 1): every expert gets one rank, the hottest 0."""
    for layer in (0, 47):
        rank = bench.ranking(layer)
        assert sorted(rank.tolist()) == list(range(512))
        b = bench.zipf_bias(layer)
        assert b[rank[0]] == 0.0
        np.testing.assert_allclose(b[rank], -1.1 * np.log(np.arange(512) + 1.0), rtol=1e-6)
        assert np.all(np.diff(b[rank]) < 0)


@pytest.mark.parametrize("kernel,workload", [
    ("tc_experts_kernel<24>", "T17"),
    ("tc_experts_kernel<24,1,1>", "config2-T17"),
    ("tc_experts_kernel<24,1,0>", "product-T17"),
])
def test_traffic_ratios_for_every_bench_line(kernel, workload):
    """Every decode line bench.py prints has a committed ncu traffic ratio, and
    the weights are read about once (within 10 %)."""
    traffic, source = bench.traffic_per_launch(kernel, workload, 1e8)
    assert traffic is not None and "ncu" in source
    assert 1e8 <= traffic < 1.1e8


def test_workload_config_names_the_stack():
    c = bench.workload_config(17, 48, 1)
    assert c["tokens"] == 17 and c["layers"] == 48 and c["parallelism"] == "single"
    assert bench.workload_config(17, 48, 8)["parallelism"] == "ep8"
