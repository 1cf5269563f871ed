"""qg_moe_routed_static (library-owned scratch, no caller workspace) against
qg_moe_routed with a caller workspace, on two calls in a row. Collected last:
the static scratch is set up by whichever call reaches the device first."""
import numpy as np
import pytest

from test_gpu_moe import Layer, random_routes


def _static(L, lay, x, ids, w):
    T = x.shape[0]
    dx, di, dw = L.Device(x), L.Device(ids), L.Device(w)
    out = L.Device.empty((T, lay.H), np.float32)
    L.call("moe_routed_static", out.p, dx.p, di.p, dw.p, T, lay.gate.p, lay.gt, lay.up.p, lay.gt, lay.down.p,
           lay.dt, lay.H, lay.F)
    return out.get()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [17, 5, 28])
def test_static_scratch_matches_workspace_twice(gpu_lib, T):
    from nebula_b200 import lib as L
    lay = Layer(L, 2048, 512, 12, 12, seed=71)
    rng = np.random.default_rng(T)
    for call in range(2):
        x = rng.normal(0, 1, (T, 2048)).astype(np.float32)
        ids, w = random_routes(rng, T)
        ref, _ = lay.routed(x, ids, w)
        got = _static(L, lay, x, ids, w)
        np.testing.assert_array_equal(got, ref, err_msg=f"call {call}")


@pytest.mark.gpu
def test_static_scratch_rejects_oversize(gpu_lib):
    from nebula_b200 import lib as L
    lay = Layer(L, 2048, 512, 12, 12, seed=72, experts=512)
    T = 29  # the first batch size whose workspace exceeds the 8 MiB scratch at 2048 / 512
    dx = L.Device(np.zeros((T, 2048), np.float32))
    di = L.Device(np.zeros((T, 10), np.int32))
    dw = L.Device(np.zeros((T, 10), np.float32))
    out = L.Device.empty((T, 2048), np.float32)
    rc = L.code("moe_routed_static", out.p, dx.p, di.p, dw.p, T, lay.gate.p, 12, lay.up.p, 12, lay.down.p, 12,
                2048, 512)
    assert rc == 1  # cudaErrorInvalidValue
