"""Expert parallelism on two GPUs (one process each): every rank's
qg_moe_layer_ep routing equals the single-GPU qg_moe_layer routing bit for bit
and its output matches within the path's float tolerance (the gate/up tiles
are split along K across SMs and their parts summed in fixed order), over
three calls (both parities of the double-buffered slot rows), with the experts
placed in snake order of a skewed ranking. A verify batch (T=17) returns every
token on every rank; a large batch (T=100) returns each rank's own block of
tokens. Skipped on a machine with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, F = 2048, 512
QROW_H, QROW_F = H // 256 * 144, F // 256 * 144  # Q4_K row bytes


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results, T):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nebula_b200 import ep
        from nebula_b200 import lib as L
        L.load()
        # identical weights and inputs on every rank
        gate, up = L.synth_weights(12, 512 * F, H, 901), L.synth_weights(12, 512 * F, H, 902)
        down = L.synth_weights(12, 512 * H, F, 903)
        router = L.synth_weights(0, 512, H, 904)
        sg, su = L.synth_weights(12, F, H, 905), L.synth_weights(12, F, H, 906)
        sd, sr = L.synth_weights(12, H, F, 907), L.synth_weights(0, 1, H, 908)
        rng = np.random.default_rng(11)
        ranking = rng.permutation(512)
        bias = np.zeros(512, np.float32)
        bias[ranking] = (-1.1 * np.log(np.arange(1, 513))).astype(np.float32)
        dbias = L.Device(bias)
        owner = ep.snake_owner(ranking, world)
        loc, experts = ep.local_map(owner, rank)
        lgate = ep.extract_experts(gate, experts, F, QROW_H)
        lup = ep.extract_experts(up, experts, F, QROW_H)
        ldown = ep.extract_experts(down, experts, H, QROW_F)
        dloc = L.Device(loc)
        grp = ep.EpGroup(T, H, F, rank, world)
        ws = L.workspace(T, H, F)
        errors = []
        for call in range(3):
            x = L.Device(np.random.default_rng(100 + call).normal(0, 1, (T, H)).astype(np.float32))
            ref = L.Device.empty((T, H), np.float32)
            rid = L.Device.empty((T, 10), np.int32)
            L.call("moe_layer", ref.p, rid.p, None, x.p, T, router.p, dbias.p, gate.p, 12, up.p, 12, down.p, 12,
                   sg.p, 12, su.p, 12, sd.p, 12, sr.p, H, F, ws.p)
            out = L.Device.empty((T, H), np.float32)
            eid = L.Device.empty((T, 10), np.int32)
            L.call("moe_layer_ep", out.p, eid.p, None, x.p, T, router.p, dbias.p, lgate.p, 12, lup.p, 12, ldown.p,
                   12, len(experts), dloc.p, sg.p, 12, su.p, 12, sd.p, 12, sr.p, call % world, H, F, rank, world,
                   grp.ptrs)
            a, b = ref.get().astype(np.float64), out.get().astype(np.float64)
            if T > 32:  # this rank's tokens only
                blk = (T + world - 1) // world
                a, b = a[rank * blk:(rank + 1) * blk], b[rank * blk:(rank + 1) * blk]
            if not np.array_equal(rid.get(), eid.get()):
                errors.append(f"call {call}: routing differs")
            r = float(np.linalg.norm(a - b) / np.linalg.norm(a))
            m = float(np.max(np.abs(a - b)))
            if not (np.isfinite(b).all() and r <= 1e-5 and m <= 1e-4 * float(np.max(np.abs(a)))):
                errors.append(f"call {call}: rel-L2 {r:.3e}, max |d| {m:.3e}")
        import ctypes as C
        inv, sel, used = C.c_int(), C.c_int(), C.c_int()
        L.call("moe_status", grp.ws.p, C.byref(inv), C.byref(sel), C.byref(used))
        dist.barrier()
        grp.close()
        results[rank] = "; ".join(errors) if errors else "ok"
    except Exception as e:  # reported to the parent
        results[rank] = f"exception: {e!r}"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", (17, 100, 2048))
def test_expert_parallel_matches_single_gpu(T):
    import torch
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results, T), nprocs=world, start_method="spawn", join=True)
    assert [results.get(r) for r in range(world)] == ["ok"] * world, dict(results)
