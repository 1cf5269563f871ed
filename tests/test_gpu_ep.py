"""Expert parallelism on two GPUs (one process each).

* Parity: every rank's qg_moe_layer_ep routing equals the single-GPU
  qg_moe_layer routing bit for bit and its output matches within the path's
  float tolerance (gate/up tiles are split along K across SMs and their parts
  summed in fixed order), over three calls (both parities of the
  double-buffered decode rows), with the experts placed in snake order of a
  skewed ranking. A verify batch (T=17) returns every token on every rank; a
  large batch (T=100, 2048) returns each rank's own block of tokens.
* One workspace, batches of changing size: a workspace sized for 100 tokens
  serves T = 17, 5, 100, 17, 33 in that order (verify batches change size
  from step to step), each call checked against qg_moe_layer.
* A rank that skips a call: rank 1 leaves one call out (it waits on the host,
  with no kernel in flight). Rank 0's combine wait runs out within its bound:
  qg_moe_status reports the timeout and the output rows are NaN. Both ranks
  then zero their workspaces and the next call passes parity again.

Skipped on a machine with fewer than two GPUs. Processes coordinate over gloo;
the kernels use plain peer stores (no multicast) and NCCL is not used.
"""
import ctypes as C
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, F = 2048, 512
TIMEOUT = 702  # cudaErrorLaunchTimeout, as qg_moe_status reports a bounded wait that ran out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Rank:
    """One rank's layer: full weights (for the single-GPU reference) and its own experts.
    Q4_K gate/up; down (and the shared down) Q4_K or IQ4_NL (dt = 20)."""

    def __init__(self, L, ep, rank, world, h=H, f=F, dt=12):
        self.L, self.rank, self.world, self.h, self.f, self.dt = L, rank, world, h, f, dt
        self.gate, self.up = L.synth_weights(12, 512 * f, h, 901), L.synth_weights(12, 512 * f, h, 902)
        self.down = L.synth_weights(dt, 512 * h, f, 903)
        self.router = L.synth_weights(0, 512, h, 904)
        self.sg, self.su = L.synth_weights(12, f, h, 905), L.synth_weights(12, f, h, 906)
        self.sd, self.sr = L.synth_weights(dt, h, f, 907), L.synth_weights(0, 1, h, 908)
        ranking = np.random.default_rng(11).permutation(512)
        bias = np.zeros(512, np.float32)
        bias[ranking] = (-1.1 * np.log(np.arange(1, 513))).astype(np.float32)
        self.bias = L.Device(bias)
        owner = ep.snake_owner(ranking, world)
        loc, experts = ep.local_map(owner, rank)
        self.n_local = len(experts)
        self.lgate = ep.extract_experts(self.gate, experts, f, L.row_bytes(12, h))
        self.lup = ep.extract_experts(self.up, experts, f, L.row_bytes(12, h))
        self.ldown = ep.extract_experts(self.down, experts, h, L.row_bytes(dt, f))
        self.loc = L.Device(loc)

    def single(self, x, T, ws):
        L, dt = self.L, self.dt
        ref = L.Device.empty((T, self.h), np.float32)
        rid = L.Device.empty((T, 10), np.int32)
        L.call("moe_layer", ref.p, rid.p, None, x.p, T, self.router.p, self.bias.p, self.gate.p, 12, self.up.p, 12,
               self.down.p, dt, self.sg.p, 12, self.su.p, 12, self.sd.p, dt, self.sr.p, self.h, self.f, ws.p)
        return ref.get(), rid.get()

    def ep_call(self, x, T, grp, shared_rank):
        L, dt = self.L, self.dt
        out = L.Device.empty((T, self.h), np.float32)
        eid = L.Device.empty((T, 10), np.int32)
        L.call("moe_layer_ep", out.p, eid.p, None, x.p, T, self.router.p, self.bias.p, self.lgate.p, 12, self.lup.p,
               12, self.ldown.p, dt, self.n_local, self.loc.p, self.sg.p, 12, self.su.p, 12, self.sd.p, dt,
               self.sr.p, shared_rank, self.h, self.f, self.rank, self.world, grp.ptrs)
        return out, eid

    def check(self, x, T, grp, ws, call, shared_rank):
        """One expert-parallel call against qg_moe_layer; a list of problems."""
        ref, rid = self.single(x, T, ws)
        out, eid = self.ep_call(x, T, grp, shared_rank)
        a, b = ref.astype(np.float64), out.get().astype(np.float64)
        if T > 32:  # this rank's tokens only
            blk = (T + self.world - 1) // self.world
            a, b = a[self.rank * blk:(self.rank + 1) * blk], b[self.rank * blk:(self.rank + 1) * blk]
        errors = []
        if not np.array_equal(rid, eid.get()):
            errors.append(f"call {call} (T={T}): routing differs")
        if b.size:
            r = float(np.linalg.norm(a - b) / np.linalg.norm(a))
            m = float(np.max(np.abs(a - b)))
            if not (np.isfinite(b).all() and r <= 1e-5 and m <= 1e-4 * float(np.max(np.abs(a)))):
                errors.append(f"call {call} (T={T}): rel-L2 {r:.3e}, max |d| {m:.3e}")
        return errors


def _x(T, seed, h=H):
    from nebula_b200 import lib as L
    return L.Device(np.random.default_rng(seed).normal(0, 1, (T, h)).astype(np.float32))


def _status(L, ws):
    inv, sel, used = C.c_int(), C.c_int(), C.c_int()
    return L.code("moe_status", ws.p, C.byref(inv), C.byref(sel), C.byref(used))


def _worker(rank, world, port, results, scenario, T):
    import torch
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nebula_b200 import ep
        from nebula_b200 import lib as L
        L.load()
        errors = []
        if scenario == "product":  # Nebula's mix: Q4_K gate/up, IQ4_NL down, 2560/640
            lay = _Rank(L, ep, rank, world, 2560, 640, 20)
            grp = ep.EpGroup(T, 2560, 640, rank, world)
            ws = L.workspace(T, 2560, 640)
            for call in range(3):
                errors += lay.check(_x(T, 400 + call, 2560), T, grp, ws, call, call % world)
        else:
            lay = _Rank(L, ep, rank, world)
        if scenario == "parity":
            grp = ep.EpGroup(T, H, F, rank, world)
            ws = L.workspace(T, H, F)
            for call in range(3):
                errors += lay.check(_x(T, 100 + call), T, grp, ws, call, call % world)
        elif scenario == "sizes":
            sizes = (17, 5, 100, 17, 33)
            grp = ep.EpGroup(max(sizes), H, F, rank, world)
            ws = L.workspace(max(sizes), H, F)
            for call, t in enumerate(sizes):
                errors += lay.check(_x(t, 200 + call), t, grp, ws, call, call % world)
        elif scenario == "skip":
            grp = ep.EpGroup(T, H, F, rank, world)
            ws = L.workspace(T, H, F)
            errors += lay.check(_x(T, 300), T, grp, ws, 0, 0)
            dist.barrier()
            if rank == 0:  # rank 1 sits this call out
                t0 = time.monotonic()
                out, _ = lay.ep_call(_x(T, 301), T, grp, 0)
                code = _status(L, grp.ws)
                waited = time.monotonic() - t0
                rows = out.get()
                if code != TIMEOUT:
                    errors.append(f"skipped peer: qg_moe_status returned {code}, expected {TIMEOUT}")
                if not np.isnan(rows).all():
                    errors.append("skipped peer: output rows are not NaN")
                if waited > 30:
                    errors.append(f"skipped peer: the call took {waited:.1f} s")
            dist.barrier()
            # recovery: both ranks zero their workspaces, then carry on
            L.call("zero", grp.ws.p, grp.ws.nbytes)
            L.call("sync")
            dist.barrier()
            errors += lay.check(_x(T, 302), T, grp, ws, 2, 1)
        _status(L, grp.ws)
        dist.barrier()
        grp.close()
        results[rank] = "; ".join(errors) if errors else "ok"
    except Exception as e:  # reported to the parent
        results[rank] = f"exception: {e!r}"
    finally:
        dist.destroy_process_group()


def _run(scenario, T):
    import torch
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results, scenario, T), nprocs=world,
                       start_method="spawn", join=True)
    assert [results.get(r) for r in range(world)] == ["ok"] * world, dict(results)


@pytest.mark.parametrize("T", (17, 100, 2048))
def test_expert_parallel_matches_single_gpu(T):
    _run("parity", T)


@pytest.mark.parametrize("T", (17, 100))
def test_expert_parallel_product_mix(T):
    """Q4_K gate/up with IQ4_NL down at hidden 2560 / ffn 640, decode and large batches."""
    _run("product", T)


def test_expert_parallel_one_workspace_changing_sizes():
    _run("sizes", 0)


def test_expert_parallel_skipped_call_times_out_then_recovers():
    _run("skip", 17)
