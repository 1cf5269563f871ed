#!/usr/bin/env python3
"""Benchmark of the routed-MoE hot path (one JSON line on rank 0).

Workload (BASELINE configs 3/5): a 48-layer stack of routed-MoE layers at
hidden 2048 / FFN 512, 512 Q4_K experts per layer (43.5 GB resident) plus a
Q4_K shared expert with its sigmoid gate, router F32 [512x2048] N(0,0.02),
Zipf-skewed routing (logit bias[perm_l[r]] = -1.1*ln(r+1), perm_l a seeded
permutation per layer), x_l ~ N(0,1) independent per layer (no residual: the
attention between layers is out of scope). One step = one speculative-verify
batch of T=17 tokens through all 48 layers (router GEMV, top-10, experts,
combine, shared expert), captured in one CUDA graph and replayed.

The stack's weights (43.5 GB) are far larger than L2 (126 MB), so every step
streams its experts from HBM; no flush is needed.

Extra keys: `prefill` (config 4: one layer, T=2048, N(0,1) logits fed to
top-10; one GPU), `prefill_ep` (config 5's prefill: one layer, T=2048 through
the router with the Zipf bias and the shared expert; expert parallel at N>1,
where rank r returns its 1/N of the tokens), `roofline` (dominant kernel vs measured HBM copy bandwidth),
`cpu_baseline` (the reference's own CPU MoE on this host's cores), `e2e`
(the same metric through the C ABI with pinned host buffers copied in and
results read back every step).

Multi-GPU: launched by torch.distributed.run, one process
per GPU, expert parallel. Every rank holds 1/N of each layer's experts (snake
order of the layer's hot-expert ranking) plus the replicated router and shared
expert, and all ranks run the same T tokens (strong scaling): each computes its
experts' rows, stores them into every rank's workspace over NVLink and reduces.
The value is T tokens per step divided by the slowest rank's step time.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, F, E, K = 2048, 512, 512, 10
Q4K = 12
EXPERT_BYTES = 3 * 589_824  # gate + up + down of one expert, Q4_K, 2048/512
ROUTER_BYTES = 512 * H * 4
SHARED_GATE_BYTES = H * 4


def zipf_bias(layer: int) -> np.ndarray:
    perm = np.random.default_rng(1000 + layer).permutation(E)
    bias = np.zeros(E, np.float32)
    bias[perm] = (-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    return bias


def layer_bytes(U: int, T: int) -> int:
    """Algorithmic HBM bytes of one layer: U experts + router + shared expert + x in/out + routing."""
    return U * EXPERT_BYTES + ROUTER_BYTES + EXPERT_BYTES + SHARED_GATE_BYTES + 2 * T * H * 4 + T * K * 8


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def pci_bus_id(torch, index: int) -> str | None:
    """NVML's PCI bus id of CUDA device `index` (CUDA and NVML may number GPUs differently)."""
    try:
        pr = torch.cuda.get_device_properties(index)
        return f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
    except (AttributeError, RuntimeError):
        return None


class Clocks:
    """SM clock and throttle-reason sampling during the timed region.

    NVML is polled from a thread every 5 ms (a timed region of a few steps is
    shorter than nvidia-smi's own sampling period); the samples are also
    written as CSV next to the other run outputs. Reading only: no setting of
    the GPU is changed."""
    REASONS = (("hw_slowdown", 8), ("hw_thermal_slowdown", 64), ("sw_thermal_slowdown", 32),
               ("sw_power_cap", 4))

    def __init__(self, index: int, pci_bus_id: str | None = None):
        self.index, self.pci = index, pci_bus_id
        self.samples: list[tuple[float, float, float, int]] = []
        self.max_mhz = None
        self.path = ROOT / "gpurun_out" / f"clocks_rank{index}.csv"
        self.thread = None
        self.stop = None

    def _handle(self, nv):
        if self.pci:
            try:
                return nv.nvmlDeviceGetHandleByPciBusId(self.pci)
            except nv.NVMLError:
                pass
        return nv.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:  # no NVML: the summary says so
            return self
        self.stop = threading.Event()

        def poll():
            t0 = time.perf_counter()
            while not self.stop.is_set():
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    why = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                    watts = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                except Exception:
                    break
                self.samples.append((time.perf_counter() - t0, mhz, watts, why))
                self.stop.wait(0.005)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.thread:
            self.stop.set()
            self.thread.join(5)
            try:
                self.path.parent.mkdir(exist_ok=True)
                with open(self.path, "w") as f:
                    f.write("t_s,sm_mhz,sm_max_mhz,power_w,reasons_mask\n")
                    for t, mhz, w, why in self.samples:
                        f.write(f"{t:.4f},{mhz:.0f},{self.max_mhz:.0f},{w:.1f},{why:#x}\n")
            except OSError:
                pass

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        reasons = sorted({name for _, _, _, why in self.samples for name, bit in self.REASONS if why & bit})
        return {"sm_mhz": float(np.median([s[1] for s in self.samples])), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "source": "NVML, 5 ms period"}


class Stack:
    """48 resident layers on the device plus per-layer inputs and outputs.

    With ``ep=(rank, world)`` the rank keeps only its share of each layer's
    experts (snake order of the layer's hot-expert ranking) and runs the
    expert-parallel layer; weights and inputs are the same on every rank."""

    def __init__(self, L, layers: int, T: int, seed0: int = 0, ep=None):
        self.L, self.T, self.layers, self.ep = L, T, layers, ep
        self.w = []
        if ep:
            from nebula_b200 import ep as epm
            rank, world = ep
            self.epg = epm.EpGroup(T, H, F, rank, world)
        for l in range(layers):
            s = seed0 + 100 * l
            d = {"router": L.synth_weights(0, E, H, s + 4)}
            if ep:
                owner = epm.snake_owner(np.random.default_rng(1000 + l).permutation(E), world)
                loc, experts = epm.local_map(owner, rank)
                for name, rows, cols, seed in (("gate", F, H, s + 1), ("up", F, H, s + 2), ("down", H, F, s + 3)):
                    full = L.synth_weights(Q4K, E * rows, cols, seed)
                    d[name] = epm.extract_experts(full, experts, rows, cols // 256 * 144)
                    full.free()
                d["local"], d["experts"], d["n_local"] = L.Device(loc), set(experts), len(experts)
            else:
                d.update({"gate": L.synth_weights(Q4K, E * F, H, s + 1), "up": L.synth_weights(Q4K, E * F, H, s + 2),
                          "down": L.synth_weights(Q4K, E * H, F, s + 3)})
            d.update({
                "sg": L.synth_weights(Q4K, F, H, s + 5), "su": L.synth_weights(Q4K, F, H, s + 6),
                "sd": L.synth_weights(Q4K, H, F, s + 7), "sr": L.synth_weights(0, 1, H, s + 8),
                "bias": L.Device(zipf_bias(l)),
                "x": L.synth_normal(T * H, 2 + l + 7919 * seed0),
                "out": L.Device.empty((T, H), np.float32),
                "ids": L.Device.empty((T, K), np.int32), "wts": L.Device.empty((T, K), np.float32),
            })
            self.w.append(d)
        self.ws = self.epg.ws if ep else L.workspace(T, H, F)

    def run_layer(self, l: int, x_ptr=None, out_ptr=None):
        d, L = self.w[l], self.L
        if self.ep:
            rank, world = self.ep
            L.call("moe_layer_ep", out_ptr or d["out"].p, d["ids"].p, d["wts"].p, x_ptr or d["x"].p, self.T,
                   d["router"].p, d["bias"].p, d["gate"].p, Q4K, d["up"].p, Q4K, d["down"].p, Q4K, d["n_local"],
                   d["local"].p, d["sg"].p, Q4K, d["su"].p, Q4K, d["sd"].p, Q4K, d["sr"].p, l % world, H, F, rank,
                   world, self.epg.ptrs)
            return
        L.call("moe_layer", out_ptr or d["out"].p, d["ids"].p, d["wts"].p, x_ptr or d["x"].p, self.T,
               d["router"].p, d["bias"].p, d["gate"].p, Q4K, d["up"].p, Q4K, d["down"].p, Q4K,
               d["sg"].p, Q4K, d["su"].p, Q4K, d["sd"].p, Q4K, d["sr"].p, H, F, self.ws.p)

    def step(self):
        for l in range(self.layers):
            self.run_layer(l)

    def capture(self):
        import ctypes as C
        g = C.c_void_p()
        self.L.call("graph_begin", C.byref(g))
        try:
            self.step()
        except Exception:
            self.L.load().qg_graph_destroy(g)
            raise
        self.L.call("graph_end", g)
        return g

    def experts_used(self) -> list[int]:
        """Experts this rank computed per layer (its share under expert parallelism)."""
        out = []
        for d in self.w:
            u = set(np.unique(d["ids"].get()).tolist()) - {-1}
            out.append(len(u & d["experts"]) if self.ep else len(u))
        return out


def cpu_reference_sample(L, stack: Stack | None, T: int, layers_sample: int, seconds: float, threads: int):
    """Times the reference CPU MoE layer (qc_matmul router + route + qc_moe + shared expert)."""
    from oracle import oracle as orc
    ref, rs = orc.RefCPU(H, F), orc.Restate()
    data = []
    for l in range(layers_sample):
        if stack is not None:
            d = stack.w[l]
            data.append(dict(x=d["x"].get().reshape(T, H), router=d["router"].get().view(np.float32).reshape(E, H),
                             gate=d["gate"].get(), up=d["up"].get(), down=d["down"].get(),
                             shared=(d["sg"].get(), Q4K, d["su"].get(), Q4K, d["sd"].get(), Q4K,
                                     d["sr"].get().view(np.float32).reshape(1, H)), bias=zipf_bias(l)))
        else:
            from oracle.blocks import random_blocks
            rng = np.random.default_rng(l)
            data.append(dict(x=rng.normal(0, 1, (T, H)).astype(np.float32),
                             router=rng.normal(0, .02, (E, H)).astype(np.float32),
                             gate=random_blocks(rng, Q4K, E * F, H, .0002, .0001),
                             up=random_blocks(rng, Q4K, E * F, H, .0002, .0001),
                             down=random_blocks(rng, Q4K, E * H, F, .0002, .0001),
                             shared=(random_blocks(rng, Q4K, F, H, .0002, .0001), Q4K,
                                     random_blocks(rng, Q4K, F, H, .0002, .0001), Q4K,
                                     random_blocks(rng, Q4K, H, F, .0002, .0001), Q4K,
                                     rng.normal(0, .02, (1, H)).astype(np.float32)), bias=zipf_bias(l)))

    def one(d):
        logits = ref.matmul(d["router"], 0, E, H, d["x"], threads) + d["bias"]
        return orc.moe_layer(ref, rs, d["x"], None, d["gate"], Q4K, d["up"], Q4K, d["down"], Q4K,
                             shared=d["shared"], logits=logits, threads=threads)

    one(data[0])  # warm-up
    times, n = [], 0
    t_end = time.perf_counter() + seconds
    while True:
        d = data[n % len(data)]
        t0 = time.perf_counter()
        one(d)
        times.append(time.perf_counter() - t0)
        n += 1
        if time.perf_counter() > t_end and n >= 3:
            break
    per_layer = float(np.median(times))
    return {"per_layer_s": per_layer, "layers_timed": n, "backend": ref.backend()}


def run_reference_arm(args, rank: int, world: int) -> None:
    """bench.py --impl reference: the reference's CPU MoE path on this host's cores."""
    if rank != 0:
        return
    from oracle import oracle as orc
    threads = orc.host_threads()
    T = args.tokens
    per_step = []
    res = None
    for _ in range(args.warmup + args.steps):
        res = cpu_reference_sample(None, None, T, 2, args.cpu_seconds / max(1, args.steps), threads)
        per_step.append(res["per_layer_s"])
    t_layer = float(np.median(per_step[args.warmup:]))
    value = T / (t_layer * args.layers)
    line = {
        "impl": "reference", "metric": "moe_verify_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_layer * args.layers * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"48-layer routed-MoE stack, T={T} verify, H=2048 F=512 E=512 top-10, Q4_K, "
                               "shared expert, Zipf routing", "layers": args.layers, "tokens": T},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"{res['layers_timed']} layer evaluations per step over 2 distinct layers "
                                   f"(median per layer x {args.layers}); qc_moe backend {res['backend']}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--tokens", type=int, default=17)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    from nebula_b200 import lib as L
    L.load()
    T = args.tokens
    ep_mode = world > 1
    stack = Stack(L, args.layers, T, seed0=0, ep=(rank, world) if ep_mode else None)
    L.call("sync")
    graph = stack.capture()

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        L.call("graph_launch", graph)
    barrier()
    used = stack.experts_used()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local, pci_bus_id(torch, local)) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            L.call("graph_launch", graph)
        stop.record()
        barrier()
    ms = start.elapsed_time(stop)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)  # every rank works on the same T tokens

    # roofline: per-phase event timing over an eager replay of the same steps
    L.call("moe_profile", 1)
    for _ in range(args.steps):
        stack.step()
    phases = ("router", "route", "plan", "gate_up", "down", "combine", "experts", "decode_router")
    prof = {}
    import ctypes as C
    for i, name in enumerate(phases):
        tot, n = C.c_double(0), C.c_int(0)
        L.call("moe_profile_read", i, C.byref(tot), C.byref(n))
        prof[name] = (tot.value, n.value)
    L.call("moe_profile", 0)
    peaks = measured_peaks()
    # algorithmic bytes per launch: every used expert's gate/up/down rows (+ the
    # shared expert) read once, x read, out written; router: its matrix and x
    u_mean = float(np.mean(used))
    shared_share = 1.0 / world  # the shared expert runs on one rank per layer
    alg_bytes = {"experts": (u_mean + shared_share) * EXPERT_BYTES + 2 * T * H * 4,
                 "decode_router": (E + 1) * H * 4 + T * H * 4 + T * K * 8}
    timed = {k: v for k, v in prof.items() if v[1] > 0 and k in alg_bytes}
    dom = max(timed, key=lambda k: timed[k][0])
    dom_bytes = alg_bytes[dom]
    dom_ms = prof[dom][0] / prof[dom][1]
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    launches_per_step = sum(v[1] for v in prof.values()) / args.steps
    total_prof_ms = sum(v[0] for v in prof.values())
    stack_bytes = sum(layer_bytes(u, T) for u in used)

    # e2e through the C ABI with pinned host buffers
    hx = torch.empty((args.layers, T, H), dtype=torch.float32, pin_memory=True)
    for l in range(args.layers):
        hx[l].copy_(torch.from_numpy(stack.w[l]["x"].get().reshape(T, H)))
    hout = torch.empty((args.layers, T, H), dtype=torch.float32, pin_memory=True)
    nbytes = T * H * 4

    def e2e_step():
        for l in range(args.layers):
            L.call("write", stack.w[l]["x"].p, hx[l].data_ptr(), nbytes)
        L.call("graph_launch", graph)
        for l in range(args.layers):
            L.call("read", hout[l].data_ptr(), stack.w[l]["out"].p, nbytes)

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    barrier()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = T * args.steps / e2e_s

    # config 5's prefill: one layer at T=2048 with the router, Zipf bias and the
    # shared expert (layer 0's weights), expert parallel at N>1; device time, max
    # over ranks
    prefill_ep = None
    if not args.no_prefill:
        P = 2048
        d0 = stack.w[0]
        dxp = L.synth_normal(P * H, 77)
        outp = L.Device.empty((P, H), np.float32)
        idp, wtp = L.Device.empty((P, K), np.int32), L.Device.empty((P, K), np.float32)
        if ep_mode:
            from nebula_b200 import ep as epm
            pg = epm.EpGroup(P, H, F, rank, world)

            def prep():
                L.call("moe_layer_ep", outp.p, idp.p, wtp.p, dxp.p, P, d0["router"].p, d0["bias"].p, d0["gate"].p,
                       Q4K, d0["up"].p, Q4K, d0["down"].p, Q4K, d0["n_local"], d0["local"].p, d0["sg"].p, Q4K,
                       d0["su"].p, Q4K, d0["sd"].p, Q4K, d0["sr"].p, 0, H, F, rank, world, pg.ptrs)
        else:
            pws2 = L.workspace(P, H, F)

            def prep():
                L.call("moe_layer", outp.p, idp.p, wtp.p, dxp.p, P, d0["router"].p, d0["bias"].p, d0["gate"].p, Q4K,
                       d0["up"].p, Q4K, d0["down"].p, Q4K, d0["sg"].p, Q4K, d0["su"].p, Q4K, d0["sd"].p, Q4K,
                       d0["sr"].p, H, F, pws2.p)
        for _ in range(3):
            prep()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, args.steps // 4)
        a.record()
        for _ in range(reps):
            prep()
        b.record()
        torch.cuda.synchronize()
        pms = a.elapsed_time(b) / reps
        if dist:
            t = torch.tensor([pms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            pms = float(t.item())
        prefill_ep = {"workload": "config 5 prefill: 1 layer, T=2048, router + Zipf bias + shared expert, "
                                  f"{'expert parallel over %d GPUs (rank r returns its 1/%d of the tokens)' % (world, world) if ep_mode else 'one GPU'}",
                      "tokens_per_s": P / (pms / 1e3), "ms_per_layer": pms}
        if ep_mode:
            barrier()
            pg.close()
            barrier()

    # prefill (config 4) on layer 0's weights
    prefill = None
    if not args.no_prefill and world == 1:  # config 4 is a single-GPU layer
        P = 2048
        rng = np.random.default_rng(3)
        dl = L.Device(rng.normal(0, 1, (P, E)).astype(np.float32))
        dx = L.synth_normal(P * H, 33)
        di, dw = L.Device.empty((P, K), np.int32), L.Device.empty((P, K), np.float32)
        dout = L.Device.empty((P, H), np.float32)
        pws = L.workspace(P, H, F)
        d0 = stack.w[0]

        def pre():
            L.call("route", di.p, dw.p, dl.p, P)
            L.call("moe_routed", dout.p, dx.p, di.p, dw.p, P, d0["gate"].p, Q4K, d0["up"].p, Q4K, d0["down"].p,
                   Q4K, H, F, pws.p)

        for _ in range(3):
            pre()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, args.steps // 4)
        a.record()
        for _ in range(reps):
            pre()
        b.record()
        torch.cuda.synchronize()
        pms = a.elapsed_time(b) / reps
        pbytes = E * EXPERT_BYTES + 2 * P * H * 4 + P * K * 8
        flops = P * 62_914_560
        prefill = {"workload": "config 4: 1 layer, T=2048, N(0,1) logits -> top-10, 512 Q4_K experts",
                   "tokens_per_s": P / (pms / 1e3), "ms_per_layer": pms,
                   "hbm_gbs": pbytes / (pms / 1e3) / 1e9, "hbm_frac": pbytes / (pms / 1e3) / 1e9 / peaks["hbm_gbs"],
                   "tflops": flops / (pms / 1e3) / 1e12,
                   "tensor_frac": flops / (pms / 1e3) / 1e12 / peaks["bf16_tflops"],
                   "path": "tcgen05 tensor-core expert kernel (Q4_K codes and fp16 hi/lo activations)"}

    cpu = None
    if not args.no_cpu and world == 1:
        from oracle import oracle as orc
        threads = orc.host_threads()
        res = cpu_reference_sample(L, stack, T, 2, args.cpu_seconds, threads)
        cpu = {"value": T / (res["per_layer_s"] * args.layers), "unit": "tokens/s", "cores": threads,
               "kind": "reference",
               "sample": f"{res['layers_timed']} layer evaluations of layers 0-1 at T={T} "
                         f"(median per layer x {args.layers}); qc_moe backend {res['backend']}"}

    line = {
        "metric": "moe_verify_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if ep_mode else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"48-layer routed-MoE stack (BASELINE config 3; config 5, expert parallel over "
                               f"{world} GPUs, at N>1), T={T} verify tokens, H=2048 F=512, 512 Q4_K experts/layer "
                               "+ Q4_K shared expert, top-10, Zipf-skewed routing",
                   "layers": args.layers, "tokens": T,
                   "parallelism": f"ep{world}" if ep_mode else "single",
                   "l2": "inputs larger than L2 (43.5 GB of weights streamed per step)",
                   "experts_used_per_layer_mean": float(np.mean(used)),
                   "stack_bytes_per_step": stack_bytes,
                   "stack_hbm_gbs": stack_bytes / (ms_step / 1e3) / 1e9},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": None, "algorithmic_bytes_per_launch": dom_bytes, "avg_launch_ms": dom_ms,
                     "phase_share": {k: v[0] / total_prof_ms for k, v in prof.items() if v[1]},
                     "phase_ms_per_launch": {k: v[0] / v[1] for k, v in prof.items() if v[1]}},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": args.layers * nbytes,
                "d2h_bytes_per_step": args.layers * nbytes},
        "gpu_launches": int(round(args.steps * launches_per_step)),
        "clocks": clk.summary(),
    }
    if prefill:
        line["prefill"] = prefill
    if prefill_ep:
        line["prefill_ep"] = prefill_ep
    if cpu:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    L.load().qg_graph_destroy(graph)
    if dist:
        dist.barrier()
        stack.epg.close()  # unmap the peers' workspaces before any rank frees its own
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
