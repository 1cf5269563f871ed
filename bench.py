#!/usr/bin/env python3
"""Benchmark of the routed-MoE hot path (one JSON line on rank 0).

Headline workload (BASELINE configs 3/5): a 48-layer stack of routed-MoE layers
at hidden 2048 / FFN 512, 512 Q4_K experts per layer (43.5 GB resident) plus a
Q4_K shared expert with its sigmoid gate, router F32 [512x2048] ~N(0,0.02),
routing skewed by a logit bias bias[perm_l[r]] = -1.1*ln(r+1) where perm_l is
the reference's own per-layer hot-expert ranking ("generation" list of
qwen/expert_ranking.json, carried as tests/golden/expert_ranking.npz), x_l
~N(0,1) independent per layer (no residual: the attention between layers is
out of scope). One step = one speculative-verify batch of T=17 tokens through
all 48 layers (router GEMV, top-10, experts, combine, shared expert), captured
in one CUDA graph and replayed. Weights are synthetic (qg_synth_*), generated
from seeds; oracle/synth.c regenerates the same bytes on the host, so the CPU
baselines run on exactly the GPU arm's layers.

The stack's weights (43.5 GB) are far larger than L2 (126 MB), so every step
streams its experts from HBM; the single-layer configs rotate through 8
independently generated layers for the same reason.

Keys beyond the contract: `parity` (layer 0 of this run against the CPU
checker at N=1, against the single-GPU layer at N>1), `prefill` (config 4: one
layer, T=2048, N(0,1) logits fed to top-10; with its CPU baseline and parity),
`prefill_ep` (config 5's prefill: T=2048 through the router with the prefill
ranking's bias and the shared expert; expert parallel at N>1, with whole-job
tensor and HBM fractions), `configs` (config 1: T=4 Q4_K; config 2: T=17
IQ4_NL; the config-3 sweep T=1..17; the product shape 2560/640 with Q4_K
gate/up and IQ4_NL down at T=17 and its prefill at T=2048 - each with its
roofline and a CPU baseline; the dense GEMV qg_matmul in five formats at T=1
and 17, bitwise against qc_matmul), `roofline` (dominant kernel vs measured HBM copy
bandwidth), `cpu_baseline` (the reference's own CPU MoE on this host's cores),
`e2e` (the same metric through the C ABI with pinned host buffers copied in
and results read back every step).

Multi-GPU: launched by torch.distributed.run, one process
per GPU, expert parallel. Every rank holds 1/N of each layer's experts (snake
order of the layer's ranking) plus the replicated router and shared expert,
and all ranks run the same T tokens (strong scaling): each computes its
experts' rows, stores them into every rank's workspace over NVLink and reduces.
The value is T tokens per step divided by the slowest rank's step time.

`--impl reference` times the reference's CPU MoE (qc_moe from qwen/cpu.c,
compiled into oracle/_ref) on the same workload and bytes, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, F, E, K = 2048, 512, 512, 10
Q4K, IQ4NL = 12, 20
ROT = 8  # independently generated layers the single-layer configs rotate through
RANKING = ROOT / "tests" / "golden" / "expert_ranking.npz"


def row_bytes(typ: int, cols: int) -> int:
    return {0: cols * 4, 8: cols // 32 * 34, 14: cols // 256 * 210, Q4K: cols // 256 * 144, IQ4NL: cols // 32 * 18}[typ]


def expert_bytes(h: int, f: int, gt: int, dt: int) -> int:
    return 2 * f * row_bytes(gt, h) + h * row_bytes(dt, f)


EXPERT_BYTES = expert_bytes(H, F, Q4K, Q4K)  # 1,769,472


def ranking(layer: int, kind: str = "generation") -> np.ndarray:
    """The reference's hot-expert ranking of one layer (hottest first)."""
    with np.load(RANKING) as d:
        return d[kind][layer % 48].astype(np.int64)


def zipf_bias(layer: int, kind: str = "generation") -> np.ndarray:
    bias = np.zeros(E, np.float32)
    bias[ranking(layer, kind)] = (-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    return bias


def layer_bytes(U: int, T: int, eb: int = EXPERT_BYTES, h: int = H, shared: bool = True) -> int:
    """Algorithmic HBM bytes of one layer: U experts + router + shared expert + x in/out + routing."""
    return U * eb + 512 * h * 4 + (eb + h * 4 if shared else 0) + 2 * T * h * 4 + T * K * 8


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def traffic_per_launch(kernel: str, workload: str, alg_bytes: float) -> tuple[float | None, str | None]:
    """DRAM bytes per launch: the committed ncu ratio of traffic to algorithmic bytes
    (profiles/traffic.txt: 'kernel workload ratio notes...') times this launch's
    algorithmic bytes."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None, None
    for line in p.read_text().splitlines():
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == kernel and f[1] == workload:
            return float(f[2]) * alg_bytes, ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one capture, "
                                             f"{float(f[2]):.4f} x the algorithmic bytes (profiles/traffic.txt: "
                                             f"{' '.join(f[3:])})")
    return None, None


def host_cores() -> dict:
    """nproc, physical cores (distinct (package, core) pairs) and the threads the CPU legs use."""
    from oracle import oracle as orc
    nproc = len(os.sched_getaffinity(0))
    phys = set()
    try:
        pkg = core = None
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("physical id"):
                    pkg = line.split(":")[1].strip()
                elif line.startswith("core id"):
                    core = line.split(":")[1].strip()
                elif not line.strip() and core is not None:
                    phys.add((pkg, core))
                    pkg = core = None
    except OSError:
        pass
    return {"nproc": nproc, "physical": len(phys) or None, "threads": orc.host_threads()}


def workload_config(T: int, layers: int, world: int) -> dict:
    """The `config` object both arms print (the same workload, whichever arm runs it)."""
    return {"workload": f"48-layer routed-MoE stack (BASELINE config 3; config 5, expert parallel over {world} "
                        f"GPUs, at N>1), T={T} verify tokens, H=2048 F=512, 512 Q4_K experts/layer + Q4_K shared "
                        "expert, top-10, routing skewed by the reference's per-layer expert ranking",
            "layers": layers, "tokens": T, "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (43.5 GB of weights streamed per step)"}


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
    shorter than nvidia-smi's own sampling period); with ``path`` the samples
    are also written there as CSV. Reading only: no setting of the GPU is
    changed."""
    REASONS = (("hw_slowdown", 8), ("hw_thermal_slowdown", 64), ("sw_thermal_slowdown", 32),
               ("sw_power_cap", 4))

    def __init__(self, index: int, pci_bus_id: str | None = None, path: str | None = None):
        self.index, self.pci = index, pci_bus_id
        self.samples: list[tuple[float, float, float, int]] = []
        self.max_mhz = None
        self.path = Path(path) if path else None
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
            if not self.path:
                return
            try:
                self.path.parent.mkdir(parents=True, exist_ok=True)
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


# ---------------------------------------------------------------- layer recipes
# Seeds of layer l of a stack with seed0: router s+4, gate s+1, up s+2, down
# s+3, shared gate/up/down s+5..s+7, shared router row s+8 (s = seed0 + 100*l),
# x from stream 2 + l + 7919*seed0. Both the device stack and the host
# restatement build layers from this one recipe.
def layer_seeds(l: int, seed0: int = 0) -> dict:
    s = seed0 + 100 * l
    return {"gate": s + 1, "up": s + 2, "down": s + 3, "router": s + 4, "sg": s + 5, "su": s + 6, "sd": s + 7,
            "sr": s + 8, "x": 2 + l + 7919 * seed0}


class View:
    """A slice of a larger device buffer (it owns nothing): `p`, `nbytes` and `get()`."""

    def __init__(self, L, base, offset: int, shape, dtype):
        self.L, self.base = L, base
        self.p = base.p + offset
        self.shape, self.dtype = tuple(shape), np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape)) * self.dtype.itemsize

    def get(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        self.L.call("read", out.ctypes.data, self.p, out.nbytes)
        return out


class Stack:
    """Resident layers on the device plus per-layer inputs and outputs.

    The layers' inputs are slices of one buffer (`xall`, [layers][T][h]) and so are
    their outputs (`oall`), so a whole step's activations cross the host link in one
    copy each way.

    With ``ep=(rank, world)`` the rank keeps only its share of each layer's
    experts (snake order of the layer's ranking) and runs the expert-parallel
    layer; weights and inputs are the same on every rank."""

    def __init__(self, L, layers: int, T: int, seed0: int = 0, ep=None, h: int = H, f: int = F, gt: int = Q4K,
                 dt: int = Q4K, shared: bool = True, bias: bool = True):
        self.L, self.T, self.layers, self.ep = L, T, layers, ep
        self.h, self.f, self.gt, self.dt, self.seed0 = h, f, gt, dt, seed0
        self.w = []
        act = T * h * 4
        self.xall, self.oall = L.Device(nbytes=layers * act), L.Device(nbytes=layers * act)
        if ep:
            from nebula_b200 import ep as epm
            rank, world = ep
            self.epg = epm.EpGroup(T, h, f, rank, world)
        for l in range(layers):
            sd = layer_seeds(l, seed0)
            d = {"router": L.synth_weights(0, E, h, sd["router"])}
            mats = (("gate", f, h, gt), ("up", f, h, gt), ("down", h, f, dt))
            if ep:
                owner = epm.snake_owner(ranking(l), world)
                loc, experts = epm.local_map(owner, rank)
                for name, rows, cols, typ in mats:
                    full = L.synth_weights(typ, E * rows, cols, sd[name])
                    d[name] = epm.extract_experts(full, experts, rows, row_bytes(typ, cols))
                    full.free()
                d["local"], d["experts"], d["n_local"] = L.Device(loc), set(experts), len(experts)
            else:
                for name, rows, cols, typ in mats:
                    d[name] = L.synth_weights(typ, E * rows, cols, sd[name])
            if shared:
                d.update({"sg": L.synth_weights(gt, f, h, sd["sg"]), "su": L.synth_weights(gt, f, h, sd["su"]),
                          "sd": L.synth_weights(dt, h, f, sd["sd"]), "sr": L.synth_weights(0, 1, h, sd["sr"])})
            L.call("synth_normal", C.c_void_p(self.xall.p + l * act), T * h, sd["x"], C.c_float(1.0))
            d.update({
                "bias": L.Device(zipf_bias(l)) if bias else None,
                "x": View(L, self.xall, l * act, (T * h,), np.float32),
                "out": View(L, self.oall, l * act, (T, h), np.float32),
                "ids": L.Device.empty((T, K), np.int32), "wts": L.Device.empty((T, K), np.float32),
            })
            self.w.append(d)
        self.ws = self.epg.ws if ep else L.workspace(T, h, f)

    def run_layer(self, l: int, T: int | None = None):
        d, L, T = self.w[l], self.L, T or self.T
        p = lambda k: d[k].p if d.get(k) is not None else None  # noqa: E731
        gt, dt = self.gt, self.dt
        if self.ep:
            rank, world = self.ep
            L.call("moe_layer_ep", d["out"].p, d["ids"].p, d["wts"].p, d["x"].p, T, d["router"].p, p("bias"),
                   d["gate"].p, gt, d["up"].p, gt, d["down"].p, dt, d["n_local"], d["local"].p, p("sg"), gt,
                   p("su"), gt, p("sd"), dt, p("sr"), l % world, self.h, self.f, rank, world, self.epg.ptrs)
            return
        L.call("moe_layer", d["out"].p, d["ids"].p, d["wts"].p, d["x"].p, T, d["router"].p, p("bias"), d["gate"].p,
               gt, d["up"].p, gt, d["down"].p, dt, p("sg"), gt, p("su"), gt, p("sd"), dt, p("sr"), self.h, self.f,
               self.ws.p)

    def step(self, T: int | None = None):
        for l in range(self.layers):
            self.run_layer(l, T)

    def capture(self, T: int | None = None):
        g = C.c_void_p()
        self.L.call("graph_begin", C.byref(g))
        try:
            self.step(T)
        except Exception:
            self.L.graph_destroy(g)  # abandons the capture
            raise
        self.L.call("graph_end", g)
        return g

    def experts_used(self, T: int | None = None) -> list[int]:
        """Experts this rank computed per layer (its share under expert parallelism)."""
        out = []
        for d in self.w:
            u = set(np.unique(d["ids"].get()[:T or self.T]).tolist()) - {-1}
            out.append(len(u & d["experts"]) if self.ep else len(u))
        return out


class HostLayers:
    """The same layers on the host (oracle/synth.c), for the reference CPU MoE.

    A layer is routed on the CPU first (qc_matmul logits, bitwise those of the
    device router, plus the bias) and only the experts its tokens select are
    generated into full-size buffers, so untouched experts cost nothing."""

    def __init__(self, T: int, seed0: int = 0, h: int = H, f: int = F, gt: int = Q4K, dt: int = Q4K,
                 shared: bool = True, bias: bool = True, threads: int | None = None):
        from oracle import oracle as orc
        self.orc = orc
        self.ref, self.rs, self.syn = orc.RefCPU(h, f), orc.Restate(), orc.Synth()
        self.T, self.seed0, self.h, self.f, self.gt, self.dt = T, seed0, h, f, gt, dt
        self.shared, self.bias = shared, bias
        self.threads = threads or orc.host_threads()

    def layer(self, l: int, T: int | None = None, all_experts: bool = False, x: np.ndarray | None = None,
              logits: np.ndarray | None = None) -> dict:
        T, h, f, gt, dt, syn = T or self.T, self.h, self.f, self.gt, self.dt, self.syn
        sd = layer_seeds(l, self.seed0)
        if x is None:
            x = syn.normal(self.T * h, sd["x"]).reshape(self.T, h)[:T]
        router = syn.weights(0, E, h, sd["router"]).view(np.float32).reshape(E, h)
        b = zipf_bias(l) if self.bias else np.zeros(E, np.float32)
        if logits is None:
            logits = self.ref.matmul(router, 0, E, h, x, self.threads) + b
        ids, _ = self.rs.route(logits)
        used = range(E) if all_experts else sorted(set(ids.ravel().tolist()) - {-1})
        gate = np.empty(E * f * row_bytes(gt, h), np.uint8)
        up = np.empty_like(gate)
        down = np.empty(E * h * row_bytes(dt, f), np.uint8)
        if all_experts:
            syn.weights(gt, E * f, h, sd["gate"], out=gate)
            syn.weights(gt, E * f, h, sd["up"], out=up)
            syn.weights(dt, E * h, f, sd["down"], out=down)
        else:
            for e in used:
                syn.weights(gt, E * f, h, sd["gate"], out=gate, row0=e * f, nrows=f)
                syn.weights(gt, E * f, h, sd["up"], out=up, row0=e * f, nrows=f)
                syn.weights(dt, E * h, f, sd["down"], out=down, row0=e * h, nrows=h)
        d = dict(x=x, router=router, bias=b, logits=logits, gate=gate, up=up, down=down, used=len(used))
        if self.shared:
            d["shared"] = (syn.weights(gt, f, h, sd["sg"]), gt, syn.weights(gt, f, h, sd["su"]), gt,
                           syn.weights(dt, h, f, sd["sd"]), dt,
                           syn.weights(0, 1, h, sd["sr"]).view(np.float32).reshape(1, h))
        return d

    def run(self, d: dict, route: bool = True):
        """One layer as the reference host runs it: router GEMV (+bias), top-10,
        qc_moe, shared expert. Returns (out, ids)."""
        if route:
            logits = self.ref.matmul(d["router"], 0, E, self.h, d["x"], self.threads) + d["bias"]
        else:
            logits = d["logits"]
        out, ids, _, _ = self.orc.moe_layer(self.ref, self.rs, d["x"], None, d["gate"], self.gt, d["up"], self.gt,
                                            d["down"], self.dt, shared=d.get("shared"), logits=logits,
                                            threads=self.threads)
        return out, ids


def time_cpu_layers(hl: HostLayers, layers: list[dict], seconds: float, min_evals: int = 3,
                    route: bool = True) -> dict:
    """Median time of one layer evaluation, rotating through `layers`."""
    hl.run(layers[0], route)  # warm-up
    times, n = [], 0
    t_end = time.perf_counter() + seconds
    while n < min_evals or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        hl.run(layers[n % len(layers)], route)
        times.append(time.perf_counter() - t0)
        n += 1
    return {"per_layer_s": float(np.median(times)), "evals": n, "backend": hl.ref.backend()}


def parity(out: np.ndarray, ref: np.ndarray, ids=None, ref_ids=None) -> dict:
    """The path's parity bar: ids bit-exact, rel-L2 <= 1e-5, max-abs <= 1e-4 * max|ref|."""
    a, b = np.asarray(out, np.float64), np.asarray(ref, np.float64)
    rel = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    mabs = float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
    r = {"rel_l2": rel, "max_abs_rel": mabs, "bitwise_equal": bool(np.array_equal(a, b)),
         "pass": bool(np.isfinite(a).all() and rel <= 1e-5 and mabs <= 1e-4)}
    if ids is not None:
        r["ids_bitexact"] = bool(np.array_equal(ids, ref_ids))
        r["pass"] = r["pass"] and r["ids_bitexact"]
    return r


def cpu_line(value: float, cores: dict, sample: str, unit: str = "tokens/s") -> dict:
    return {"value": value, "unit": unit, "cores": cores["threads"], "nproc": cores["nproc"],
            "physical_cores": cores["physical"], "kind": "reference", "sample": sample}


# ---------------------------------------------------------------- reference arm
def run_reference_arm(args, rank: int, world: int) -> None:
    """bench.py --impl reference: the reference's CPU MoE path on this host's cores,
    on the headline workload's own bytes (8 rotated layers of the stack)."""
    if rank != 0:
        return
    cores = host_cores()
    T = args.tokens
    hl = HostLayers(T)
    layers = [hl.layer(l) for l in range(min(ROT, args.layers))]
    hl.run(layers[0])  # warm-up
    per_step = []
    for _ in range(args.warmup + args.steps):
        t = []
        for d in layers:  # one step: each rotated layer once
            t0 = time.perf_counter()
            hl.run(d)
            t.append(time.perf_counter() - t0)
        per_step.append(float(np.median(t)))
    t_layer = float(np.median(per_step[args.warmup:]))
    value = T / (t_layer * args.layers)
    sample = (f"each step evaluates layers 0-{len(layers) - 1} of the stack once (identical bytes to the GPU arm, "
              f"regenerated by oracle/synth.c); median layer time x {args.layers}; qc_moe backend "
              f"{hl.ref.backend()}, {cores['threads']} threads on {cores['nproc']} logical / "
              f"{cores['physical']} physical cores")
    line = {
        "impl": "reference", "metric": "moe_verify_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_layer * args.layers * 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config(T, args.layers, world),
        "cpu_baseline": cpu_line(value, cores, sample),
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm helpers
def event_ms(torch, fn, reps: int) -> float:
    """Average device time of fn() over reps launches (CUDA events on the legacy stream)."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def read_profile(L) -> dict:
    phases = ("router", "route", "plan", "gate_up", "down", "combine", "experts", "decode_router", "lean")
    prof = {}
    for i, name in enumerate(phases):
        tot, n = C.c_double(0), C.c_int(0)
        L.call("moe_profile_read", i, C.byref(tot), C.byref(n))
        prof[name] = (tot.value, n.value)
    return prof


def single_layer_config(torch, L, peaks, T: int, h: int, f: int, gt: int, dt: int, shared: bool, seed0: int,
                        cpu: bool, cpu_seconds: float, what: str, steps: int, traffic_key=None) -> dict:
    """One routed-MoE layer at T tokens, timed over ROT rotated layers (graph replay),
    with its roofline and the reference CPU MoE on the same bytes."""
    st = Stack(L, ROT, T, seed0=seed0, h=h, f=f, gt=gt, dt=dt, shared=shared, bias=False)
    L.call("sync")
    g = st.capture()
    for _ in range(3):
        L.call("graph_launch", g)
    reps = max(5, steps // 2)
    ms_layer = event_ms(torch, lambda: L.call("graph_launch", g), reps) / ROT
    used = st.experts_used()
    eb = expert_bytes(h, f, gt, dt)
    lb = float(np.mean([layer_bytes(u, T, eb, h, shared) for u in used]))
    # the dominant kernel alone (per-phase events over an eager pass)
    L.call("moe_profile", 1)
    st.step()
    prof = read_profile(L)
    L.call("moe_profile", 0)
    kern = max((k for k in prof if prof[k][1]), key=lambda k: prof[k][0])
    kms = prof[kern][0] / prof[kern][1]
    kbytes = (float(np.mean(used)) + (1 if shared else 0)) * eb + 2 * T * h * 4
    if kern == "decode_router":
        kbytes = (E + 1) * h * 4 + T * h * 4 + T * K * 8
    elif kern == "lean":  # the whole layer in one kernel: the router's rows too
        kbytes += (E + 1) * h * 4
    res = {"workload": what, "tokens": T, "tokens_per_s": T / (ms_layer / 1e3), "ms_per_layer": ms_layer,
           "experts_used_mean": float(np.mean(used)), "layer_bytes": lb,
           "hbm_gbs": lb / (ms_layer / 1e3) / 1e9, "hbm_frac": lb / (ms_layer / 1e3) / 1e9 / peaks["hbm_gbs"],
           "roofline": {"bound": "hbm", "kernel": kern, "achieved": kbytes / (kms / 1e3) / 1e9,
                        "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": kbytes / (kms / 1e3) / 1e9 / peaks["hbm_gbs"], "avg_launch_ms": kms,
                        "algorithmic_bytes_per_launch": kbytes,
                        "phase_ms_per_launch": {k: v[0] / v[1] for k, v in prof.items() if v[1]}},
           "l2": f"{ROT} rotated layers ({ROT * E * eb / 1e9:.1f} GB of experts)"}
    if traffic_key and kern == "experts":
        tr, src = traffic_per_launch(*traffic_key, kbytes)
        res["roofline"]["traffic"], res["roofline"]["traffic_source"] = tr, src
    if cpu:
        cores = host_cores()
        hl = HostLayers(T, seed0=seed0, h=h, f=f, gt=gt, dt=dt, shared=shared, bias=False)
        d0 = hl.layer(0)
        out, ids = hl.run(d0)
        res["parity"] = parity(st.w[0]["out"].get(), out, st.w[0]["ids"].get(), ids)
        layers = [d0] + [hl.layer(l) for l in range(1, 3)]
        c = time_cpu_layers(hl, layers, cpu_seconds)
        res["cpu_baseline"] = cpu_line(T / c["per_layer_s"], cores,
                                       f"{c['evals']} evaluations of layers 0-2 (same bytes); qc_moe backend "
                                       f"{c['backend']}")
    L.graph_destroy(g)
    del st
    L.call("sync")
    return res


def product_small_batches(torch, L, peaks, cpu: bool, steps: int) -> dict:
    """Nebula's production mix (2560/640, Q4_K gate/up + IQ4_NL down, router and
    shared expert) at T = 1..4 over ROT rotated layers, one graph per T: the range
    the single-kernel layer takes at this shape. Per T: time per layer, the kernel
    that ran (per-phase events over one eager pass), the layer's bytes and, with
    `cpu`, layer 0 of that pass against the reference CPU MoE on the same bytes."""
    h, f = 2560, 640
    st = Stack(L, ROT, 4, seed0=15, h=h, f=f, gt=Q4K, dt=IQ4NL, shared=True, bias=False)
    hl = HostLayers(4, seed0=15, h=h, f=f, gt=Q4K, dt=IQ4NL, shared=True, bias=False) if cpu else None
    eb = expert_bytes(h, f, Q4K, IQ4NL)
    pts = {}
    for t in range(1, 5):
        g = st.capture(t)
        for _ in range(3):
            L.call("graph_launch", g)
        ms = event_ms(torch, lambda: L.call("graph_launch", g), max(5, steps // 2)) / ROT
        L.graph_destroy(g)
        used = st.experts_used(t)
        L.call("moe_profile", 1)
        st.step(t)
        prof = read_profile(L)
        L.call("moe_profile", 0)
        lb = float(np.mean([layer_bytes(u, t, eb, h, True) for u in used]))
        pts[str(t)] = {"us_per_layer": ms * 1e3, "tokens_per_s": t / (ms / 1e3),
                       "experts_used_mean": float(np.mean(used)), "layer_bytes": lb,
                       "hbm_frac": lb / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                       "kernels": sorted(k for k in prof if prof[k][1])}
        if hl is not None:
            out, ids = hl.run(hl.layer(0, t))
            pts[str(t)]["parity"] = parity(st.w[0]["out"].get()[:t], out, st.w[0]["ids"].get()[:t], ids)
    del st
    L.call("sync")
    return {"workload": f"product shape at T = 1..4: {ROT} rotated layers of 2560/640, Q4_K gate/up + IQ4_NL "
                        "down, router + shared expert, unbiased routing (graph per T)", "points": pts}


def dense_blocks(typ: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Random Q8_0 (8) or Q6_K (14) rows with valid fp16 scales (the device generator
    covers F32, Q4_K and IQ4_NL)."""
    rng = np.random.default_rng(seed)
    rb = row_bytes(typ, cols)
    w = rng.integers(0, 256, rows * rb, dtype=np.uint8)
    blk, d_off = (34, 0) if typ == 8 else (210, 208)
    b = w.reshape(-1, blk)
    b[:, d_off:d_off + 2] = np.frombuffer(np.full(len(b), 0.001, np.float16).tobytes(), np.uint8).reshape(-1, 2)
    return w


def dense_gemv(torch, L, peaks, cpu: bool, steps: int) -> dict:
    """qg_matmul (the dense dequant GEMV that serves every non-MoE projection) on an 8192 x 2560
    projection in five formats at T = 1 and 17, rotated over copies that exceed L2, with its HBM
    roofline and a bitwise check against the reference qc_matmul."""
    rows, cols = 8192, 2560
    res = {"workload": f"qg_matmul, {rows} x {cols} weights, T = 1 and 17, rotated copies > 300 MB (past L2), "
                       "one CUDA graph of all copies' launches per timed step"}
    ref = None
    if cpu:
        from oracle import oracle as orc
        ref = orc.RefCPU(2560, 640)
    for name, typ in (("f32", 0), ("q8_0", 8), ("q6_k", 14), ("q4_k", Q4K), ("iq4_nl", IQ4NL)):
        mb = rows * row_bytes(typ, cols)
        copies = max(2, -(-300_000_000 // mb))
        if typ in (8, 14):
            host = dense_blocks(typ, rows, cols, 40 + typ)
            ws = [L.Device(host) for _ in range(copies)]
        else:
            ws = [L.synth_weights(typ, rows, cols, 40 + typ + i) for i in range(copies)]
        line = {"copies": copies, "weight_bytes": mb}
        for T in (1, 17):
            x = L.synth_normal(T * cols, 77)
            out = L.Device.empty((T, rows), np.float32)

            L.call("matmul", out.p, ws[0].p, typ, rows, cols, x.p, T)  # eager first use (module load, attributes)
            g = C.c_void_p()  # one graph of all copies' launches, so launch overhead is not timed
            L.call("graph_begin", C.byref(g))
            for w in ws:
                L.call("matmul", out.p, w.p, typ, rows, cols, x.p, T)
            L.call("graph_end", g)
            for _ in range(3):
                L.call("graph_launch", g)
            ms = event_ms(torch, lambda: L.call("graph_launch", g), max(3, steps // 4)) / copies
            L.graph_destroy(g)
            nbytes = mb + T * cols * 4 + T * rows * 4
            line[f"T{T}"] = {"us": ms * 1e3, "gbs": nbytes / (ms / 1e3) / 1e9,
                             "hbm_frac": nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
            if ref is not None and T == 17:
                L.call("matmul", out.p, ws[0].p, typ, rows, cols, x.p, T)
                hw = host if typ in (8, 14) else ws[0].get()
                line["bitwise_vs_qc_matmul"] = bool(np.array_equal(
                    out.get(), ref.matmul(hw, typ, rows, cols, x.get().reshape(T, cols))))
        res[name] = line
        del ws
    L.call("sync")
    return res


def prefill_product(torch, L, peaks, cpu: bool, cpu_seconds: float, steps: int) -> dict:
    """Prefill of the production mix (hidden 2560 / FFN 640, Q4_K gate/up + IQ4_NL down): one
    layer at T=2048 routed from N(0,1) logits (about 40 tokens per expert), routed experts only,
    with parity and the reference CPU MoE on the same bytes."""
    P, h, f, seed0 = 2048, 2560, 640, 14
    st = Stack(L, 1, P, seed0=seed0, h=h, f=f, gt=Q4K, dt=IQ4NL, shared=False, bias=False)
    d0 = st.w[0]
    logits = np.random.default_rng(5).normal(0, 1, (P, E)).astype(np.float32)
    dl = L.Device(logits)

    def pre():
        L.call("route", d0["ids"].p, d0["wts"].p, dl.p, P)
        L.call("moe_routed", d0["out"].p, d0["x"].p, d0["ids"].p, d0["wts"].p, P, d0["gate"].p, Q4K, d0["up"].p,
               Q4K, d0["down"].p, IQ4NL, h, f, st.ws.p)

    for _ in range(3):
        pre()
    pms = event_ms(torch, pre, max(3, steps // 4))
    pbytes = E * expert_bytes(h, f, Q4K, IQ4NL) + 2 * P * h * 4 + P * K * 8
    flops = P * K * 3 * h * f * 2
    res = {"workload": "product-shape prefill: 1 layer, T=2048, hidden 2560 / FFN 640, Q4_K gate/up + IQ4_NL "
                       "down, N(0,1) logits -> top-10, 512 experts",
           "tokens_per_s": P / (pms / 1e3), "ms_per_layer": pms,
           "hbm_gbs": pbytes / (pms / 1e3) / 1e9, "hbm_frac": pbytes / (pms / 1e3) / 1e9 / peaks["hbm_gbs"],
           "tflops": flops / (pms / 1e3) / 1e12, "tensor_frac": flops / (pms / 1e3) / 1e12 / peaks["bf16_tflops"],
           "path": "tcgen05 tensor-core expert kernel (IQ4_NL down as fp16 hi/lo planes of d*code)"}
    if cpu:
        cores = host_cores()
        hl = HostLayers(P, seed0=seed0, h=h, f=f, gt=Q4K, dt=IQ4NL, shared=False, bias=False)
        dp = hl.layer(0, P, all_experts=True, logits=logits)
        out_c, ids_c = hl.run(dp, route=False)
        res["parity"] = parity(d0["out"].get(), out_c, d0["ids"].get(), ids_c)
        c = time_cpu_layers(hl, [dp], cpu_seconds, min_evals=2, route=False)
        res["cpu_baseline"] = cpu_line(P / c["per_layer_s"], cores,
                                       f"{c['evals']} evaluations of the same layer (same bytes, qc_moe large-batch "
                                       f"path); backend {c['backend']}")
        del dp
    del st
    L.call("sync")
    return res


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
    ap.add_argument("--no-configs", action="store_true", help="skip configs 1, 2, the T sweep and the product shape")
    ap.add_argument("--dense-only", action="store_true",
                    help="print only the dense GEMV measurement (qg_matmul, five formats) as one JSON line")
    ap.add_argument("--routes", default=None,
                    help="also replay this QROUTE1 route trace (the reference's route profiler output) through "
                         "qg_moe_routed on the stack's layers (record layer modulo the stack depth)")
    ap.add_argument("--clock-log", default=None,
                    help="write the NVML clock samples of the timed region as CSV here ({rank} is replaced)")
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
    peaks = measured_peaks()
    if args.dense_only:
        if rank == 0:
            print(json.dumps({"dense_gemv": dense_gemv(torch, L, peaks, not args.no_cpu, args.steps)}))
        return
    stack = Stack(L, args.layers, T, seed0=0, ep=(rank, world) if ep_mode else None)
    L.call("sync")
    graph = stack.capture()

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        L.call("graph_launch", graph)
    barrier()
    used = stack.experts_used()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clock_log = args.clock_log.replace("{rank}", str(rank)) if args.clock_log else None
    with Clocks(local, pci_bus_id(torch, local), clock_log) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            L.call("graph_launch", graph)
        stop.record()
        barrier()
    ms = max_over_ranks(start.elapsed_time(stop))
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)  # every rank works on the same T tokens

    # roofline: per-phase event timing over an eager replay of the same steps
    L.call("moe_profile", 1)
    for _ in range(args.steps):
        stack.step()
    prof = read_profile(L)
    L.call("moe_profile", 0)
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
    traffic, traffic_src = traffic_per_launch("tc_experts_kernel<24>" if dom == "experts" else dom,
                                              f"T{T}_ep{world}" if ep_mode else f"T{T}", dom_bytes)
    phase_us = {k: max_over_ranks(1e3 * v[0] / args.steps / args.layers) for k, v in sorted(prof.items()) if v[1]}

    # e2e through the C ABI with pinned host buffers
    hx = torch.empty((args.layers, T, H), dtype=torch.float32, pin_memory=True)
    for l in range(args.layers):
        hx[l].copy_(torch.from_numpy(stack.w[l]["x"].get().reshape(T, H)))
    hout = torch.empty((args.layers, T, H), dtype=torch.float32, pin_memory=True)
    nbytes = T * H * 4

    def e2e_step():  # the 48 layers' inputs and outputs are contiguous: one copy each way
        L.call("write", stack.xall.p, hx.data_ptr(), args.layers * nbytes)
        L.call("graph_launch", graph)
        L.call("read", hout.data_ptr(), stack.oall.p, args.layers * nbytes)

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = T * args.steps / e2e_s

    # parity of layer 0 (the outputs of the last e2e step)
    par = None
    if ep_mode:
        # this rank's expert-parallel layer 0 against the single-GPU layer on full weights
        d0, sd = stack.w[0], layer_seeds(0)
        full = {n: L.synth_weights(Q4K, E * r, c, sd[n]) for n, r, c in (("gate", F, H), ("up", F, H),
                                                                         ("down", H, F))}
        ref_out, ref_ids = L.Device.empty((T, H), np.float32), L.Device.empty((T, K), np.int32)
        ws1 = L.workspace(T, H, F)
        L.call("moe_layer", ref_out.p, ref_ids.p, None, d0["x"].p, T, d0["router"].p, d0["bias"].p, full["gate"].p,
               Q4K, full["up"].p, Q4K, full["down"].p, Q4K, d0["sg"].p, Q4K, d0["su"].p, Q4K, d0["sd"].p, Q4K,
               d0["sr"].p, H, F, ws1.p)
        p = parity(d0["out"].get(), ref_out.get(), d0["ids"].get(), ref_ids.get())
        par = {"against": "single-GPU qg_moe_layer on layer 0's full weights, every rank", "tokens": T,
               "rel_l2": max_over_ranks(p["rel_l2"]), "max_abs_rel": max_over_ranks(p["max_abs_rel"]),
               "ids_bitexact": max_over_ranks(0.0 if p["ids_bitexact"] else 1.0) == 0.0,
               "pass": max_over_ranks(0.0 if p["pass"] else 1.0) == 0.0}
        for v in full.values():
            v.free()
        del ws1

    # config 5's prefill: one layer at T=2048 with the router, the prefill
    # ranking's bias and the shared expert (layer 0's weights), expert parallel
    # at N>1; device time, max over ranks
    prefill_ep = None
    if not args.no_prefill:
        P = 2048
        d0 = stack.w[0]
        dxp = L.synth_normal(P * H, 77)
        pbias = L.Device(zipf_bias(0, "prefill"))
        outp = L.Device.empty((P, H), np.float32)
        idp, wtp = L.Device.empty((P, K), np.int32), L.Device.empty((P, K), np.float32)
        if ep_mode:
            from nebula_b200 import ep as epm
            pg = epm.EpGroup(P, H, F, rank, world)

            def prep():
                L.call("moe_layer_ep", outp.p, idp.p, wtp.p, dxp.p, P, d0["router"].p, pbias.p, d0["gate"].p,
                       Q4K, d0["up"].p, Q4K, d0["down"].p, Q4K, d0["n_local"], d0["local"].p, d0["sg"].p, Q4K,
                       d0["su"].p, Q4K, d0["sd"].p, Q4K, d0["sr"].p, 0, H, F, rank, world, pg.ptrs)
        else:
            pws2 = L.workspace(P, H, F)

            def prep():
                L.call("moe_layer", outp.p, idp.p, wtp.p, dxp.p, P, d0["router"].p, pbias.p, d0["gate"].p, Q4K,
                       d0["up"].p, Q4K, d0["down"].p, Q4K, d0["sg"].p, Q4K, d0["su"].p, Q4K, d0["sd"].p, Q4K,
                       d0["sr"].p, H, F, pws2.p)
        for _ in range(3):
            prep()
        barrier()
        pms = max_over_ranks(event_ms(torch, prep, max(3, args.steps // 4)))
        prefill_ep = {"workload": "config 5 prefill: 1 layer, T=2048, router + bias from the reference's prefill "
                                  "ranking + shared expert, " +
                                  (f"expert parallel over {world} GPUs (rank r returns its 1/{world} of the tokens)"
                                   if ep_mode else "one GPU"),
                      "tokens_per_s": P / (pms / 1e3), "ms_per_layer": pms}
        # whole-job roofline over the N GPUs: the experts' tensor work (10 routed + the shared
        # expert per token, 3 H x F products) and every weight byte read once plus x in, out written
        ep_flops = P * (K + 1) * 3 * H * F * 2
        ep_bytes = (E + 1) * EXPERT_BYTES + (E + 1) * H * 4 + 2 * P * H * 4
        prefill_ep.update({"tflops": ep_flops / (pms / 1e3) / 1e12,
                           "tensor_frac": ep_flops / (pms / 1e3) / 1e12 / (world * peaks["bf16_tflops"]),
                           "hbm_frac": ep_bytes / (pms / 1e3) / 1e9 / (world * peaks["hbm_gbs"])})
        if ep_mode:
            # this rank's rows against the single-GPU layer
            sd = layer_seeds(0)
            full = {n: L.synth_weights(Q4K, E * r, c, sd[n]) for n, r, c in (("gate", F, H), ("up", F, H),
                                                                             ("down", H, F))}
            ref_out, ref_ids = L.Device.empty((P, H), np.float32), L.Device.empty((P, K), np.int32)
            ws1 = L.workspace(P, H, F)
            L.call("moe_layer", ref_out.p, ref_ids.p, None, dxp.p, P, d0["router"].p, pbias.p, full["gate"].p,
                   Q4K, full["up"].p, Q4K, full["down"].p, Q4K, d0["sg"].p, Q4K, d0["su"].p, Q4K, d0["sd"].p, Q4K,
                   d0["sr"].p, H, F, ws1.p)
            blk = (P + world - 1) // world
            rows = slice(rank * blk, min(P, (rank + 1) * blk))
            p = parity(outp.get()[rows], ref_out.get()[rows], idp.get(), ref_ids.get())
            prefill_ep["parity"] = {"against": "single-GPU qg_moe_layer, each rank's own tokens",
                                    "rel_l2": max_over_ranks(p["rel_l2"]),
                                    "max_abs_rel": max_over_ranks(p["max_abs_rel"]),
                                    "ids_bitexact": max_over_ranks(0.0 if p["ids_bitexact"] else 1.0) == 0.0,
                                    "pass": max_over_ranks(0.0 if p["pass"] else 1.0) == 0.0}
            for v in full.values():
                v.free()
            del ws1
            barrier()
            pg.close()
            barrier()

    # prefill (config 4) on layer 0's weights
    prefill = None
    if not args.no_prefill and world == 1:  # config 4 is a single-GPU layer
        P = 2048
        logits = np.random.default_rng(3).normal(0, 1, (P, E)).astype(np.float32)
        dl = L.Device(logits)
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
        pms = event_ms(torch, pre, max(3, args.steps // 4))
        pbytes = E * EXPERT_BYTES + 2 * P * H * 4 + P * K * 8
        flops = P * 62_914_560
        prefill = {"workload": "config 4: 1 layer, T=2048, N(0,1) logits -> top-10, 512 Q4_K experts",
                   "tokens_per_s": P / (pms / 1e3), "ms_per_layer": pms,
                   "hbm_gbs": pbytes / (pms / 1e3) / 1e9, "hbm_frac": pbytes / (pms / 1e3) / 1e9 / peaks["hbm_gbs"],
                   "tflops": flops / (pms / 1e3) / 1e12,
                   "tensor_frac": flops / (pms / 1e3) / 1e12 / peaks["bf16_tflops"],
                   "path": "tcgen05 tensor-core expert kernel (Q4_K codes and fp16 hi/lo activations)"}
        if not args.no_cpu:
            cores = host_cores()
            hl = HostLayers(P, shared=False, bias=False)
            hx0 = hl.syn.normal(P * H, 33).reshape(P, H)
            dp = hl.layer(0, P, all_experts=True, x=hx0, logits=logits)
            out_c, ids_c = hl.run(dp, route=False)
            prefill["parity"] = parity(dout.get(), out_c, di.get(), ids_c)
            c = time_cpu_layers(hl, [dp], args.cpu_seconds / 2, min_evals=2, route=False)
            prefill["cpu_baseline"] = cpu_line(P / c["per_layer_s"], cores,
                                               f"{c['evals']} evaluations of the same layer (same bytes, qc_moe "
                                               f"large-batch path); backend {c['backend']}")
            del dp

    cpu = None
    if not args.no_cpu and world == 1:
        cores = host_cores()
        hl = HostLayers(T)
        layers = [hl.layer(l) for l in range(min(ROT, args.layers))]
        out_c, ids_c = hl.run(layers[0])
        par = parity(stack.w[0]["out"].get(), out_c, stack.w[0]["ids"].get(), ids_c)
        par["against"] = "the reference CPU MoE (qc_moe + restated routing) on layer 0's bytes"
        c = time_cpu_layers(hl, layers, args.cpu_seconds)
        cpu = cpu_line(T / (c["per_layer_s"] * args.layers), cores,
                       f"{c['evals']} layer evaluations rotating over layers 0-{len(layers) - 1} at T={T} (identical "
                       f"bytes, regenerated by oracle/synth.c); median per layer x {args.layers}; qc_moe backend "
                       f"{c['backend']}")

    configs = None
    if not args.no_configs and world == 1:
        configs = {}
        want_cpu = not args.no_cpu
        configs["config1"] = single_layer_config(
            torch, L, peaks, 4, H, F, Q4K, Q4K, False, 11, want_cpu, 3.0,
            "config 1: 1 layer, T=4, 512 Q4_K experts, router -> top-10, routed only", args.steps,
            ("tc_experts_kernel<24>", "T17"))
        configs["config2"] = single_layer_config(
            torch, L, peaks, 17, H, F, IQ4NL, IQ4NL, False, 12, want_cpu, 3.0,
            "config 2: 1 layer, T=17, 512 IQ4_NL experts, router -> top-10, routed only", args.steps,
            ("tc_experts_kernel<24,1,1>", "config2-T17"))
        configs["product"] = single_layer_config(
            torch, L, peaks, 17, 2560, 640, Q4K, IQ4NL, True, 13, want_cpu, 3.0,
            "product shape: 1 layer, T=17, hidden 2560 / FFN 640, Q4_K gate/up + IQ4_NL down, router + shared "
            "expert", args.steps, ("tc_experts_kernel<24,1,0>", "product-T17"))
        configs["product_small_batches"] = product_small_batches(torch, L, peaks, want_cpu, args.steps)
        configs["product_prefill"] = prefill_product(torch, L, peaks, want_cpu, 4.0, args.steps)
        configs["dense_gemv"] = dense_gemv(torch, L, peaks, want_cpu, args.steps)
        sweep = {}
        for t in range(1, T + 1):
            g = stack.capture(t)
            for _ in range(2):
                L.call("graph_launch", g)
            ms_t = event_ms(torch, lambda: L.call("graph_launch", g), max(5, args.steps // 10))
            u = stack.experts_used(t)
            sb = sum(layer_bytes(x, t) for x in u)
            sweep[str(t)] = {"tokens_per_s": t / (ms_t / 1e3), "ms_per_step": ms_t,
                             "stack_hbm_gbs": sb / (ms_t / 1e3) / 1e9, "experts_used_mean": float(np.mean(u))}
            L.graph_destroy(g)
        configs["sweep_T1_17"] = {"workload": "config 3: the 48-layer stack at T = 1..17 (graph per T)",
                                  "points": sweep}

    trace_replay = None
    if args.routes and world == 1:
        from nebula_b200 import trace as tr
        xcache = {}

        def x_of(layer, nt):
            if nt not in xcache:
                xcache[nt] = L.synth_normal(nt * H, 9000 + nt)
            return xcache[nt]

        def experts_of(layer):
            d = stack.w[layer % args.layers]
            return d["gate"], Q4K, d["up"], Q4K, d["down"], Q4K

        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nrec = ntok = 0
        torch.cuda.synchronize()
        a.record()
        for _layer, _pos, _out, _ws in tr.replay(args.routes, experts_of, x_of, H, F):
            nrec += 1
            ntok += _out.shape[0]
        b.record()
        torch.cuda.synchronize()
        rms = a.elapsed_time(b)
        trace_replay = {"file": os.path.basename(args.routes), "records": nrec, "token_layers": ntok,
                        "ms": rms, "token_layers_per_s": ntok / (rms / 1e3),
                        "note": "recorded routing through qg_moe_routed on the stack's resident experts; "
                                "includes the host's per-record uploads of ids and weights"}

    line = {
        "metric": "moe_verify_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if ep_mode else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(T, args.layers, world),
        "stack": {"experts_used_per_layer_mean": u_mean, "stack_bytes_per_step": stack_bytes,
                  "stack_hbm_gbs": stack_bytes / (ms_step / 1e3) / 1e9,
                  "stack_hbm_frac": stack_bytes / (ms_step / 1e3) / 1e9 / peaks["hbm_gbs"],
                  "phase_us_per_layer": phase_us},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": traffic, "traffic_source": traffic_src,
                     "algorithmic_bytes_per_launch": dom_bytes, "avg_launch_ms": dom_ms,
                     "phase_share": {k: v[0] / total_prof_ms for k, v in prof.items() if v[1]},
                     "phase_ms_per_launch": {k: v[0] / v[1] for k, v in prof.items() if v[1]}},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": args.layers * nbytes,
                "d2h_bytes_per_step": args.layers * nbytes},
        "gpu_launches": int(round(args.steps * launches_per_step)),
        "clocks": clk.summary(),
    }
    if par:
        line["parity"] = par
    if prefill:
        line["prefill"] = prefill
    if prefill_ep:
        line["prefill_ep"] = prefill_ep
    if cpu:
        line["cpu_baseline"] = cpu
    if configs:
        line["configs"] = configs
    if trace_replay:
        line["trace_replay"] = trace_replay
    if rank == 0:
        print(json.dumps(line), flush=True)
    L.graph_destroy(graph)
    if dist:
        dist.barrier()
        stack.epg.close()  # unmap the peers' workspaces before any rank frees its own
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
