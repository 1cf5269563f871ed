"""Link recipe: the reference model runtime (qwen/qwen.c) with this library's MoE.

The reference links its runtime as ``qwen.o gpu.o ssd.o`` plus the CPU objects
into ``libqwen.so`` (qwen/Makefile:43-45; the probe variant with
``-DQWEN_TEST_HOOKS``, qwen/Makefile:52-56). This recipe builds the same
library with two changes:

* ``qwen.c`` is compiled from a copy in which two definitions are renamed -
  ``moe`` becomes ``moe_reference`` with ``integration/qwen_moe.c`` (the
  all-resident MoE on ``qg_moe_layer``) included in its place, and
  ``qwen_close`` becomes ``qwen_close_reference`` behind a wrapper that first
  releases what qwen_moe.c allocated. Nothing else in the file changes; the
  copy lives only under ``integration/_build/``.
* ``gpu.cu`` (the reference's kernels for everything outside the MoE path:
  attention, Gated DeltaNet, norms, hyper-connections, ...) is compiled for
  sm_100a from a copy whose thread-local launch stream (``capture_stream``,
  qwen/gpu.cu:10) is declared as this library's per-thread launch stream
  (``nebula_launch_stream``) instead of a private one, so both halves launch
  on the same stream and join the same graph captures; every ``qg_*`` symbol
  this library also defines is made weak in that object (``objcopy
  --weaken-symbol``), so the linker takes this library's definitions for the
  whole MoE path, the runtime and the graph functions, and the reference's for
  the rest.

Outputs (``integration/_build/``, git-ignored, shipped with the working tree):
``libqwen.so`` and ``libqwen_probe.so`` (the reference's diagnostic hooks
compiled in). ``--harness`` also builds ``libqwen_moe_probe.so`` from
``tests/integration/moe_probe.c``, the GPU test's entry into the drop-in.
Needs the reference tree ($NEBULA_REFERENCE, else ``reference`` beside this
repository), gcc, nvcc and objcopy; the product library is built first.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
OUT = HERE / "_build"
sys.path.insert(0, str(REPO))

from nebula_b200 import build as nbuild  # noqa: E402

CFLAGS = ["-O3", "-std=c11", "-Wall", "-Wextra", "-Wpedantic", "-fPIC"]
CPU_BASE = CFLAGS + ["-march=x86-64", "-mtune=generic", "-fopenmp"]
CPU_VARIANTS = (  # qwen/Makefile:27-38
    ("cpu_scalar.o", ["-ffp-contract=off", "-DQC_PREFIX=qcs_"]),
    ("cpu_avx2.o", ["-mavx2", "-mfma", "-mf16c", "-DQC_AVX2", "-DQC_PREFIX=qc2_"]),
    ("cpu_avx512.o", ["-mavx512f", "-mavx512dq", "-mavx512bw", "-mavx512vl", "-mfma", "-mf16c", "-DQC_AVX512",
                      "-DQC_PREFIX=qc5_"]),
)
# (anchor in qwen.c, replacement): each anchor must occur exactly once
RENAMES = (
    ("static int moe(qwen_model *m,layer *l,int nt,int mtp){",
     '#include "qwen_moe.c"\nstatic int moe_reference(qwen_model *m,layer *l,int nt,int mtp){'),
    ("void qwen_close(qwen_model *m){",
     "static void nebula_moe_release(qwen_model *m);\nstatic void qwen_close_reference(qwen_model *m);\n"
     "void qwen_close(qwen_model *m){nebula_moe_release(m);qwen_close_reference(m);}\n"
     "static void qwen_close_reference(qwen_model *m){"),
)


def reference_root() -> Path:
    return Path(os.environ.get("NEBULA_REFERENCE") or REPO.parent / "reference")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"{' '.join(cmd)}\n{r.stdout}{r.stderr}")


def patched_qwen_c(qdir: Path) -> Path:
    text = (qdir / "qwen.c").read_text()
    for anchor, repl in RENAMES:
        if text.count(anchor) != 1:
            raise RuntimeError(f"qwen.c: expected one occurrence of {anchor!r}")
        text = text.replace(anchor, repl)
    out = OUT / "qwen.c"
    out.write_text(text)
    return out


STREAM_DECL = ("static __thread cudaStream_t capture_stream;",
               'extern __thread cudaStream_t capture_stream __asm__("nebula_launch_stream");')


def patched_gpu_cu(qdir: Path) -> Path:
    text = (qdir / "gpu.cu").read_text()
    anchor, repl = STREAM_DECL
    if text.count(anchor) != 1:
        raise RuntimeError(f"gpu.cu: expected one occurrence of {anchor!r}")
    out = OUT / "gpu.cu"
    out.write_text(text.replace(anchor, repl))
    return out


def defined_globals(obj: Path) -> set[str]:
    r = subprocess.run(["nm", "-g", "--defined-only", str(obj)], capture_output=True, text=True, check=True)
    return {f[2] for f in (line.split() for line in r.stdout.splitlines()) if len(f) == 3}


def weakened_reference_gpu(qdir: Path, ours: list[Path]) -> tuple[Path, list[str]]:
    """gpu.cu for sm_100a with every symbol this library defines made weak."""
    obj = OUT / "gpu_ref.o"
    _run([nbuild.nvcc(), "-O3", "-std=c++17", *nbuild.ARCH, "-Xcompiler", "-fPIC", f"-I{qdir}", "-c",
          str(patched_gpu_cu(qdir)), "-o", str(obj)])
    mine = set().union(*(defined_globals(o) for o in ours))
    shared = sorted(defined_globals(obj) & mine)
    weak = OUT / "gpu_ref_weak.o"
    _run(["objcopy", *[f"--weaken-symbol={s}" for s in shared], str(obj), str(weak)])
    return weak, shared


def build(harness: bool = False) -> dict:
    qdir = reference_root() / "qwen"
    if not (qdir / "qwen.c").exists():
        raise FileNotFoundError(f"reference runtime sources not found under {qdir}")
    nbuild.build()
    OUT.mkdir(exist_ok=True)
    ours = [nbuild.OBJ / (s.stem + ".o") for s in nbuild.sources()]
    src = patched_qwen_c(qdir)
    inc = [f"-I{qdir}", f"-I{HERE}"]
    objs = {}
    for name, extra in (("qwen.o", []), ("qwen_probe.o", ["-DQWEN_TEST_HOOKS"])):
        _run(["gcc", *CFLAGS, *extra, *inc, "-c", str(src), "-o", str(OUT / name)])
        objs[name] = OUT / name
    _run(["gcc", *CFLAGS, "-pthread", f"-I{qdir}", "-c", str(qdir / "ssd.c"), "-o", str(OUT / "ssd.o")])
    cpu = [OUT / "cpu.o"]
    _run(["gcc", *CPU_BASE, f"-I{qdir}", "-c", str(qdir / "cpu_dispatch.c"), "-o", str(cpu[0])])
    for name, flags in CPU_VARIANTS:
        _run(["gcc", *CPU_BASE, *flags, f"-I{qdir}", "-c", str(qdir / "cpu.c"), "-o", str(OUT / name)])
        cpu.append(OUT / name)
    gpu, weakened = weakened_reference_gpu(qdir, ours)
    common = [str(gpu), str(OUT / "ssd.o"), *map(str, cpu), *map(str, ours)]
    gomp = subprocess.run(["gcc", "-print-file-name=libgomp.so"], capture_output=True, text=True).stdout.strip()
    libs = ([f"-L{os.path.dirname(gomp)}"] if os.path.isabs(gomp) else []) + ["-lgomp"]
    built = {}
    for lib, qobj in (("libqwen.so", "qwen.o"), ("libqwen_probe.so", "qwen_probe.o")):
        _run([nbuild.nvcc(), *nbuild.ARCH, "-shared", str(objs[qobj]), *common, *libs, "-o", str(OUT / lib)])
        built[lib] = OUT / lib
    if harness:
        probe_src = REPO / "tests" / "integration" / "moe_probe.c"
        hobj = OUT / "moe_probe.o"
        _run(["gcc", *CFLAGS, "-DQWEN_TEST_HOOKS", f"-I{OUT}", *inc, "-c", str(probe_src), "-o", str(hobj)])
        _run([nbuild.nvcc(), *nbuild.ARCH, "-shared", str(hobj), *common, *libs,
              "-o", str(OUT / "libqwen_moe_probe.so")])
        built["libqwen_moe_probe.so"] = OUT / "libqwen_moe_probe.so"
    (OUT / "weakened_symbols.txt").write_text("\n".join(weakened) + "\n")
    return built


if __name__ == "__main__":
    for name, path in build(harness="--harness" in sys.argv).items():
        print(name, path)
