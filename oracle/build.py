"""TEST INFRASTRUCTURE ONLY - builds the CPU checker for the routed-MoE path.

Three products:

* ``oracle/_build/librestate.so`` from ``oracle/restate.c`` (our C restatement
  of the reference's device-side routing steps). Builds anywhere with gcc.
* ``oracle/_build/libsynth.so`` from ``oracle/synth.c``: the library's
  synthetic weight generator restated on the host, bit for bit, so CPU
  baselines run on the GPU arm's exact bytes without the product library.
* ``oracle/_ref/libqwen_cpu_<H>x<F>.so``: the reference's own CPU MoE
  (``qwen/cpu.c`` + ``cpu_dispatch.c``), compiled from the reference tree the
  way its ``qwen/Makefile:24-41`` does (three ISA objects with private
  prefixes plus the dispatcher). ``qwen/cpu.c:11`` hard-codes
  ``WIDTH=2560, FF=640``; the 2048/512 shape named by the benchmark configs is
  built from a temporary copy whose enum line alone is rewritten. The copy is
  deleted after compiling and never enters the repository. Only the built
  ``.so`` files travel to GPU machines, where the reference tree is absent.

Linking uses ``-lgomp`` instead of ``-fopenmp``: on this image gcc cannot
read ``libgomp.spec`` at link time, while compiling with ``-fopenmp`` works.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
SHAPES = ((2560, 640), (2048, 512))

CFLAGS = ["-O3", "-std=c11", "-Wall", "-Wextra", "-Wpedantic", "-fPIC"]
CPU_BASE = CFLAGS + ["-march=x86-64", "-mtune=generic", "-fopenmp"]
VARIANTS = (
    ("cpu_scalar.o", ["-ffp-contract=off", "-DQC_PREFIX=qcs_"]),
    ("cpu_avx2.o", ["-mavx2", "-mfma", "-mf16c", "-DQC_AVX2", "-DQC_PREFIX=qc2_"]),
    ("cpu_avx512.o", ["-mavx512f", "-mavx512dq", "-mavx512bw", "-mavx512vl", "-mfma", "-mf16c",
                      "-DQC_AVX512", "-DQC_PREFIX=qc5_"]),
)


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def _gomp_dir() -> str | None:
    out = subprocess.run(["gcc", "-print-file-name=libgomp.so"], capture_output=True, text=True).stdout.strip()
    return os.path.dirname(out) if out and os.path.isabs(out) else None


def restate_path() -> Path:
    return BUILD / "librestate.so"


def ref_path(hidden: int, ffn: int) -> Path:
    return REF_OUT / f"libqwen_cpu_{hidden}x{ffn}.so"


def build_restate() -> Path:
    BUILD.mkdir(exist_ok=True)
    out = restate_path()
    src = HERE / "restate.c"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        _run(["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-fPIC", "-shared", str(src), "-lm", "-o", str(out)])
    return out


def synth_path() -> Path:
    return BUILD / "libsynth.so"


def build_synth() -> Path:
    """oracle/synth.c (host restatement of the synthetic generator): no multiply-add
    contraction, so every float step rounds as the device's does."""
    BUILD.mkdir(exist_ok=True)
    out = synth_path()
    src = HERE / "synth.c"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
               str(src), "-o", str(out)]
        gomp = _gomp_dir()
        if gomp:
            cmd.append(f"-L{gomp}")
        _run(cmd + ["-lgomp", "-lm"])
    return out


def build_ref(reference_root: Path, force: bool = False) -> list[Path]:
    """Compile the reference CPU MoE at both shapes. Returns the built libraries."""
    qdir = Path(reference_root) / "qwen"
    if not (qdir / "cpu.c").exists():
        raise FileNotFoundError(f"reference CPU sources not found under {qdir}")
    REF_OUT.mkdir(exist_ok=True)
    built = []
    gomp = _gomp_dir()
    for hidden, ffn in SHAPES:
        out = ref_path(hidden, ffn)
        if out.exists() and not force:
            built.append(out)
            continue
        work = REF_OUT / f"tmp_{hidden}x{ffn}"
        if work.exists():
            shutil.rmtree(work)
        work.mkdir()
        try:
            source = qdir / "cpu.c"
            if (hidden, ffn) != (2560, 640):
                text = source.read_text()
                new, n = re.subn(r"enum\s*\{\s*WIDTH=2560,\s*FF=640,",
                                 f"enum {{ WIDTH={hidden}, FF={ffn},", text)
                if n != 1:
                    raise RuntimeError("reference cpu.c shape enum not found exactly once")
                source = work / "cpu.c"
                source.write_text(new)
            objs = []
            for name, flags in VARIANTS:
                obj = work / name
                _run(["gcc", *CPU_BASE, *flags, f"-I{qdir}", "-c", str(source), "-o", str(obj)])
                objs.append(str(obj))
            disp = work / "cpu.o"
            _run(["gcc", *CPU_BASE, f"-I{qdir}", "-c", str(qdir / "cpu_dispatch.c"), "-o", str(disp)])
            objs.append(str(disp))
            link = ["gcc", "-shared", "-pthread", *objs]
            if gomp:
                link.append(f"-L{gomp}")
            _run(link + ["-lgomp", "-lm", "-o", str(out)])
        finally:
            shutil.rmtree(work, ignore_errors=True)
        built.append(out)
    return built


def main(argv: list[str]) -> int:
    build_restate()
    build_synth()
    # the reference tree: $NEBULA_REFERENCE, else a "reference" directory beside the repository
    ref = os.environ.get("NEBULA_REFERENCE") or str(Path(__file__).resolve().parents[2] / "reference")
    if Path(ref, "qwen", "cpu.c").exists():
        for p in build_ref(Path(ref), force="--force" in argv):
            print(p)
    print(restate_path())
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
