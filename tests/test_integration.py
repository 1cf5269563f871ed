"""The drop-in into the reference model runtime, on the CPU (needs the
reference tree; skipped without it).

* The link recipe (nebula_b200/integration/build.py) builds libqwen.so from
  the reference's qwen.c / gpu.cu / ssd.c / CPU objects and this library, as
  qwen/Makefile:43-45 links it: every symbol qwen/gpu.h declares and every
  qwen_* entry of qwen/qwen.h is defined, and each qg_* this library provides
  is weak in the reference's GPU object, so this library's definition is the
  one linked.
* The all-resident moe() (nebula_b200/integration/qwen_moe.c) runs inside the
  reference runtime with inert GPU stand-ins (tests/integration/moe_stub.c, the
  pattern of qwen/test_handoffs.c)."""
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "nebula_b200" / "integration"))
import build as ibuild  # noqa: E402

QDIR = ibuild.reference_root() / "qwen"
pytestmark = pytest.mark.skipif(not (QDIR / "qwen.c").exists(), reason="reference tree not present")


@pytest.fixture(scope="module")
def built():
    return ibuild.build(harness=False)


def symbols(path, *flags):
    out = subprocess.run(["nm", *flags, str(path)], capture_output=True, text=True, check=True).stdout
    return {f[-1]: f[-2] for f in (line.split() for line in out.splitlines()) if len(f) >= 2}


def test_libqwen_defines_every_reference_entry_point(built):
    dyn = symbols(built["libqwen.so"], "-D", "--defined-only")
    gpu_h = set(re.findall(r"\b(qg_[a-z0-9_]+)\s*\(", (QDIR / "gpu.h").read_text()))
    qwen_h = set(re.findall(r"\b(qwen_[a-z0-9_]+)\s*\(", (QDIR / "qwen.h").read_text()))
    assert len(gpu_h) > 40 and len(qwen_h) > 20
    assert sorted(gpu_h - set(dyn)) == []
    assert sorted(qwen_h - set(dyn)) == []
    # this library's additions are there too
    assert {"qg_moe_layer", "qg_moe_workspace_bytes", "qg_upload_experts"} <= set(dyn)


def test_moe_path_symbols_are_this_librarys(built):
    weak = symbols(ibuild.OUT / "gpu_ref_weak.o", "-g", "--defined-only")
    weakened = (ibuild.OUT / "weakened_symbols.txt").read_text().split()
    for name in ("qg_route", "qg_matmul", "qg_moe_map", "qg_moe_reduce", "qg_mtp_moe", "qg_graph_begin", "qg_zero"):
        assert name in weakened and weak[name] == "W", name
    # attention and the other non-MoE kernels stay the reference's (strong)
    assert weak["qg_attention"] == "T" and weak["qg_hc_write"] == "T"
    ours = {}
    from nebula_b200 import build as nbuild
    for src in nbuild.sources():
        ours.update(symbols(nbuild.OBJ / (src.stem + ".o"), "-g", "--defined-only"))
    for name in weakened:
        assert ours.get(name) == "T", name


def test_moe_drop_in_with_stub_gpu(built, tmp_path):
    exe = tmp_path / "moe_stub"
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-ffunction-sections", "-fdata-sections",
           f"-I{ibuild.OUT}", f"-I{QDIR}", f"-I{ibuild.HERE}", str(ROOT / "tests" / "integration" / "moe_stub.c"),
           "-Wl,--gc-sections", "-lm", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, env={**os.environ})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "passed" in r.stdout
