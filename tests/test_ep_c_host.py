"""Expert parallelism from a plain C host (tests/integration/ep_c_host.c).

The C program forks one process per GPU, exchanges the workspaces' IPC
handles through shared memory, and checks qg_moe_layer_ep against
qg_moe_layer on the full layer (ids bit for bit, output within rel-L2 1e-5)
over verify batches of 17, 5 and 17 tokens on one workspace. It uses only the
C ABI of include/gpu.h and cudaSetDevice.

* CPU: the program compiles and links against the built library with -Wall
  -Wextra -Werror.
* GPU (two or more devices): it runs with two ranks and every rank passes."""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "integration" / "ep_c_host.c"
LIB = ROOT / "nebula_b200" / "libqwen_gpu.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _build(out: Path) -> Path:
    if not LIB.exists():
        pytest.skip("libqwen_gpu.so not built")
    exe = out / "ep_c_host"
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}", str(SRC),
           f"-L{LIB.parent}", "-lqwen_gpu", f"-Wl,-rpath,{LIB.parent}", f"-L{CUDA / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{CUDA / 'lib64'}", "-lm", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_ep_c_host_builds(tmp_path):
    assert _build(tmp_path).exists()


def _gpus() -> int:
    r = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True)
    return r.stdout.count("GPU ") if r.returncode == 0 else 0


@pytest.mark.gpu
def test_ep_c_host_two_ranks(tmp_path):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    exe = _build(tmp_path)
    r = subprocess.run([str(exe), "2"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count(" ok") == 6 and "all ranks passed" in r.stdout, r.stdout
