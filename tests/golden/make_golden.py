"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's own
code on seeded inputs (test infrastructure; rerun only where the reference
tree is present):

* formats.npz - packed rows of every GGML type the reference decodes and the
  values the reference's NumPy decoder ``qwen/quant.py:dequant`` gives them;
* matmul.npz  - ``qc_matmul`` outputs (reference ``qwen/cpu.c:119-148``,
  compiled unmodified into oracle/_ref) for F32 / Q4_K / IQ4_NL rows;
* moe.npz     - ``qc_moe`` outputs (``qwen/cpu.c:235-261``) at the product
  shape 2560/640 and the benchmark shape 2048/512, pinned by SHA-256 (plus
  the first output row for diagnostics).

Inputs are regenerated from their seeds (numpy PCG64) and pinned by a
SHA-256 of their bytes, so the fixtures stay small.

Usage: python tests/golden/make_golden.py [reference_root]
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import build as obuild  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from oracle.blocks import random_blocks  # noqa: E402

OUT = Path(__file__).resolve().parent
TYPES = (0, 1, 30, 2, 6, 7, 8, 12, 13, 14, 20)

MOE_CASES = (  # (hidden, ffn, gate_type, down_type, seed)
    (2560, 640, 12, 20, 91011),
    (2048, 512, 12, 12, 7),
    (2048, 512, 12, 20, 8),
    (2048, 512, 20, 20, 9),
)
MOE_EXPERTS = 12
MOE_TOKENS = (1, 5, 17, 18)


def moe_case_inputs(hidden, ffn, gt, dt, seed):
    """Expert matrices, x, ids and weights of one moe.npz case (deterministic)."""
    rng = np.random.default_rng(seed)
    gate = random_blocks(rng, gt, MOE_EXPERTS * ffn, hidden, d=0.0002, dmin=0.0001)
    up = random_blocks(rng, gt, MOE_EXPERTS * ffn, hidden, d=0.0002, dmin=0.0001)
    down = random_blocks(rng, dt, MOE_EXPERTS * hidden, ffn, d=0.0002, dmin=0.0001)
    nt = max(MOE_TOKENS)
    x = rng.normal(0, 0.2, (nt, hidden)).astype(np.float32)
    ids = np.stack([rng.choice(MOE_EXPERTS, 10, replace=False) for _ in range(nt)]).astype(np.int32)
    w = rng.uniform(0.01, 0.2, (nt, 10)).astype(np.float32)
    # omitted routes as qg_prune_routes writes them: -e-2 with weight 0
    for t in range(0, nt, 3):
        ids[t, 9] = -ids[t, 9] - 2
        w[t, 9] = 0.0
    return gate, up, down, x, ids, w


MATMUL_SHAPES = ((7, 512), (5, 2048))
MATMUL_TOKENS = (1, 3, 4, 5, 17, 18)


def matmul_case_inputs(typ, rows, cols):
    """Weights and the token batches of one matmul.npz case (deterministic)."""
    rng = np.random.default_rng(1000 * typ + cols)
    w = random_blocks(rng, typ, rows, cols)
    xs = [rng.normal(0, 0.2, (nt, cols)).astype(np.float32) for nt in MATMUL_TOKENS]
    return w, xs


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main(reference_root: Path) -> None:
    spec = importlib.util.spec_from_file_location("ref_quant", reference_root / "qwen" / "quant.py")
    ref_quant = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref_quant)
    obuild.build_ref(reference_root)

    # formats: reference NumPy decoder on random legal blocks
    rng = np.random.default_rng(20240531)
    fmt = {}
    for typ in TYPES:
        rows, cols = 3, 512
        packed = random_blocks(rng, typ, rows, cols, d=0.002, dmin=0.001)
        fmt[f"packed_{typ}"] = packed
        fmt[f"values_{typ}"] = ref_quant.dequant(packed.tobytes(), typ, rows, cols).astype(np.float32)
    np.savez_compressed(OUT / "formats.npz", **fmt)

    # matmul: reference qc_matmul
    ref = orc.RefCPU(2048, 512)
    mm = {}
    for typ in (0, 12, 20):
        for rows, cols in MATMUL_SHAPES:
            w, xs = matmul_case_inputs(typ, rows, cols)
            mm[f"sha_{typ}_{cols}"] = np.array(digest(w, *xs))
            for nt, x in zip(MATMUL_TOKENS, xs):
                mm[f"out_{typ}_{cols}_{nt}"] = ref.matmul(w, typ, rows, cols, x, threads=2)
    mm["backend"] = np.array(ref.backend())
    np.savez_compressed(OUT / "matmul.npz", **mm)

    # moe: reference qc_moe
    moe = {}
    for hidden, ffn, gt, dt, seed in MOE_CASES:
        refs = orc.RefCPU(hidden, ffn)
        gate, up, down, x, ids, w = moe_case_inputs(hidden, ffn, gt, dt, seed)
        key = f"{hidden}_{ffn}_{gt}_{dt}"
        moe[f"sha_{key}"] = np.array(digest(gate, up, down, x, ids, w))
        for nt in MOE_TOKENS:
            out = refs.moe(x[:nt], ids[:nt], w[:nt], gate, gt, up, gt, down, dt, threads=2)
            # the full output is pinned by digest; its first row is kept for diagnostics
            moe[f"outsha_{key}_{nt}"] = np.array(digest(out))
            moe[f"row0_{key}_{nt}"] = out[0]
    np.savez_compressed(OUT / "moe.npz", **moe)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    # the reference tree: argv[1], $NEBULA_REFERENCE, else a "reference" directory beside the repository
    root = Path(sys.argv[1] if len(sys.argv) > 1 else
                os.environ.get("NEBULA_REFERENCE") or Path(__file__).resolve().parents[3] / "reference")
    main(root)
