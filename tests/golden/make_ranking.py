"""Writes tests/golden/expert_ranking.npz from the reference's per-layer hot-expert
ranking (qwen/expert_ranking.json), for the benchmark's routing skew and the
expert-parallel placement.

The reference checks the file against a pinned digest before using it
(qwen/storage.py:7, RANKING_SHA256; loader at qwen/storage.py:29-36) and
requires every layer's list to be a permutation of the 512 experts; this
script applies the same two checks and keeps both lists the file holds:
"generation" (decode / verify traffic) and "prefill", 48 layers x 512 expert
ids each, hottest first. The GPU machines have no reference tree, so the
arrays travel as this small fixture, with the digest of the source file.

Run from the repository root:
    python tests/golden/make_ranking.py [reference_root]
"""
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "expert_ranking.npz"
RANKING_SHA256 = "3f698494cb9c0e1d4882b60bbde60cdbe10ca371be86a2a1470a3e87b7571855"  # qwen/storage.py:7
LAYERS, EXPERTS = 48, 512


def main(root: Path) -> None:
    raw = (root / "qwen" / "expert_ranking.json").read_bytes()
    digest = hashlib.sha256(raw).hexdigest()
    if digest != RANKING_SHA256:
        raise SystemExit(f"expert_ranking.json digest {digest} differs from the reference's pinned digest")
    doc = json.loads(raw)
    arrays = {}
    for key in ("generation", "prefill"):
        rows = doc[key]
        if len(rows) != LAYERS or any(sorted(r) != list(range(EXPERTS)) for r in rows):
            raise SystemExit(f"{key}: expected a permutation of the 512 experts for each of 48 layers")
        arrays[key] = np.array(rows, dtype=np.int16)
    np.savez_compressed(OUT, sha256=np.array(digest), **arrays)
    print("wrote", OUT)


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else
              os.environ.get("NEBULA_REFERENCE") or Path(__file__).resolve().parents[3] / "reference"))
