"""The all-resident MoE drop-in inside the reference runtime, on the GPU.

A synthetic one-layer model (target layer 12 with every tensor the reference
loader binds for it, in the product's types and shapes: hidden 2560, FFN 640,
Q4_K gate/up and IQ4_NL down experts, F32 router, Q4_K/IQ4_NL shared expert)
is written as a COB_QWEN_INDEX_V1 index and opened with the reference's own
diagnostic loader (qwen_probe_layer_open, qwen/qwen.c:429-433). moe() - the
drop-in of nebula_b200/integration/qwen_moe.c inside the reference's qwen.c -
runs on 17 verify tokens twice (the second call reuses the experts made
resident by the first). Checked against the CPU checker (the reference's
qc_matmul / qc_moe at 2560/640 plus the restated routing and shared expert):
ids bit-exact, outputs within rel-L2 1e-5 and max-abs 1e-4 * max|ref|.
Needs libqwen_moe_probe.so, which the build step makes where the reference
tree is present."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from conftest import assert_parity
from oracle.blocks import random_blocks

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PROBE = ROOT / "nebula_b200" / "integration" / "_build" / "libqwen_moe_probe.so"
D, FF, HD, T = 2560, 640, 10240, 17

# Layer 12's tensors as the reference loader binds them (qwen/qwen.c:96-106,
# 151-171): name suffix, GGML type, dims (dims[0] = row length).
LAYER12 = (
    ("ffn_gate_exps.weight", 12, (D, FF, 512, 1)), ("ffn_up_exps.weight", 12, (D, FF, 512, 1)),
    ("ffn_down_exps.weight", 20, (FF, D, 512, 1)), ("ffn_gate_inp.weight", 0, (D, 512, 1, 1)),
    ("ffn_gate_shexp.weight", 12, (D, FF, 1, 1)), ("ffn_up_shexp.weight", 12, (D, FF, 1, 1)),
    ("ffn_down_shexp.weight", 20, (FF, D, 1, 1)), ("ffn_gate_inp_shexp.weight", 0, (D, 1, 1, 1)),
    ("hc_attn_norm.weight", 0, (HD, 1, 1, 1)), ("hc_attn_down.weight", 12, (HD, 320, 1, 1)),
    ("hc_attn_up.weight", 20, (320, HD, 1, 1)), ("hc_attn_inject.weight", 0, (HD, 4, 1, 1)),
    ("hc_ffn_norm.weight", 0, (HD, 1, 1, 1)), ("hc_ffn_down.weight", 12, (HD, 320, 1, 1)),
    ("hc_ffn_up.weight", 20, (320, HD, 1, 1)), ("hc_ffn_inject.weight", 0, (HD, 4, 1, 1)),
    ("attn_qkv.weight", 12, (D, 10240, 1, 1)), ("attn_gate.weight", 12, (D, 6144, 1, 1)),
    ("ssm_alpha.weight", 0, (D, 48, 1, 1)), ("ssm_beta.weight", 0, (D, 48, 1, 1)), ("ssm_a", 0, (48, 1, 1, 1)),
    ("ssm_dt.bias", 0, (48, 1, 1, 1)), ("ssm_conv1d.weight", 0, (4, 10240, 1, 1)),
    ("ssm_norm.weight", 0, (128, 1, 1, 1)), ("ssm_out.weight", 12, (6144, D, 1, 1)),
)


def tensor_bytes(rng, typ, dims):
    rows = dims[1] * dims[2] * dims[3]
    if typ == 0:
        return rng.normal(0, 0.02, rows * dims[0]).astype("<f4").view(np.uint8)
    return random_blocks(rng, typ, rows, dims[0], d=0.0002, dmin=0.0001).reshape(-1)


@pytest.fixture(scope="module")
def layer_index(tmp_path_factory):
    if not PROBE.exists():
        pytest.skip("libqwen_moe_probe.so not built (the reference tree was absent at build time)")
    d = tmp_path_factory.mktemp("qwen_layer12")
    rng = np.random.default_rng(1212)
    blobs, recs, off = [], [], 0
    for suffix, typ, dims in LAYER12:
        b = tensor_bytes(rng, typ, dims)
        recs.append((f"blk.12.{suffix}", off, b.nbytes, typ, dims))
        blobs.append(b)
        off += (b.nbytes + 255) // 256 * 256
    data = np.zeros(off, np.uint8)
    for (name, o, n, typ, dims), b in zip(recs, blobs):
        data[o:o + n] = b
    wpath = d / "layer12.bin"
    data.tofile(wpath)
    text = "COB_QWEN_INDEX_V1\nVERIFIED 1\n" + " ".join(["1"] * 35) + " 0\n" + f"FILE\t0\t{off}\t{wpath}\n"
    for name, o, n, typ, dims in recs:
        text += f"TENSOR\t{name}\t0\t{o}\t{n}\t{typ}\t" + "\t".join(map(str, dims)) + "\n"
    (d / "index.txt").write_text(text)
    tensors = {name.split(".", 2)[2]: (data[o:o + n], typ) for name, o, n, typ, dims in recs}
    return d / "index.txt", tensors


def test_all_resident_moe_inside_reference_runtime(layer_index, ref2560, restate):
    from oracle import oracle as orc
    path, t = layer_index
    lib = C.CDLL(str(PROBE))
    lib.nebula_probe_moe.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.POINTER(C.c_double)]
    lib.nebula_probe_moe.restype = C.c_int
    lib.qwen_last_error.restype = C.c_char_p
    x = np.random.default_rng(7).normal(0, 1, (2, T, D)).astype(np.float32)
    out = np.zeros((2, T, D), np.float32)
    ids = np.zeros((2, T, 10), np.int32)
    w = np.zeros((2, T, 10), np.float32)
    uploaded = C.c_double()
    rc = lib.nebula_probe_moe(str(path).encode(), 12, T, x.ctypes.data, out.ctypes.data, ids.ctypes.data,
                              w.ctypes.data, C.byref(uploaded))
    assert rc == 0, lib.qwen_last_error().decode()
    expert_bytes = sum(t[n][0].nbytes for n in ("ffn_gate_exps.weight", "ffn_up_exps.weight",
                                                 "ffn_down_exps.weight"))
    assert uploaded.value == expert_bytes  # all 512 experts of the three matrices, uploaded once
    router = t["ffn_gate_inp.weight"][0].view(np.float32).reshape(512, D)
    shared = (t["ffn_gate_shexp.weight"][0], 12, t["ffn_up_shexp.weight"][0], 12, t["ffn_down_shexp.weight"][0], 20,
              t["ffn_gate_inp_shexp.weight"][0].view(np.float32).reshape(1, D))
    for call in range(2):
        ref, ref_ids, _, _ = orc.moe_layer(ref2560, restate, x[call], router, t["ffn_gate_exps.weight"][0], 12,
                                           t["ffn_up_exps.weight"][0], 12, t["ffn_down_exps.weight"][0], 20,
                                           shared=shared)
        np.testing.assert_array_equal(ids[call], ref_ids, err_msg=f"call {call}: routing")
        assert_parity(out[call], ref, f"call {call}")
