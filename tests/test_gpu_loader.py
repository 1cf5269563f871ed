"""Loading an all-resident MoE layer through the C ABI: a COB_QWEN_INDEX_V1
index over a weights file holding one layer's 512 experts (gate, up, down,
router), qg_index_tensor to find them in the mapped file, and
qg_upload_experts to bring all 512 experts (or one rank's snake-order share)
into device memory. The uploaded bytes equal the file's, and a layer run on
them equals the same layer run on weights generated in place."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, F, E = 2048, 512, 512
ROW_H, ROW_F = H // 256 * 144, F // 256 * 144


@pytest.fixture(scope="module")
def layer_files(gpu_lib, tmp_path_factory):
    from nebula_b200 import lib as L
    d = tmp_path_factory.mktemp("index")
    mats = {"ffn_gate_exps": (L.synth_weights(12, E * F, H, 601), 12, (H, F, E, 1)),
            "ffn_up_exps": (L.synth_weights(12, E * F, H, 602), 12, (H, F, E, 1)),
            "ffn_down_exps": (L.synth_weights(12, E * H, F, 603), 12, (F, H, E, 1)),
            "ffn_gate_inp": (L.synth_weights(0, E, H, 604), 0, (H, E, 1, 1))}
    blobs, lines, off = [], [], 4096  # tensors start past a leading gap, 4 KiB aligned
    for name, (dev, typ, dims) in mats.items():
        b = dev.get()
        lines.append((f"blk.12.{name}.weight", off, b.nbytes, typ, dims))
        blobs.append((off, b))
        off = (off + b.nbytes + 4095) // 4096 * 4096
    data = np.zeros(off, np.uint8)
    for o, b in blobs:
        data[o:o + b.nbytes] = b
    wpath = d / "weights.bin"
    data.tofile(wpath)
    text = "COB_QWEN_INDEX_V1\nVERIFIED 1\n" + " ".join(["1"] * 35) + " 0\n"
    text += f"FILE\t0\t{off}\t{wpath}\n"
    for name, o, n, typ, dims in lines:
        text += f"TENSOR\t{name}\t0\t{o}\t{n}\t{typ}\t" + "\t".join(map(str, dims)) + "\n"
    (d / "index.txt").write_text(text)
    return d / "index.txt", {k: v[0] for k, v in mats.items()}


def tensor(L, ix, name):
    host, typ, nbytes = C.c_void_p(), C.c_int(), C.c_uint64()
    dims = (C.c_uint64 * 4)()
    L.call("index_tensor", ix, name.encode(), C.byref(host), C.byref(typ), dims, C.byref(nbytes))
    return host.value, typ.value, list(dims), nbytes.value


def test_index_bulk_upload_all_experts_and_run_layer(layer_files):
    from nebula_b200 import lib as L
    path, gen = layer_files
    ix, msg = C.c_void_p(), C.create_string_buffer(256)
    L.call("index_open", str(path).encode(), C.byref(ix), msg, 256)
    up = L.load().qg_upload_create(3 * 589_824)
    assert up
    try:
        loaded = {}
        for name in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"):
            host, typ, dims, nbytes = tensor(L, ix, f"blk.12.{name}.weight")
            assert typ == 12 and dims[2] == E
            dst = L.Device(nbytes=nbytes)
            L.call("upload_experts", up, dst.p, host, nbytes // E, None, E)
            loaded[name] = dst
        host, _, _, nbytes = tensor(L, ix, "blk.12.ffn_gate_inp.weight")
        router = L.Device(nbytes=nbytes)
        L.call("write", router.p, host, nbytes)
        L.call("sync")
        assert L.load().qg_upload_seconds(up) > 0
        for name, dst in loaded.items():
            np.testing.assert_array_equal(dst.get(), gen[name].get(), err_msg=name)
        # one layer on the loaded weights equals the layer on the generated ones
        T = 17
        x = L.synth_normal(T * H, 605)
        outs = []
        for g, u, dn, r in ((loaded["ffn_gate_exps"], loaded["ffn_up_exps"], loaded["ffn_down_exps"], router),
                            (gen["ffn_gate_exps"], gen["ffn_up_exps"], gen["ffn_down_exps"], gen["ffn_gate_inp"])):
            out = L.Device.empty((T, H), np.float32)
            ids = L.Device.empty((T, 10), np.int32)
            ws = L.workspace(T, H, F)
            L.call("moe_layer", out.p, ids.p, None, x.p, T, r.p, None, g.p, 12, u.p, 12, dn.p, 12,
                   None, 12, None, 12, None, 12, None, H, F, ws.p)
            outs.append((out.get(), ids.get()))
        np.testing.assert_array_equal(outs[0][1], outs[1][1])
        np.testing.assert_array_equal(outs[0][0], outs[1][0])
    finally:
        L.load().qg_upload_destroy(up)
        L.load().qg_index_close(ix)


def test_bulk_upload_of_one_ranks_experts(layer_files):
    """Expert parallelism: rank 3 of 8 loads its 64 experts (snake order of a
    ranking) straight from the mapped file, as ep.extract_experts copies them."""
    from nebula_b200 import ep
    from nebula_b200 import lib as L
    path, gen = layer_files
    ix, msg = C.c_void_p(), C.create_string_buffer(256)
    L.call("index_open", str(path).encode(), C.byref(ix), msg, 256)
    up = L.load().qg_upload_create(8 << 20)  # several experts per pinned block
    try:
        owner = ep.snake_owner(np.random.default_rng(3).permutation(E), 8)
        _, experts = ep.local_map(owner, 3)
        lst = np.array(experts, np.int32)
        host, _, _, nbytes = tensor(L, ix, "blk.12.ffn_down_exps.weight")
        dst = L.Device(nbytes=len(experts) * (nbytes // E))
        L.call("upload_experts", up, dst.p, host, nbytes // E, lst.ctypes.data, len(experts))
        L.call("sync")
        ref = ep.extract_experts(gen["ffn_down_exps"], experts, H, ROW_F)
        np.testing.assert_array_equal(dst.get(), ref.get())
    finally:
        L.load().qg_upload_destroy(up)
        L.load().qg_index_close(ix)
