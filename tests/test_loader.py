"""Host-side loading entry points (no GPU needed): the COB_QWEN_INDEX_V1 weight
index reader (the format and checks of qwen/qwen.c:108-146) and the QROUTE1
route-trace reader (qwen/qwen.c:87-94,638-646), through the C ABI."""
import ctypes as C
import struct

import numpy as np
import pytest

INVALID, NOT_FOUND = 1, 301  # cudaErrorInvalidValue, cudaErrorFileNotFound
Q4K_ROW_256 = 144


@pytest.fixture(scope="module")
def lib():
    from nebula_b200 import lib as L
    return L.load()


def header(vocab0=5):
    nums = [1, 2, 3] + list(range(10, 26)) + [vocab0] + list(range(101, 116)) + [-1]
    return "COB_QWEN_INDEX_V1\nVERIFIED 1\n" + " ".join(map(str, nums)) + "\n"


def write_weights(tmp_path, nbytes=4096, seed=0):
    data = np.random.default_rng(seed).integers(0, 256, nbytes, dtype=np.uint8)
    path = tmp_path / "w0.bin"
    path.write_bytes(data.tobytes())
    return path, data


def open_index(lib, path):
    ix, msg = C.c_void_p(), C.create_string_buffer(512)
    rc = lib.qg_index_open(str(path).encode(), C.byref(ix), msg, 512)
    return rc, ix, msg.value.decode()


def test_index_reads_files_and_tensors(lib, tmp_path):
    wpath, data = write_weights(tmp_path)
    text = header() + f"FILE\t0\t{data.nbytes}\t{wpath}\n\n"
    text += f"TENSOR\tblk.12.ffn_gate_exps.weight\t0\t128\t{Q4K_ROW_256 * 8}\t12\t256\t4\t2\t1\n"
    text += "TENSOR\tblk.12.ffn_gate_inp.weight\t0\t2048\t1024\t0\t256\t1\t1\t1\n"
    (tmp_path / "index.txt").write_text(text)
    rc, ix, msg = open_index(lib, tmp_path / "index.txt")
    assert rc == 0, msg
    try:
        host, typ = C.c_void_p(), C.c_int()
        dims, nbytes = (C.c_uint64 * 4)(), C.c_uint64()
        assert lib.qg_index_tensor(ix, b"blk.12.ffn_gate_exps.weight", C.byref(host), C.byref(typ), dims,
                                   C.byref(nbytes)) == 0
        assert (typ.value, list(dims), nbytes.value) == (12, [256, 4, 2, 1], 1152)
        assert C.string_at(host.value, 1152) == data[128:128 + 1152].tobytes()
        assert lib.qg_index_tensor(ix, b"blk.12.ffn_gate_inp.weight", C.byref(host), C.byref(typ), dims,
                                   C.byref(nbytes)) == 0
        assert C.string_at(host.value, 1024) == data[2048:3072].tobytes()
        assert lib.qg_index_tensor(ix, b"blk.13.ffn_gate_exps.weight", C.byref(host), None, None, None) == INVALID
    finally:
        lib.qg_index_close(ix)


@pytest.mark.parametrize("case,code", [
    ("version", INVALID), ("unverified", INVALID), ("vocab0", INVALID), ("short_header", INVALID),
    ("file_size", NOT_FOUND), ("file_missing", NOT_FOUND), ("file_twice", INVALID),
    ("tensor_bytes", INVALID), ("tensor_range", INVALID), ("tensor_twice", INVALID),
    ("tensor_file", INVALID), ("tensor_ragged", INVALID), ("junk", INVALID)])
def test_index_rejects_malformed(lib, tmp_path, case, code):
    wpath, data = write_weights(tmp_path)
    n = data.nbytes
    good_t = f"TENSOR\tt\t0\t0\t{Q4K_ROW_256}\t12\t256\t1\t1\t1\n"
    parts = {"head": header(), "file": f"FILE\t0\t{n}\t{wpath}\n", "tensor": good_t}
    if case == "version":
        parts["head"] = header().replace("V1", "V2", 1)
    elif case == "unverified":
        parts["head"] = header().replace("VERIFIED 1", "VERIFIED 0")
    elif case == "vocab0":
        parts["head"] = header(vocab0=0)
    elif case == "short_header":
        parts["head"] = "\n".join(header().split("\n")[:2]) + "\n1 2 3\n"
    elif case == "file_size":
        parts["file"] = f"FILE\t0\t{n + 1}\t{wpath}\n"
    elif case == "file_missing":
        parts["file"] = f"FILE\t0\t{n}\t{tmp_path / 'absent.bin'}\n"
    elif case == "file_twice":
        parts["file"] += parts["file"]
    elif case == "tensor_bytes":
        parts["tensor"] = f"TENSOR\tt\t0\t0\t{Q4K_ROW_256 + 1}\t12\t256\t1\t1\t1\n"
    elif case == "tensor_range":
        parts["tensor"] = f"TENSOR\tt\t0\t{n - 100}\t{Q4K_ROW_256}\t12\t256\t1\t1\t1\n"
    elif case == "tensor_twice":
        parts["tensor"] += good_t
    elif case == "tensor_file":
        parts["tensor"] = good_t.replace("TENSOR\tt\t0", "TENSOR\tt\t3")
    elif case == "tensor_ragged":
        parts["tensor"] = f"TENSOR\tt\t0\t0\t{Q4K_ROW_256}\t12\t200\t1\t1\t1\n"
    elif case == "junk":
        parts["tensor"] += "WEIGHTS\tt\n"
    (tmp_path / "index.txt").write_text(parts["head"] + parts["file"] + parts["tensor"])
    rc, ix, msg = open_index(lib, tmp_path / "index.txt")
    assert rc == code and not ix.value, (case, rc, msg)
    assert msg


def write_trace(path, records, magic=b"QROUTE1\n", cut=0):
    blob = bytearray(magic)
    for layer, pos, ids, w in records:
        nt = ids.shape[0]
        blob += struct.pack("<3I", layer, pos, nt)
        blob += np.ascontiguousarray(ids, "<i4").tobytes() + np.ascontiguousarray(w, "<f4").tobytes()
    path.write_bytes(bytes(blob[:len(blob) - cut]))


def read_all(lib, path, capacity=64):
    tr = C.c_void_p()
    rc = lib.qg_route_trace_open(str(path).encode(), C.byref(tr))
    if rc:
        return rc, []
    out = []
    try:
        ids = np.zeros((capacity, 10), np.int32)
        w = np.zeros((capacity, 10), np.float32)
        while True:
            layer, pos, nt = C.c_int(), C.c_int(), C.c_int()
            rc = lib.qg_route_trace_next(tr, C.byref(layer), C.byref(pos), C.byref(nt), ids.ctypes.data,
                                         w.ctypes.data, capacity)
            if rc or nt.value == 0:
                return rc, out
            out.append((layer.value, pos.value, ids[:nt.value].copy(), w[:nt.value].copy()))
    finally:
        lib.qg_route_trace_close(tr)


def test_route_trace_round_trip(lib, tmp_path):
    rng = np.random.default_rng(5)
    recs = [(l, p, rng.integers(-1, 512, (nt, 10)).astype(np.int32), rng.random((nt, 10)).astype(np.float32))
            for l, p, nt in ((0, 0, 17), (1, 0, 17), (47, 17, 3), (12, 4096, 64))]
    write_trace(tmp_path / "r.bin", recs)
    rc, got = read_all(lib, tmp_path / "r.bin")
    assert rc == 0 and len(got) == len(recs)
    for (l, p, i, w), (gl, gp, gi, gw) in zip(recs, got):
        assert (l, p) == (gl, gp)
        np.testing.assert_array_equal(i, gi)
        np.testing.assert_array_equal(w, gw)


def test_route_trace_rejects_bad_input(lib, tmp_path):
    rec = [(3, 0, np.zeros((5, 10), np.int32), np.zeros((5, 10), np.float32))]
    write_trace(tmp_path / "magic.bin", rec, magic=b"QROUTE2\n")
    assert read_all(lib, tmp_path / "magic.bin")[0] == INVALID
    write_trace(tmp_path / "cut.bin", rec, cut=7)
    assert read_all(lib, tmp_path / "cut.bin")[0] == INVALID
    write_trace(tmp_path / "cap.bin", rec)
    assert read_all(lib, tmp_path / "cap.bin", capacity=4)[0] == INVALID
    assert read_all(lib, tmp_path / "absent.bin")[0] == NOT_FOUND
