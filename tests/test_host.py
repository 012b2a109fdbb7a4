"""Host pipeline pieces (C++ libshoehorn_host.so): the reference's own tests
for parse_size, the solver and GGUF metadata, plus checks of the GGUF writer
and the imatrix loader against gguf-py as an independent implementation."""
import ctypes
import os
import struct
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST_LIB = os.path.join(ROOT, "shoehorn_b200", "libshoehorn_host.so")
CLI = os.path.join(ROOT, "shoehorn_b200", "shoehorn-gpu")
gguf = pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def H():
    L = ctypes.CDLL(HOST_LIB)
    L.shh_parse_size.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]
    L.shh_solve.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64,
                            ctypes.c_void_p]
    L.shh_imatrix_probe.restype = ctypes.c_int64
    L.shh_imatrix_probe.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.POINTER(ctypes.c_int64)]
    L.shh_gguf_rewrite.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
    return L


def parse_size(H, s):
    v = ctypes.c_uint64()
    assert H.shh_parse_size(s.encode(), ctypes.byref(v)) == 0
    return v.value


# main.rs:238-249
def test_bare_small_numbers_read_as_gib(H):
    assert parse_size(H, "16") == 16 << 30
    assert parse_size(H, "0.5") == 1 << 29
    assert parse_size(H, "0") == 0
    assert parse_size(H, "884736") == 884736
    assert parse_size(H, "16GiB") == 16 << 30
    assert parse_size(H, "800MB") == 800_000_000
    assert parse_size(H, "160MiB") == 160 << 20
    v = ctypes.c_uint64()
    assert H.shh_parse_size(b"lots", ctypes.byref(v)) != 0


def solve(H, tensors, budget):
    bytes_, errs, offs = [], [], [0]
    for opts in tensors:
        for b, e in opts:
            bytes_.append(b)
            errs.append(e)
        offs.append(len(bytes_))
    b = np.array(bytes_, np.uint64)
    e = np.array(errs, np.float64)
    o = np.array(offs, np.int64)
    sel = np.zeros(len(tensors), np.int64)
    rc = H.shh_solve(b.ctypes.data, e.ctypes.data, o.ctypes.data, len(tensors), budget, sel.ctypes.data)
    return list(sel) if rc == 1 else None


# solver.rs:125-144
def test_solver_picks_max_quality_when_it_fits(H):
    assert solve(H, [[(10, 5.0), (20, 1.0)], [(10, 5.0), (20, 1.0)]], 100) == [1, 1]


def test_solver_respects_budget(H):
    assert solve(H, [[(10, 5.0), (20, 1.0)], [(10, 5.0), (20, 4.9)]], 30) == [1, 0]


def test_solver_infeasible(H):
    assert solve(H, [[(10, 5.0)]], 5) is None


def test_solver_bisection_and_greedy_fill_budget(H):
    rng = np.random.default_rng(5)
    tensors = []
    for _ in range(40):
        sizes = np.sort(rng.integers(10, 1000, 6))
        errs = np.sort(rng.random(6))[::-1] * 100
        tensors.append(list(zip(sizes.tolist(), errs.tolist())))
    smallest = sum(t[0][0] for t in tensors)
    largest = sum(t[-1][0] for t in tensors)
    budget = (smallest + largest) // 2
    sel = solve(H, tensors, budget)
    used = sum(t[i][0] for t, i in zip(tensors, sel))
    assert used <= budget
    # no single upgrade still fits with a better error (the greedy pass ran to completion)
    slack = budget - used
    for t, i in zip(tensors, sel):
        for b, e in t:
            assert not (b > t[i][0] and e < t[i][1] and b - t[i][0] <= slack)


# e2e_tests.rs:71-115, with gguf-py as the writer of the original and the reader of ours
def test_gguf_metadata_roundtrips_every_value_type(H, tmp_path):
    src, out = str(tmp_path / "kv.gguf"), str(tmp_path / "kv2.gguf")
    w = gguf.GGUFWriter(src, "llama")
    w.add_uint8("t.u8", 7)
    w.add_int8("t.i8", -7)
    w.add_uint16("t.u16", 300)
    w.add_int16("t.i16", -300)
    w.add_uint32("t.u32", 70000)
    w.add_int32("t.i32", -70000)
    w.add_float32("t.f32", 0.25)
    w.add_bool("t.bool", True)
    w.add_string("t.str", "hé\U0001F980")
    w.add_uint64("t.u64", 1 << 40)
    w.add_int64("t.i64", -(1 << 40))
    w.add_float64("t.f64", 0.125)
    w.add_array("t.arr.str", ["a", "b"])
    w.add_array("t.arr.f32", [1.5, -2.5])
    w.add_tensor("output_norm.weight", np.arange(32, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    assert H.shh_gguf_rewrite(src.encode(), out.encode()) == 0
    a, b = gguf.GGUFReader(src), gguf.GGUFReader(out)
    fa = {k: v for k, v in a.fields.items() if not k.startswith("GGUF.")}
    fb = {k: v for k, v in b.fields.items() if not k.startswith("GGUF.")}
    assert list(fa) == list(fb)
    for k in fa:
        assert fa[k].types == fb[k].types, k
        assert [bytes(p.tobytes()) for p in fa[k].parts[-len(fa[k].data):]] == \
               [bytes(p.tobytes()) for p in fb[k].parts[-len(fb[k].data):]], k
    assert np.array_equal(a.tensors[0].data, b.tensors[0].data)
    assert b.tensors[0].name == "output_norm.weight"


def lcg_bf16(seed, n):
    """e2e_tests.rs:10-26: 64-bit LCG, f32 in [-0.5, 0.5), BF16 round to nearest even."""
    s = seed
    out = np.empty(n, np.uint16)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        f = np.float32(np.float32(s >> 33) / np.float32(2.0 ** 31)) - np.float32(0.5)
        u = int(np.float32(f).view(np.uint32))
        out[i] = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return out


def test_synthetic_e2e_fixture_matches_the_reference_generator(tmp_path):
    path = str(tmp_path / "e2e.gguf")
    subprocess.run([CLI, "synth", "e2e", path], check=True, capture_output=True)
    r = gguf.GGUFReader(path)
    names = [t.name for t in r.tensors]
    assert names == ["token_embd.weight", "blk.0.attn_q.weight", "blk.0.ffn_down.weight", "blk.1.attn_q.weight",
                     "output_norm.weight"]
    t = r.tensors[2]  # seed 3, [256, 64]
    got = np.asarray(t.data).reshape(-1).view(np.uint16)[:300]
    assert np.array_equal(got, lcg_bf16(3, 300))


def test_legacy_and_gguf_imatrix_loading(H, tmp_path):
    # legacy: n_entries, then {name_len, name, ncall, nval, f32[nval]}
    p = str(tmp_path / "a.imatrix")
    vals = np.array([2.0, 4.0, 0.0, -1.0, np.nan, 8.0], np.float32)
    with open(p, "wb") as f:
        f.write(struct.pack("<i", 1))
        f.write(struct.pack("<i", 9) + b"blk.0.ffn")
        f.write(struct.pack("<ii", 2, vals.size) + vals.tobytes())
    out = np.zeros(6, np.float32)
    n = ctypes.c_int64()
    assert H.shh_imatrix_probe(p.encode(), b"blk.0.ffn", out.ctypes.data, 6, ctypes.byref(n)) == 1
    # divided by ncall, then non-positive / non-finite replaced by max * 1e-9 (imatrix.rs:95-120)
    want = vals / np.float32(2)
    floor = np.float32(4.0) * np.float32(1e-9)
    want = np.where(np.isfinite(want) & (want > 0), want, floor).astype(np.float32)
    assert np.array_equal(out, want)
    # truncated file
    with open(p, "rb") as f:
        data = f.read()
    with open(p, "wb") as f:
        f.write(data[:-3])
    assert H.shh_imatrix_probe(p.encode(), b"blk.0.ffn", None, 0, ctypes.byref(n)) == -1
    # GGUF imatrix: <name>.in_sum2 / <name>.counts
    g = str(tmp_path / "b.gguf")
    w = gguf.GGUFWriter(g, "imatrix")
    w.add_tensor("blk.1.attn_q.weight.in_sum2", np.array([3.0, 6.0, 9.0, 12.0], np.float32))
    w.add_tensor("blk.1.attn_q.weight.counts", np.array([3.0], np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = np.zeros(4, np.float32)
    assert H.shh_imatrix_probe(g.encode(), b"blk.1.attn_q.weight", out.ctypes.data, 4, ctypes.byref(n)) == 1
    assert np.array_equal(out, np.array([1, 2, 3, 4], np.float32))
