"""The C-ABI library builds for sm_100a, loads on a CPU-only host and
exports exactly the entry points include/afterimage_b200.h declares; host
validation rejects bad arguments before any CUDA call."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

from afterimage_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "afterimage_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(aib_[a-z_0-9]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.load()
    names = declared_functions()
    assert len(names) >= 15, names
    for n in names:
        assert hasattr(L, n), f"{n} declared in the header but not exported"
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == names


def test_library_exports_nothing_else():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.lib_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = sorted({line.split()[-1] for line in out.splitlines()
                       if line.split()[1] in ("T", "W", "i")})
    extra = [s for s in exported if not s.startswith("aib_") and not s.startswith("_init")
             and not s.startswith("_fini")]
    assert extra == [], extra[:20]


@pytest.mark.parametrize("ctype,cname", [(_lib.StreamDesc, "aib_stream_desc"), (_lib.GemvDesc, "aib_gemv_desc"),
                                         (_lib.ArGroup, "aib_ar_group")])
def test_descriptor_layout_matches_header_order(tmp_path, ctype, cname):
    """The ctypes descriptors must have the C compiler's size and field offsets."""
    import subprocess
    fields = [f for f, _ in ctype._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"afterimage_b200.h\"\n"
                   "int main(void){printf(\"%%zu\\n\", sizeof(%s));" % cname
                   + "".join('printf("%%zu\\n", offsetof(%s, %s));' % (cname, f) for f in fields)
                   + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got[0] == ctypes.sizeof(ctype)
    assert got[1:] == [getattr(ctype, f).offset for f in fields]


def test_host_validation_rejects_bad_descriptors_without_a_gpu():
    L = _lib.load()
    d = _lib.StreamDesc()
    d.chunk_size = 0
    d.n_symbols = 10
    d.elem_end = 10
    rc = L.aib_decode_bf16(ctypes.byref(d), None, None)
    assert rc == _lib.AIB_EINVAL
    assert b"chunk_size" in L.aib_last_error()
    d.chunk_size = 16
    d.max_bits = 17
    assert L.aib_decode_bf16(ctypes.byref(d), None, None) == _lib.AIB_EINVAL
    assert b"max_bits" in L.aib_last_error()
    d.max_bits = 8
    d.elem_begin, d.elem_end = 5, 3
    assert L.aib_decode_exponents_u8(ctypes.byref(d), None, None) == _lib.AIB_EINVAL
    # empty range: nothing to do, no CUDA call needed
    d.elem_begin, d.elem_end = 3, 3
    assert L.aib_decode_exponents_u8(ctypes.byref(d), None, None) == _lib.AIB_OK
    assert L.aib_decode_bf16_batch(ctypes.byref(d), 0, None, None) == _lib.AIB_EINVAL
    assert L.aib_decode_bf16_batch(ctypes.byref(d), 17, None, None) == _lib.AIB_EINVAL


def test_gemv_host_validation_without_a_gpu():
    """Every argument check of the fused decode-GEMV runs on the host."""
    L = _lib.load()
    g = _lib.GemvDesc()
    d = g.stream
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 0, None, None) == _lib.AIB_EINVAL
    # no rows: nothing to check or do
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_OK
    d.n_symbols, d.elem_end = 64, 64
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"null x" in L.aib_last_error()
    g.x, g.partial, g.y = 0x1000, 0x2000, 0x3000
    g.x = 0x1004
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"aligned" in L.aib_last_error()
    g.x = 0x1000
    d.chunk_size = 6
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"multiple of 4" in L.aib_last_error()
    d.chunk_size = 64
    g.cols = 100
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"cols" in L.aib_last_error()
    g.cols = 128
    d.n_symbols, d.elem_begin, d.elem_end = 512, 64, 512
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"whole rows" in L.aib_last_error()
    d.elem_begin = 128
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"sign_mantissa" in L.aib_last_error()
    d.sign_mantissa = 0x4000
    d.max_bits = 8
    # the shared stream checks follow (null packed here)
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"packed" in L.aib_last_error()
    # an empty range needs no device
    d.elem_begin = d.elem_end = 256
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_OK


def test_tables_bytes_and_abi_version():
    L = _lib.load()
    assert L.aib_abi_version() == 2
    assert L.aib_tables_bytes() % 16 == 0 and L.aib_tables_bytes() >= 4096 * 8


def test_encoder_entry_points_via_c_abi():
    L = _lib.load()
    bits = np.array([0, 0x8000, 0x7F80, 0xFF80, 0x3F80, 0xBF81, 1, 0x7F], dtype=np.uint16)
    e = np.zeros(8, np.uint8)
    sm = np.zeros(8, np.uint8)
    assert L.aib_split_bf16(bits.ctypes.data, 8, e.ctypes.data, sm.ctypes.data) == 0
    assert list(e) == [(int(b) >> 7) & 0xFF for b in bits]
    assert list(sm) == [(((int(b) >> 15) & 1) << 7) | (int(b) & 0x7F) for b in bits]
    counts = np.zeros(256, np.int64)
    assert L.aib_histogram(e.ctypes.data, 8, counts.ctypes.data) == 0
    assert counts.sum() == 8
    assert L.aib_build_code(counts.ctypes.data, 0, None, None, None) == _lib.AIB_EINVAL


def test_pread_batch_reads_pieces_in_parallel(tmp_path):
    import os
    L = _lib.load()
    data = np.random.default_rng(3).integers(0, 256, 1 << 20, dtype=np.uint8)
    path = tmp_path / "f.bin"
    data.tofile(path)
    fd = os.open(path, os.O_RDONLY)
    try:
        pieces = [(0, 4096), (4096, 70000), (500000, 3), (1048000, 576), (123, 0)]
        dst = np.zeros(sum(n for _, n in pieces), dtype=np.uint8)
        offs, sizes, dests, pos = [], [], [], 0
        for o, n in pieces:
            offs.append(o), sizes.append(n), dests.append(dst.ctypes.data + pos)
            pos += n
        A = ctypes.c_int64 * len(pieces)
        D = ctypes.c_void_p * len(pieces)
        got = ctypes.c_int64(-1)
        assert L.aib_pread_batch(fd, A(*offs), A(*sizes), None, D(*dests), len(pieces), 4,
                                 ctypes.byref(got)) == _lib.AIB_OK
        assert got.value == dst.size
        want = np.concatenate([data[o:o + n] for o, n in pieces])
        assert np.array_equal(dst, want)
        # past the end of the file: short unless min_sizes allows it
        tail = np.zeros(8192, dtype=np.uint8)
        one = (ctypes.c_int64 * 1)
        args = (fd, one((1 << 20) - 100), one(8192))
        assert L.aib_pread_batch(*args, None, (ctypes.c_void_p * 1)(tail.ctypes.data), 1, 2,
                                 ctypes.byref(got)) == _lib.AIB_ESHORT
        assert b"short read" in L.aib_last_error()
        assert L.aib_pread_batch(*args, one(100), (ctypes.c_void_p * 1)(tail.ctypes.data), 1, 2,
                                 ctypes.byref(got)) == _lib.AIB_OK
        assert np.array_equal(tail[:100], data[-100:])
    finally:
        os.close(fd)
    assert L.aib_pread_batch(-1, None, None, None, None, 0, 1, None) == _lib.AIB_EINVAL


def test_wait_timeout_selftest_validates_on_the_host():
    L = _lib.load()
    m = re.search(r"#define AIB_WAIT_LIMIT_POLLS \(1u << (\d+)\)", HEADER.read_text())
    assert m and _lib.WAIT_LIMIT_POLLS == 1 << int(m.group(1))
    status = ctypes.c_void_p(16)  # never dereferenced: each call fails validation first
    assert L.aib_selftest_wait_timeout(0, status, None) == _lib.AIB_EINVAL
    assert L.aib_selftest_wait_timeout(_lib.WAIT_LIMIT_POLLS + 1, status, None) == _lib.AIB_EINVAL
    assert L.aib_selftest_wait_timeout(1, None, None) == _lib.AIB_EINVAL
    assert b"polls" in L.aib_last_error() or b"null" in L.aib_last_error()


def test_decode_tables_unpack_like_the_reference_pair():
    """No device needed: the tables object is a (sym_lut, len_lut) pair that
    also carries the library's table block."""
    import torch
    from afterimage_b200.runtime.gpu_decode_v2 import DecodeTables
    sym, ln, blk = torch.zeros(8, dtype=torch.int32), torch.zeros(8, dtype=torch.int8), torch.zeros(16, dtype=torch.uint8)
    t = DecodeTables(sym, ln, blk, 3)
    a, b = t
    assert isinstance(t, tuple) and len(t) == 2 and a is sym and b is ln
    assert t.block is blk and t.max_bits == 3 and t.sym_lut is sym and t.len_lut is ln


def test_capped_batch_decode_rejects_a_zero_cap_without_a_gpu():
    L = _lib.load()
    d = _lib.StreamDesc()
    assert L.aib_decode_bf16_batch_ctas(ctypes.byref(d), 1, 0, None, None) == _lib.AIB_EINVAL
    assert b"max_ctas" in L.aib_last_error()
