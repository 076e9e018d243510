"""CPU checks of the C ABI: the library loads, exports every symbol the headers
declare, and rejects bad arguments before touching a GPU."""
import ctypes as C
import glob
import os
import re

import pytest

from spindle_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"^SG_API\s+[\w\s\*]+?\b(sg_\w+)\s*\(", src, re.M))
    return names


def test_every_declared_symbol_is_exported():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 19
    for n in names:
        assert hasattr(lib, n), n
    # and the Python binding knows each one's signature
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_library_is_self_contained():
    out = os.popen("ldd %s" % _lib.LIB_PATH).read()
    assert "libcudart" not in out  # static runtime: no loader-path dependence
    assert "libcuda." not in out   # driver calls come through cudaGetDriverEntryPoint


@pytest.mark.gpu
def test_library_kernels_are_sm100(dev):
    # the architecture the runtime loaded the kernels for, as it reports it
    v = C.c_int32()
    assert _lib.load().sg_binary_version(C.byref(v)) == 0
    assert v.value == 100


def test_row_bytes_and_supports():
    lib = _lib.load()
    out = C.c_uint64()
    for dt, cols, want in [(12, 4096, 2304), (14, 1024, 840), (8, 64, 68), (0, 3, 12), (1, 5, 10)]:
        assert lib.sg_row_bytes(dt, cols, C.byref(out)) == 0 and out.value == want
    assert lib.sg_row_bytes(12, 100, C.byref(out)) == 3
    assert lib.sg_row_bytes(99, 256, C.byref(out)) == 2
    m = _lib.SgMat(12, 0, 0, 1024, 8)
    assert lib.sg_supports(C.byref(m)) == 1
    lib.sg_set_int_kernels(0)
    assert lib.sg_supports(C.byref(m)) == 0
    lib.sg_set_int_kernels(1)
    assert lib.sg_supports(C.byref(_lib.SgMat(14, 0, 0, 1000, 8))) == 0
    assert lib.sg_supports(C.byref(_lib.SgMat(8, 0, 0, 1024, 8))) == 0


def test_invalid_arguments_fail_before_the_gpu():
    lib = _lib.load()
    q = _lib.SgQ8K(None, None, None, 1024)
    outs = (C.c_void_p * 1)(0x1000)
    fake = C.c_void_p(0x100000)
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(1, 0, 0, 1024, 4)), C.byref(q), outs, 1, 0, 4, None) == 2
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 0, 1000, 4)), C.byref(q), outs, 1, 0, 4, None) == 3
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 0, 1024, 4)), C.byref(q), outs, 1, 0, 5, None) == 1
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 8, 1024, 4)), C.byref(q), outs, 1, 3, 2, None) == 1
    assert lib.sg_matmul_rows(C.c_void_p(0x100008), C.byref(_lib.SgMat(12, 0, 0, 1024, 4)), C.byref(q), outs, 1,
                              0, 4, None) == 4
    # empty range / no vectors: nothing to do
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 0, 1024, 4)), C.byref(q), outs, 1, 2, 2, None) == 0
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 0, 1024, 4)), C.byref(q), outs, 0, 0, 4, None) == 0
    # Q8K descriptor with null buffers
    assert lib.sg_matmul_rows(fake, C.byref(_lib.SgMat(12, 0, 0, 1024, 4)), C.byref(q), outs, 1, 0, 4, None) == 1
    assert lib.sg_q8k_quantize(fake, 1000, 1, 1000, C.byref(q), None) == 1
    assert lib.sg_quantize_weights(0, fake, 4, 256, fake, None) == 2
    assert lib.sg_quantize_weights(12, fake, 4, 100, fake, None) == 3
    assert lib.sg_status_string(4) == b"misaligned device pointer"


def test_q8k_layout():
    lib = _lib.load()
    q = _lib.SgQ8K()
    assert lib.sg_q8k_bytes(1024) == 16 + 1024 + 128
    assert lib.sg_q8k_view(C.c_void_p(0x10000), 1024, C.byref(q)) == 0
    assert (q.d, q.qs, q.bsums, q.n) == (0x10000, 0x10010, 0x10410, 1024)
    assert lib.sg_q8k_view(C.c_void_p(0x10004), 1024, C.byref(q)) == 4


def test_scratch_limits_do_not_wrap():
    # n_vec * sg_q8k_bytes(cols) would wrap a 64-bit product for n_vec near
    # 2^64 / qb; both scratch entry points compare by division, so such a
    # request is rejected before anything is launched
    lib = _lib.load()
    fake = C.c_void_p(0x100000)
    m = _lib.SgMat(12, 0, 0, 1024, 16)
    qb = lib.sg_q8k_bytes(1024)
    big = (1 << 64) // qb + 1          # big * qb wraps to a small number
    assert (big * qb) % (1 << 64) < 262144
    assert lib.sg_matvec_scratch_bytes(1024, big) == (1 << 64) - 1  # saturates
    huge_ld = 1 << 40
    assert lib.sg_matvec_static(fake, C.byref(m), fake, huge_ld, fake, huge_ld, big, 0, 16, None) == 9
    assert lib.sg_matvec_scratch(fake, C.byref(m), fake, huge_ld, fake, huge_ld, big, 0, 16, fake, 1 << 20,
                                 None) == 1
