"""The kernels' expf / sinf / cosf against the host's glibc.

The reference calls f32::exp and f32::sin_cos, which Rust's std takes from
glibc on Linux (expf, sinf, cosf).  spindle_b200/csrc/glibc_math.h restates
glibc's algorithms for the device.  The CPU test compiles that header as host
C and compares it with glibc on every one of the 2^32 float inputs; the GPU
test runs the device build (sg_libm_eval) over a stride of all inputs and
compares with glibc input by input.  NaN results agree when both are NaN.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FNS = {0: "expf", 1: "sinf", 2: "cosf"}
NT = min(os.cpu_count() or 1, 64)


@pytest.fixture(scope="module")
def check_lib(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("libm") / "libm_check.so")
    subprocess.run(["gcc", "-O2", "-mfma", "-ffp-contract=off", "-shared", "-fPIC", "-o", out,
                    os.path.join(ROOT, "tests", "libm_check.c"), "-lm", "-lpthread"], check=True)
    L = C.CDLL(out)
    L.lm_count_mismatch.restype = C.c_uint64
    L.lm_count_mismatch.argtypes = [C.c_int, C.c_uint64, C.c_uint64, C.c_int, C.POINTER(C.c_uint32)]
    L.lm_compare_strided.restype = C.c_uint64
    L.lm_compare_strided.argtypes = [C.c_int, C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p, C.c_int,
                                     C.POINTER(C.c_uint32)]
    L.lm_host.restype = C.c_float
    L.lm_host.argtypes = [C.c_int, C.c_float]
    L.lm_mine.restype = C.c_float
    L.lm_mine.argtypes = [C.c_int, C.c_float]
    return L


def test_known_values(check_lib):
    L = check_lib
    for fn, x, want in [(0, 0.0, 1.0), (0, 1.0, np.float32(np.e)), (0, -np.inf, 0.0), (0, np.inf, np.inf),
                        (0, 89.0, np.inf), (0, -104.0, 0.0), (1, 0.0, 0.0), (2, 0.0, 1.0)]:
        assert L.lm_mine(fn, x) == want, (FNS[fn], x)
    assert np.isnan(L.lm_mine(0, np.nan)) and np.isnan(L.lm_mine(1, np.inf)) and np.isnan(L.lm_mine(2, -np.inf))
    # the two reduction branches of sinf / cosf (|x| < 120, and larger) and the RoPE range
    for x in [0.5, 1.0, 3.0, -7.5, 100.0, 119.9, 120.0, 4095.0 * 0.9, 1e6, -3e9, 3.4e38]:
        for fn in (1, 2):
            assert L.lm_mine(fn, x) == L.lm_host(fn, x), (FNS[fn], x)


@pytest.mark.parametrize("fn", [0, 1, 2])
def test_every_float_input_matches_glibc(check_lib, fn):
    # all 2^32 bit patterns, split over the host's cores (a few seconds each)
    first = C.c_uint32()
    bad = check_lib.lm_count_mismatch(fn, 0, 1 << 32, NT, C.byref(first))
    assert bad == 0, "%s: %d inputs differ, first 0x%08x" % (FNS[fn], bad, first.value)


@pytest.mark.gpu
@pytest.mark.parametrize("fn", [0, 1, 2])
def test_device_build_matches_glibc(check_lib, fn, dev):
    import torch

    from spindle_b200 import _lib

    lib = _lib.load()
    stride = 61                                  # prime: every exponent and mantissa pattern is visited
    for start in (0, 17):
        count = ((1 << 32) - start + stride - 1) // stride
        out = torch.empty(count, dtype=torch.float32, device=dev)
        _lib.check(lib.sg_libm_eval(fn, start, stride, count, C.c_void_p(out.data_ptr()), None), "sg_libm_eval")
        host = out.cpu().numpy()
        first = C.c_uint32()
        bad = check_lib.lm_compare_strided(fn, start, stride, count, host.ctypes.data, NT, C.byref(first))
        assert bad == 0, "%s: %d of %d inputs differ, first 0x%08x" % (FNS[fn], bad, count, first.value)
    # every float of the ranges the kernels feed: softmax/SiLU arguments in [-128, 128], RoPE angles to 2^17
    lo, hi = np.array([-128.0, 128.0], np.float32).view(np.uint32)
    for a, b in ([0, int(hi)], [0x80000000, int(lo)]) if fn == 0 else ([0, 0x48000000],):
        count = b - a + 1
        for s in range(a, a + count, 1 << 28):
            n = min(1 << 28, a + count - s)
            out = torch.empty(n, dtype=torch.float32, device=dev)
            _lib.check(lib.sg_libm_eval(fn, s, 1, n, C.c_void_p(out.data_ptr()), None), "sg_libm_eval")
            host = out.cpu().numpy()
            first = C.c_uint32()
            bad = check_lib.lm_compare_strided(fn, s, 1, n, host.ctypes.data, NT, C.byref(first))
            assert bad == 0, "%s: %d differ in [0x%08x, +%d), first 0x%08x" % (FNS[fn], bad, s, n, first.value)
