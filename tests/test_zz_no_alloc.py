"""sg_matvec_static: the matvec entry point for callers that cannot allocate
device memory (their Q8_K scratch lives in a static device array inside the
library).  Checked through the C ABI against sg_matvec_scratch, the entry point
that takes caller-owned scratch, on two calls in a row: the shared array keeps
the first call's contents, and the second call must not see them.

This file is collected last on purpose, so that a run stopping at its first
failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg
from spindle_b200 import _lib

pytestmark = pytest.mark.gpu

LIMIT = 262144  # SG_NOALLOC_SCRATCH_BYTES


def call_static(w, m, xs, out, r0=0, r1=None):
    r1 = m.rows if r1 is None else r1
    return sg.lib().sg_matvec_static(C.c_void_p(w.data_ptr()), C.byref(m.c()), C.c_void_p(xs.data_ptr()),
                                     xs.stride(0), C.c_void_p(out.data_ptr()), out.stride(0), xs.shape[0], r0, r1,
                                     C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_static_scratch_matches_caller_scratch_twice(dev, dt):
    for n, rows, nvec in [(4096, 45, 3), (1024, 301, 1), (14336, 20, 15)]:
        rng = O.Rng(7 * n + rows)
        w = torch.from_numpy(O.random_matrix(dt, n, rows, rng)).to(dev)
        t, mt = sg.repack_tiled16(dt, w, rows, n)
        for base, m in [(w, sg.Mat(dt, n, rows)), (t, mt)]:
            for call in range(2):   # the second call runs over the first call's leftovers
                xs = torch.from_numpy(np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])).to(dev)
                want = sg.matvec_scratch(base, m, xs)
                got = torch.full((nvec, rows), float("nan"), device=dev)
                assert call_static(base, m, xs, got) == 0
                torch.cuda.synchronize()
                assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (n, nvec, call)


def test_static_scratch_limit_and_row_range(dev):
    n = 65536
    per_vec = sg.lib().sg_matvec_scratch_bytes(n, 1)
    too_many = LIMIT // per_vec + 1
    w = torch.zeros(16 * 144 * (n // 256), dtype=torch.uint8, device=dev)
    m = sg.Mat(sg.Q4_K, n, 16)
    xs = torch.zeros(too_many, n, device=dev)
    out = torch.zeros(too_many, 16, device=dev)
    assert call_static(w, m, xs, out) == 9  # SG_ERR_NOALLOC_LIMIT, nothing launched
    # a row range inside the matrix, the remaining rows untouched
    rng = O.Rng(99)
    wr = torch.from_numpy(O.random_matrix(sg.Q6_K, 2048, 40, rng)).to(dev)
    m2 = sg.Mat(sg.Q6_K, 2048, 40)
    x2 = torch.from_numpy(np.stack([rng.fill(-1.0, 1.0, 2048) for _ in range(2)])).to(dev)
    want = sg.matvec_scratch(wr, m2, x2)
    got = torch.full((2, 40), float("nan"), device=dev)
    assert call_static(wr, m2, x2, got, 5, 33) == 0
    torch.cuda.synchronize()
    assert torch.equal(got[:, 5:33].view(torch.int32), want[:, 5:33].view(torch.int32))
    assert torch.isnan(got[:, :5]).all() and torch.isnan(got[:, 33:]).all()
    sg.device_status()


def test_static_scratch_allocates_nothing(dev):
    # the property the entry point exists for: after its first call on the
    # device (which only looks the array up), further calls leave the
    # device's free memory exactly as it was, so nothing was allocated
    rng = O.Rng(123)
    n, rows, nvec = 4096, 300, 4
    w = torch.from_numpy(O.random_matrix(sg.Q4_K, n, rows, rng)).to(dev)
    t, mt = sg.repack_tiled16(sg.Q4_K, w, rows, n)
    xs = torch.from_numpy(np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])).to(dev)
    out = torch.empty(nvec, rows, device=dev)
    assert call_static(t, mt, xs, out) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(50):
        assert call_static(t, mt, xs, out) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    want = sg.matvec_scratch(t, mt, xs)
    assert torch.equal(out.view(torch.int32), want.view(torch.int32))
