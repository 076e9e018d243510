"""GPU parity of the tensor-core batch GEMMs (gemm_tc.cu, SG_GEMM_TC=2 for
Q4_K and Q6_K:
tcgen05.mma over f16 operands that hold the exact integers sc * q and y, fp32
accumulators in TMEM): bit-identical to the oracle's Q8K::quantize +
matmul_rows (quant_q8k.rs:84-121, :166-295) and to the dp4a GEMV, with
non-finite inputs, ragged row counts, row ranges and token counts that leave
a 16-token group part empty."""
import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc(monkeypatch):
    monkeypatch.setenv("SG_GEMM_TC", "2")


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits(a):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_tc_gemm_matches_oracle(dev, tc, dt):
    for n, rows, nvec in [(256, 37, 9), (1024, 301, 16), (2048, 45, 17), (512, 130, 33), (2048, 64, 64),
                          (4096, 19, 40), (256, 16, 1), (768, 90, 5), (1536, 257, 63), (1024, 140, 65),
                          (512, 40, 128), (768, 130, 97)]:
        rng = O.Rng(7 * n + rows + nvec)
        w = O.random_matrix(dt, n, rows, rng)
        xs = np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])
        xs[0, 5] = np.nan
        if n >= 512:
            xs[-1, 256:512] = 0.0
            xs[-1, 300] = np.inf if nvec > 1 else 0.0
        want = O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x) for x in xs])
        t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
        xd = torch.zeros(nvec, n + 64, device=dev)
        xd[:, :n] = to_dev(xs, dev)
        got = sg.matmul_batch(t, m, xd[:, :n])
        assert np.array_equal(bits(got), bits(want)), (n, rows, nvec)
        out = torch.full((nvec, rows + 7), float("nan"), device=dev)
        sg.matmul_batch(t, m, xd[:, :n], out[:, :rows], 3, rows - 2)
        o = out.cpu().numpy()
        assert np.array_equal(bits(o[:, 3:rows - 2]), bits(want[:, 3:rows - 2])), (n, rows, nvec)
        assert np.isnan(o[:, :3]).all() and np.isnan(o[:, rows - 2:]).all()
    sg.device_status()


def test_tc_gemm_extreme_blocks(dev, tc):
    # Q4_K: every scale and min at 63, every nibble at 15 (lane sums near
    # their bound 32 * 945 * 127) against inputs of one sign
    n, rows, nvec = 1024, 48, 24
    rng = O.Rng(99)
    w = O.random_matrix(O.Q4_K, n, rows, rng).reshape(rows, n // 256, 144)
    w[:, :, 4:16] = 0xFF
    w[:, :, 16:] = 0xFF
    w = w.reshape(-1)
    xs = np.stack([np.full(n, 1.0 + v, np.float32) * (1 if v % 2 else -1) for v in range(nvec)])
    xs[3] = rng.fill(-2.0, 2.0, n)
    want = O.gemv_int(w, O.Mat(O.Q4_K, n, rows), [O.quantize(x) for x in xs])
    t, m = sg.repack_tiled16(O.Q4_K, to_dev(w, dev), rows, n)
    got = sg.matmul_batch(t, m, to_dev(xs, dev))
    assert np.array_equal(bits(got), bits(want))
    sg.device_status()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_tc_gemm_matches_gemv_at_model_shapes(dev, tc, dt):
    g = torch.Generator(device=dev).manual_seed(11)
    for rows, cols, nvec in [(4608, 2048, 64), (512, 2048, 9), (2048, 4096, 64), (151936, 1024, 9), (3072, 1024, 24),
                             (4608, 2048, 128), (2048, 4096, 128)]:
        wq = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=g) * 0.02)
        t, m = sg.repack_tiled16(dt, wq, rows, cols)
        xs = torch.randn(nvec, cols, device=dev, generator=g)
        want = sg.matvec(t, m, xs)
        got = sg.matmul_batch(t, m, xs)
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (rows, cols, nvec)
    sg.device_status()


def test_tc_gemm_extreme_blocks_q6k(dev, tc):
    # Q6_K: scales at -128 and 127, every 6-bit value at 63 or 0 (lane sums
    # beyond 2^24, split into two exact halves) against inputs of one sign
    n, rows, nvec = 1024, 48, 24
    rng = O.Rng(98)
    w = O.random_matrix(O.Q6_K, n, rows, rng).reshape(rows, n // 256, 210)
    w[:, :, 0:192] = 0xFF
    w[1::2, :, 0:192] = 0x00
    w[:, :, 192:208] = np.array([0x80, 0x7F] * 8, np.uint8)
    w = w.reshape(-1)
    xs = np.stack([np.full(n, 1.0 + v, np.float32) * (1 if v % 2 else -1) for v in range(nvec)])
    xs[3] = rng.fill(-2.0, 2.0, n)
    want = O.gemv_int(w, O.Mat(O.Q6_K, n, rows), [O.quantize(x) for x in xs])
    t, m = sg.repack_tiled16(O.Q6_K, to_dev(w, dev), rows, n)
    got = sg.matmul_batch(t, m, to_dev(xs, dev))
    assert np.array_equal(bits(got), bits(want))
    sg.device_status()
