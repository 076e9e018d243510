"""GPU parity of the dp4a batch GEMM (sg_matmul_batch: matvec_multi over 9..128
vectors, one pass per group of 64, smollm_chat.rs:447-512): bit-identical to the oracle's
Q8K::quantize + matmul_rows (quant_q8k.rs:84-121, :255-295) and to the GEMV,
including non-finite inputs, ragged row counts, row ranges and every token
group size."""
import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def dp4a_path(monkeypatch):
    # Q4_K batches run on the tensor cores by default (test_gemm_tc_gpu.py);
    # this file checks the dp4a kernel
    monkeypatch.setenv("SG_GEMM_TC", "0")


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits(a):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_batch_gemm_matches_oracle(dev, dt):
    for n, rows, nvec in [(256, 37, 9), (1024, 301, 16), (2048, 45, 17), (512, 130, 33), (2048, 64, 64),
                          (4096, 19, 40), (256, 16, 1), (768, 90, 5), (1024, 77, 65), (512, 40, 128), (768, 33, 100)]:
        rng = O.Rng(7 * n + rows + nvec)
        w = O.random_matrix(dt, n, rows, rng)
        xs = np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])
        xs[0, 5] = np.nan
        if n >= 512:
            xs[-1, 256:512] = 0.0
            xs[-1, 300] = np.inf if nvec > 1 else 0.0
        want = O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x) for x in xs])
        t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
        xd = torch.zeros(nvec, n + 64, device=dev)   # padded rows: ldx > cols
        xd[:, :n] = to_dev(xs, dev)
        got = sg.matmul_batch(t, m, xd[:, :n])
        assert np.array_equal(bits(got), bits(want)), (n, rows, nvec)
        out = torch.full((nvec, rows + 7), float("nan"), device=dev)
        sg.matmul_batch(t, m, xd[:, :n], out[:, :rows], 3, rows - 2)
        o = out.cpu().numpy()
        assert np.array_equal(bits(o[:, 3:rows - 2]), bits(want[:, 3:rows - 2])), (n, rows, nvec)
        assert np.isnan(o[:, :3]).all() and np.isnan(o[:, rows - 2:]).all()
    sg.device_status()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_batch_gemm_matches_gemv_at_model_shapes(dev, dt):
    # the decoder's projections and LM head at prefill / verify widths
    g = torch.Generator(device=dev).manual_seed(11)
    for rows, cols, nvec in [(4608, 2048, 64), (512, 2048, 9), (2048, 4096, 64), (151936, 1024, 9), (3072, 1024, 24),
                             (512, 2048, 128), (2048, 4096, 128)]:
        wq = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=g) * 0.02)
        t, m = sg.repack_tiled16(dt, wq, rows, cols)
        xs = torch.randn(nvec, cols, device=dev, generator=g)
        want = sg.matvec(t, m, xs)
        got = sg.matmul_batch(t, m, xs)
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (rows, cols, nvec)
    sg.device_status()


def test_batch_gemm_rejects(dev):
    w = torch.zeros(144 * 4, dtype=torch.uint8, device=dev)
    with pytest.raises(sg.SgError):   # GGUF layout
        sg.matmul_batch(w, sg.Mat(sg.Q4_K, 1024, 1), torch.zeros(9, 1024, device=dev))
    t, m = sg.repack_tiled16(O.Q4_K, torch.zeros(144 * 4 * 16, dtype=torch.uint8, device=dev), 16, 1024)
    with pytest.raises(sg.SgError):   # more than 128 vectors
        sg.matmul_batch(t, m, torch.zeros(129, 1024, device=dev))
