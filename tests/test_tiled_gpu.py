"""GPU parity of the TILED16 weight layout: the repack is a byte permutation
(round trip exact) and the tiled GEMV is bit-identical to the oracle."""
import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits(a):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.ascontiguousarray(a).view(np.uint32)


def _case(dt, n, rows, seed, nvec):
    rng = O.Rng(seed)
    w = O.random_matrix(dt, n, rows, rng)
    xs = [rng.fill(-2.0, 2.0, n) for _ in range(nvec)]
    return w, xs


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_repack_round_trip(dev, dt):
    for n, rows in [(256, 1), (768, 37), (4096, 16), (1024, 33)]:
        w, _ = _case(dt, n, rows, 3 + rows, 0)
        t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
        assert t.numel() == (rows + 15) // 16 * 16 * O.row_bytes(dt, n)
        back = sg.unpack_tiled16(dt, t, rows, n).cpu().numpy()
        assert np.array_equal(back, w)
        # padding rows of the last tile are zero
        if rows % 16:
            tb = t.cpu().numpy().reshape(-1, 16 * (144 if dt == O.Q4_K else 210))
            assert tb.shape[0] == (rows + 15) // 16 * (n // 256)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n", [256, 768, 1024, 2048, 4096, 14336])
def test_tiled_gemv_bitexact(dev, dt, n):
    rows = 45 if n >= 4096 else 301
    w, xs = _case(dt, n, rows, 0x7E57 + n, 3)
    oq = [O.quantize(x) for x in xs]
    want = O.gemv_int(w, O.Mat(dt, n, rows), oq)
    t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
    gq = [sg.quantize(to_dev(x, dev)) for x in xs]
    for k in (1, 2, 3):
        got = sg.gemv(t, m, gq[:k])
        assert np.array_equal(bits(got), bits(want[:k])), k


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_tiled_every_batch_size_and_split(dev, dt):
    n, rows = 768, 37
    w, xs = _case(dt, n, rows, 77, 16)
    oq = [O.quantize(x) for x in xs]
    t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
    gq = [sg.quantize(to_dev(x, dev)) for x in xs]
    for bsz in range(1, 17):
        want = O.gemv_int(w, O.Mat(dt, n, rows), oq[:bsz])
        out = torch.full((bsz, rows), float("nan"), device=dev)
        for r0, r1 in [(0, 3), (3, 17), (17, 37)]:
            sg.matmul_rows(t, m, gq[:bsz], [out[b] for b in range(bsz)], r0, r1)
        assert np.array_equal(bits(out), bits(want)), bsz


@pytest.mark.parametrize("dt,rows,cols", [(O.Q4_K, 3072, 1024), (O.Q4_K, 14336, 4096), (O.Q6_K, 4096, 14336),
                                          (O.Q6_K, 151936, 1024)])
def test_tiled_baseline_shapes(dev, dt, rows, cols):
    gen = torch.Generator(device=dev).manual_seed(rows * 3 + cols)
    wq = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=gen) * 0.02)
    t, m = sg.repack_tiled16(dt, wq, rows, cols)
    xs = torch.randn(8, cols, device=dev, generator=gen)
    w_host, xs_host = wq.cpu().numpy(), xs.cpu().numpy()
    for nvec in (1, 8):
        got = sg.gemv(t, m, sg.quantize(xs[:nvec])).cpu().numpy()
        want = O.gemv_int(w_host, O.Mat(dt, cols, rows), [O.quantize(x) for x in xs_host[:nvec]])
        assert np.array_equal(bits(got), bits(want)), nvec
    sg.device_status()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_matvec_fused_quantize_bitexact(dev, dt):
    # sg_matvec quantizes inside the GEMV kernel; the bits must equal the
    # oracle's Q8K::quantize + matmul_rows, including non-finite inputs.
    for n, rows, nvec in [(256, 37, 1), (1024, 301, 3), (4096, 45, 8), (14336, 19, 2), (2048, 64, 11)]:
        rng = O.Rng(n + rows)
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
        got = sg.matvec(t, m, xd[:, :n])
        assert np.array_equal(bits(got), bits(want)), (n, rows, nvec)
        # a row range
        out = torch.full((nvec, rows), float("nan"), device=dev)
        sg.matvec(t, m, xd[:, :n], out, 3, rows - 2)
        o = out.cpu().numpy()
        assert np.array_equal(bits(o[:, 3:rows - 2]), bits(want[:, 3:rows - 2]))
        assert np.isnan(o[:, :3]).all() and np.isnan(o[:, rows - 2:]).all()


def test_matvec_rejects_gguf_layout(dev):
    w = torch.zeros(144 * 4, dtype=torch.uint8, device=dev)
    with pytest.raises(sg.SgError):
        sg.matvec(w, sg.Mat(sg.Q4_K, 1024, 1), torch.zeros(1024, device=dev))
