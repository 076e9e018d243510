"""GPU parity of the integer K-quant path against the CPU oracle.

Bar: bit-exact.  Q8_K quantization (d, qs, bsums), the int32 lane sums of
every super-block, and the fp32 GEMV outputs must equal the oracle's (the
reference's AVX2 arithmetic) bit for bit, for every vector count and row split.
"""
import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits(t):
    a = t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a).view(np.uint32)


def q8k_equal(gq, oq):
    assert np.array_equal(bits(gq.d), bits(oq.d))
    assert np.array_equal(gq.qs.cpu().numpy(), oq.qs)
    assert np.array_equal(gq.bsums.cpu().numpy(), oq.bsums)


def test_quantize_matches_oracle(dev):
    rng = O.Rng(11)
    for n in [256, 768, 1024, 4096, 14336]:
        x = rng.fill(-3.0, 3.0, n)
        q = sg.quantize(to_dev(x, dev))
        q8k_equal(q, O.quantize(x))


def test_quantize_edge_blocks(dev):
    g = np.random.default_rng(1)
    x = g.normal(0, 1, 256 * 10).astype(np.float32)
    x[0:256] = 0.0                    # all zero -> d = 0
    x[256 + 5] = np.inf               # non-finite amax -> zero block
    x[512 + 7] = np.nan               # NaN not last in its lane: lost by MAXPS, quantizes to -128
    x[768 + 8 * 31 + 2] = np.nan      # NaN last in its lane: amax NaN -> zero block
    x[1024:1280] = 1e-42              # subnormal amax: 127/amax overflows -> all -128
    x[1280:1536] *= 1e30              # huge
    x[1536:1792] = -0.0
    x[1792 + 100] = -np.inf
    q = sg.quantize(to_dev(x, dev))
    q8k_equal(q, O.quantize(x))


def test_quantize_batch_strided(dev):
    g = np.random.default_rng(2)
    xs = g.normal(0, 1, (5, 1100)).astype(np.float32)
    t = to_dev(xs, dev)[:, :1024]
    outs = [sg.Q8K(1024, dev) for _ in range(5)]
    sg.quantize_into(t, outs)
    for b in range(5):
        q8k_equal(outs[b], O.quantize(xs[b, :1024]))


def _case(dt, n, rows, seed, nvec):
    rng = O.Rng(seed)
    w = O.random_matrix(dt, n, rows, rng)
    xs = [rng.fill(-2.0, 2.0, n) for _ in range(nvec)]
    return w, xs


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n", [256, 768, 1024, 2048, 4096, 14336])
def test_gemv_bitexact_shapes(dev, dt, n):
    rows = 37 if n >= 4096 else 301
    w, xs = _case(dt, n, rows, 0x51ED + n, 3)
    oq = [O.quantize(x) for x in xs]
    want = O.gemv_int(w, O.Mat(dt, n, rows), oq)
    m = sg.Mat(dt, n, rows)
    gq = [sg.quantize(to_dev(x, dev)) for x in xs]
    got = sg.gemv(to_dev(w, dev), m, gq)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_gemv_every_batch_size_and_split(dev, dt):
    # quant_q8k.rs:368-411 shapes: 37 rows, batch 1..16, split [0,3) + [3,37).
    n, rows = 768, 37
    w, xs = _case(dt, n, rows, 77, 16)
    oq = [O.quantize(x) for x in xs]
    wd = to_dev(w, dev)
    gq = [sg.quantize(to_dev(x, dev)) for x in xs]
    m = sg.Mat(dt, n, rows)
    for bsz in range(1, 17):
        want = O.gemv_int(w, O.Mat(dt, n, rows), oq[:bsz])
        out = torch.full((bsz, rows), float("nan"), device=dev)
        sg.matmul_rows(wd, m, gq[:bsz], [out[b] for b in range(bsz)], 0, 3)
        sg.matmul_rows(wd, m, gq[:bsz], [out[b] for b in range(bsz)], 3, rows)
        assert np.array_equal(bits(out), bits(want)), bsz


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_gemv_odd_row_ranges(dev, dt):
    # Row ranges that start and end at unaligned byte offsets, and the last
    # rows of a tensor whose size is not a multiple of 16 bytes.
    n, rows = 768, 203
    w, xs = _case(dt, n, rows, 5, 2)
    oq = [O.quantize(x) for x in xs]
    want = O.gemv_int(w, O.Mat(dt, n, rows), oq)
    wd = to_dev(w, dev)
    gq = [sg.quantize(to_dev(x, dev)) for x in xs]
    m = sg.Mat(dt, n, rows)
    for r0, r1 in [(0, 1), (1, 2), (5, 9), (7, 203), (202, 203), (100, 100), (0, 203)]:
        out = torch.full((2, rows), float("nan"), device=dev)
        sg.matmul_rows(wd, m, gq, [out[0], out[1]], r0, r1)
        o = out.cpu().numpy()
        assert np.array_equal(bits(o[:, r0:r1]), bits(want[:, r0:r1]))
        assert np.isnan(o[:, :r0]).all() and np.isnan(o[:, r1:]).all()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_block_sums_bitexact(dev, dt):
    for n, rows in [(256, 5), (768, 37), (4096, 9), (14336, 3)]:
        w, xs = _case(dt, n, rows, 9 + n, 1)
        oq = O.quantize(xs[0])
        want = O.block_sums(w, O.Mat(dt, n, rows), oq, 0, rows)
        gq = sg.quantize(to_dev(xs[0], dev))
        got = sg.block_sums(to_dev(w, dev), sg.Mat(dt, n, rows), gq, 0, rows)
        assert np.array_equal(got.cpu().numpy(), want)
        got2 = sg.block_sums(to_dev(w, dev), sg.Mat(dt, n, rows), gq, 1, rows)
        assert np.array_equal(got2.cpu().numpy(), want[1:])


def test_int_kernel_matches_reference_on_gpu(dev):
    # The reference's own comparator (quant_q8k.rs:368-411) on the GPU output.
    rng = O.Rng(0x51ED)
    for dt in [O.Q4_K, O.Q6_K]:
        for n in [256, 768, 2048]:
            rows = 37
            w = O.random_matrix(dt, n, rows, rng)
            rb = O.row_bytes(dt, n)
            wrows = [O.dequant_row(dt, w[r * rb:(r + 1) * rb], n).astype(np.float64) for r in range(rows)]
            wd = to_dev(w, dev)
            m = sg.Mat(dt, n, rows)
            for bsz in range(1, 12):
                xs = [rng.fill(-2.0, 2.0, n) for _ in range(bsz)]
                gq = [sg.quantize(to_dev(x, dev)) for x in xs]
                got = sg.gemv(wd, m, gq).cpu().numpy().astype(np.float64)
                for b in range(bsz):
                    xq = O.quantize(xs[b]).dequant().astype(np.float64)
                    for r in range(rows):
                        want = (wrows[r] * xq).sum()
                        scale = np.abs(wrows[r] * xq).sum()
                        assert abs(got[b, r] - want) <= 1e-4 * scale + 1e-6


def test_batch_is_bitwise_on_gpu(dev):
    # quant_q8k.rs:416-442: a vector alone == the same vector inside a batch.
    for dt in [O.Q4_K, O.Q6_K]:
        w, xs = _case(dt, 768, 37, 77, 11)
        wd = to_dev(w, dev)
        m = sg.Mat(dt, 768, 37)
        gq = [sg.quantize(to_dev(x, dev)) for x in xs]
        batch = sg.gemv(wd, m, gq)
        for b in range(11):
            one = sg.gemv(wd, m, [gq[b]])
            assert torch.equal(one[0].view(torch.int32), batch[b].view(torch.int32))


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_weight_quantizer_matches_cpu_twin(dev, dt):
    g = np.random.default_rng(3)
    w = g.normal(0, 0.02, (64, 2048)).astype(np.float32)
    w[3, :256] = 0.0
    w[5, 256:512] = np.abs(w[5, 256:512])
    got = sg.quantize_weights(dt, to_dev(w, dev)).cpu().numpy()
    want = O.quantize_weights(dt, w)
    bb = 144 if dt == O.Q4_K else 210
    bad = np.nonzero((got != want).reshape(-1, bb).any(1))[0]
    if bad.size:
        b = bad[0]
        diff = np.nonzero(got[b * bb:(b + 1) * bb] != want[b * bb:(b + 1) * bb])[0]
        raise AssertionError("%d of %d blocks differ; block %d bytes %s: gpu %s cpu %s" % (
            bad.size, got.size // bb, b, diff[:12].tolist(), got[b * bb + diff[:12]].tolist(),
            want[b * bb + diff[:12]].tolist()))


@pytest.mark.parametrize("dt,rows,cols", [(O.Q4_K, 3072, 1024), (O.Q4_K, 4096, 4096), (O.Q6_K, 4096, 4096),
                                          (O.Q4_K, 14336, 4096), (O.Q6_K, 14336, 4096),
                                          (O.Q4_K, 4096, 14336), (O.Q6_K, 4096, 14336),
                                          (O.Q6_K, 151936, 1024)])
def test_baseline_shapes_bitexact(dev, dt, rows, cols):
    # The benchmark configurations at full size, N(0, 0.02) weights through the
    # weight quantizer, N = 1 and N = 16, checked row for row.
    gen = torch.Generator(device=dev).manual_seed(rows + cols)
    wf = torch.randn(rows, cols, device=dev, generator=gen) * 0.02
    wq = sg.quantize_weights(dt, wf)
    del wf
    xs = torch.randn(16, cols, device=dev, generator=gen)
    m = sg.Mat(dt, cols, rows)
    w_host = wq.cpu().numpy()
    xs_host = xs.cpu().numpy()
    for nvec in (1, 16):
        gq = sg.quantize(xs[:nvec])
        got = sg.gemv(wq, m, gq).cpu().numpy()
        want = O.gemv_int(w_host, O.Mat(dt, cols, rows), [O.quantize(x) for x in xs_host[:nvec]])
        assert np.array_equal(bits(got), bits(want)), nvec


def test_bad_arguments_raise(dev):
    w = torch.zeros(144 * 4, dtype=torch.uint8, device=dev)
    q = sg.Q8K(1024, dev)
    out = torch.zeros(1, device=dev)
    with pytest.raises(sg.SgError):
        sg.matmul_rows(w, sg.Mat(sg.Q4_K, 1000, 1), [q], [out], 0, 1)  # cols % 256
    with pytest.raises(sg.SgError):
        sg.matmul_rows(w, sg.Mat(sg.F16, 1024, 1), [q], [out], 0, 1)  # not an integer format
    with pytest.raises(sg.SgError):
        sg.matmul_rows(w[1:], sg.Mat(sg.Q4_K, 1024, 1), [q], [out], 0, 1)  # misaligned tensor
    with pytest.raises(sg.SgError):
        sg.matmul_rows(w, sg.Mat(sg.Q4_K, 1024, 1), [q], [out], 0, 2)  # r1 > rows
    sg.device_status()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_matvec_scratch_both_layouts(dev, dt):
    # Quantize into caller scratch + integer GEMV, GGUF rows and TILED16.
    for n, rows, nvec in [(768, 37, 1), (4096, 45, 5), (14336, 20, 2)]:
        rng = O.Rng(3 * n + rows)
        w = O.random_matrix(dt, n, rows, rng)
        xs = np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])
        want = O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x) for x in xs])
        wd = to_dev(w, dev)
        xd = to_dev(xs, dev)
        got = sg.matvec_scratch(wd, sg.Mat(dt, n, rows), xd)
        assert np.array_equal(bits(got), bits(want))
        t, m = sg.repack_tiled16(dt, wd, rows, n)
        assert np.array_equal(bits(sg.matvec_scratch(t, m, xd)), bits(want))
        small = torch.empty(16, dtype=torch.uint8, device=dev)
        with pytest.raises(sg.SgError):
            sg.matvec_scratch(wd, sg.Mat(dt, n, rows), xd, scratch=small)
