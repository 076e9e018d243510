"""The CUDA float path (sg_matvec_rows_float / sg_matmul_rows_float) against
the oracle's restatement of matvec_rows_avx2 (quant.rs:939-1094) and
matmul_rows_avx2 / rows_multi (quant_multi.rs:126-273): bit for bit.

Inputs are the reference tests' own generators (random_row, quant.rs:1693-1723;
random_matrix, quant_q8k.rs:323-336 and quant_multi.rs:301-322), weights from
the library's quantizer, the frozen golden fixtures, and edge cases (scalar
tails, odd row ranges, NaN / Inf activations, batches across the 8-vector
groups)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu
G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
FLOAT = [O.F32, O.F16, O.Q8_0, O.Q4_K, O.Q6_K]


def dev_t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits_equal(got, want):
    """Bit-identical, except that any NaN matches any NaN (payloads differ
    between x86 and the GPU)."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    gn, wn = np.isnan(got), np.isnan(want)
    return np.array_equal(gn, wn) and np.array_equal(got[~gn].view(np.uint32), want[~wn].view(np.uint32))


def oracle_rows(w, m, xs, r0, r1):
    out = np.full((len(xs), m.rows), np.nan, np.float32)
    for b, x in enumerate(xs):
        out[b, r0:r1] = O.matvec_rows(w, m, x, r0, r1 - r0)
    return out


def run(dev, dt, w, xs, rows, r0=0, r1=None, multi=False):
    n = xs.shape[1]
    r1 = rows if r1 is None else r1
    m = sg.Mat(dt, n, rows)
    f = sg.matmul_rows_float if multi else sg.matvec_rows_float
    return f(dev_t(w, dev), m, dev_t(xs, dev), r0=r0, r1=r1).cpu().numpy()


def test_float_golden_fixtures(dev):
    for name, dt in [("f32", sg.F32), ("f16", sg.F16), ("q8_0", sg.Q8_0), ("fq4k", sg.Q4_K), ("fq6k", sg.Q6_K)]:
        w, xv, want = G[name + "_w"], G[name + "_x"], G[name + "_out"]
        assert bits_equal(run(dev, dt, w, xv[None], want.size)[0], want), name
    for name, dt in [("mf32", sg.F32), ("mq8_0", sg.Q8_0), ("mq4k", sg.Q4_K), ("mq6k", sg.Q6_K)]:
        w, xs, want = G[name + "_w"], G[name + "_x"], G[name + "_out"]
        assert bits_equal(run(dev, dt, w, xs, want.shape[1], multi=True), want), name


@pytest.mark.parametrize("dt", FLOAT)
def test_matvec_rows_float_reference_generators(dev, dt):
    rng = O.Rng(0x2545F4914F6CDD1D + dt)
    for n in [256, 768, 2048]:
        for rows in [1, 5, 33, 70]:
            w = np.concatenate([O.random_row(dt, n, rng) for _ in range(rows)])
            xs = np.stack([rng.fill(-1.0, 1.0, n) for _ in range(3)])
            m = O.Mat(dt, n, rows)
            r0, r1 = (1, rows - 1) if rows > 2 else (0, rows)
            got = run(dev, dt, w, xs, rows, r0, r1)
            assert bits_equal(got, oracle_rows(w, m, xs, r0, r1)), (dt, n, rows)


@pytest.mark.parametrize("dt", [O.F32, O.Q8_0, O.Q4_K, O.Q6_K])
def test_matmul_rows_float_multi(dev, dt):
    rng = O.Rng(0x9E3779B97F4A7C15 + dt)
    for n in [256, 768, 2048]:
        rows = 37
        w = O.random_matrix(dt, n, rows, rng)
        m = O.Mat(dt, n, rows)
        for bsz in [1, 2, 3, 5, 8, 9, 11, 16, 17]:
            xs = np.stack([rng.fill(-1.0, 1.0, n) for _ in range(bsz)])
            got = run(dev, dt, w, xs, rows, 3, rows, multi=True)
            want = O.matmul_rows_multi(w, m, list(xs), 3, rows)
            assert bits_equal(got, want), (dt, n, bsz)


def test_float_scalar_tails(dev):
    # F32 / F16 rows of any width: the 8-lane chains plus the scalar tail
    rng = np.random.default_rng(3)
    for dt in [O.F32, O.F16]:
        for n in [1, 7, 8, 13, 100, 1000, 4099]:
            rows = 19
            wf = rng.standard_normal((rows, n)).astype(np.float32)
            w = (wf if dt == O.F32 else wf.astype(np.float16)).view(np.uint8).reshape(-1)
            xs = rng.standard_normal((2, n)).astype(np.float32)
            m = O.Mat(dt, n, rows)
            assert bits_equal(run(dev, dt, w, xs, rows), oracle_rows(w, m, xs, 0, rows)), (dt, n)
            if dt == O.F32 and n % 8 == 0:
                got = run(dev, dt, w, xs, rows, multi=True)
                assert bits_equal(got, O.matmul_rows_multi(w, m, list(xs), 0, rows)), n


def test_float_quantizer_weights_and_shapes(dev):
    # the library's own K-quant weights at BASELINE-like shapes
    g = torch.Generator(device=dev).manual_seed(7)
    for dt, rows, cols in [(sg.Q4_K, 3072, 1024), (sg.Q6_K, 2048, 768), (sg.Q4_K, 512, 14336)]:
        wf = torch.randn(rows, cols, device=dev, generator=g) * 0.02
        w = sg.quantize_weights(dt, wf)
        xs = torch.randn(2, cols, device=dev, generator=g)
        m = sg.Mat(dt, cols, rows)
        got = sg.matvec_rows_float(w, m, xs).cpu().numpy()
        wn, xn = w.cpu().numpy(), xs.cpu().numpy()
        assert bits_equal(got, oracle_rows(wn, O.Mat(dt, cols, rows), xn, 0, rows)), (dt, rows, cols)
        got = sg.matmul_rows_float(w, m, xs).cpu().numpy()
        assert bits_equal(got, O.matmul_rows_multi(wn, O.Mat(dt, cols, rows), list(xn), 0, rows))


def test_float_router_shape(dev):
    # the MoE router of Qwen3-30B-A3B: F32 128 x 2048
    g = np.random.default_rng(11)
    w = (g.standard_normal((128, 2048)) / 2048 ** 0.5).astype(np.float32)
    xs = g.standard_normal((1, 2048)).astype(np.float32)
    wb = w.view(np.uint8).reshape(-1)
    got = run(dev, O.F32, wb, xs, 128)
    assert bits_equal(got, oracle_rows(wb, O.Mat(O.F32, 2048, 128), xs, 0, 128))


def test_float_nonfinite(dev):
    rng = O.Rng(99)
    for dt in FLOAT:
        n, rows = 512, 9
        w = np.concatenate([O.random_row(dt, n, rng) for _ in range(rows)])
        xs = np.stack([rng.fill(-1.0, 1.0, n) for _ in range(2)])
        xs[0, 17] = np.inf
        xs[1, 300] = np.nan
        m = O.Mat(dt, n, rows)
        assert bits_equal(run(dev, dt, w, xs, rows), oracle_rows(w, m, xs, 0, rows)), dt
        if dt != O.F16:
            got = run(dev, dt, w, xs, rows, multi=True)
            assert bits_equal(got, O.matmul_rows_multi(w, m, list(xs), 0, rows)), dt


def test_float_bad_args(dev):
    w = torch.zeros(4096, dtype=torch.uint8, device=dev)
    x = torch.zeros(256, device=dev)
    with pytest.raises(sg.SgError) as e:
        sg.matvec_rows_float(w, sg.Mat(2, 256, 4), x)  # Q4_0 is not on the path
    assert e.value.status == 2
    with pytest.raises(sg.SgError) as e:
        sg.matvec_rows_float(w, sg.Mat(sg.Q8_0, 100, 4), x[:100])  # cols % 32
    assert e.value.status == 3
    with pytest.raises(sg.SgError) as e:
        sg.matvec_rows_float(w, sg.Mat(sg.Q4_K, 256, 4, layout=sg.TILED16), x)
    assert e.value.status == 1
    with pytest.raises(sg.SgError) as e:
        sg.matvec_rows_float(w, sg.Mat(sg.Q4_K, 256, 4, offset=8), x)  # 16-byte alignment
    assert e.value.status == 4
    out = torch.full((1, 4), 7.0, device=dev)
    sg.matvec_rows_float(w, sg.Mat(sg.F32, 256, 4), x, out=out, r0=2, r1=2)  # empty range
    assert bool((out == 7.0).all())
