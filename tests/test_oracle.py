"""Pins the CPU oracle to the reference's own known-answer tests.

The reference ships no golden vectors; its kernel tests compare the SIMD code
with a scalar f64 reference on seeded random inputs.  These are ports of those
tests, with the same generators, seeds and draw order, run against the oracle:
  quantize_round_trip_and_sums        quant_q8k.rs:343-362
  int_kernel_matches_reference        quant_q8k.rs:368-411
  int_kernel_batch_is_bitwise         quant_q8k.rs:416-442
  simd_kernels_match_scalar_reference quant.rs:1728-1771
  multi_matvec_matches_scalar_ref.    quant_multi.rs:372-417
"""
import numpy as np
import pytest

import oracle as O


def f64_dot(w, x):
    p = w.astype(np.float64) * x.astype(np.float64)
    return p.sum(), np.abs(p).sum()


def test_quantize_round_trip_and_sums():
    rng = O.Rng(11)
    x = rng.fill(-3.0, 3.0, 768)
    q = O.quantize(x)
    back = q.dequant()
    for b in range(3):
        chunk = x[b * 256:(b + 1) * 256]
        amax = np.abs(chunk).max()
        assert np.all(np.abs(back[b * 256:(b + 1) * 256] - chunk) <= amax / 127.0 * 0.5 + 1e-6)
    s = q.qs.astype(np.int32).reshape(-1, 16).sum(1)
    assert np.array_equal(q.bsums.astype(np.int32), s)
    z = O.quantize(np.zeros(256, np.float32))
    assert not z.qs.any() and z.d[0] == 0.0


def test_quantize_nonfinite_and_edge_blocks():
    # !(amax > 0) or non-finite amax -> an all-zero block (quant_q8k.rs:100-105).
    x = np.ones(1024, np.float32)
    x[3] = np.inf
    x[300] = -np.inf
    x[512:768] = -0.0
    q = O.quantize(x)
    assert q.d[0] == 0 and q.d[1] == 0 and q.d[2] == 0
    assert q.d[3] == np.float32(1.0) / np.float32(127.0)
    assert not q.qs[:768].any() and np.all(q.qs[768:] == 127)


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_int_kernel_matches_reference(dtype):
    # The reference walks Q4_K then Q6_K from one generator; replay the Q4_K
    # draws first so the Q6_K case sees the same inputs it does.
    rng = O.Rng(0x51ED)
    for dt in [O.Q4_K, O.Q6_K]:
        for n in [256, 768, 2048]:
            rows = 37
            mat = O.random_matrix(dt, n, rows, rng)
            m = O.Mat(dt, n, rows)
            rb = O.row_bytes(dt, n)
            wrows = [O.dequant_row(dt, mat[r * rb:(r + 1) * rb], n) for r in range(rows)]
            for bsz in range(1, 12):
                xs = [rng.fill(-2.0, 2.0, n) for _ in range(bsz)]
                if dt != dtype:
                    continue
                qs = [O.quantize(x) for x in xs]
                outs = np.full((bsz, rows), np.nan, np.float32)
                ol = [outs[b] for b in range(bsz)]
                O.matmul_rows(mat, m, qs, ol, 0, 3)
                O.matmul_rows(mat, m, qs, ol, 3, rows)
                for b in range(bsz):
                    xq = qs[b].dequant()
                    for r in range(rows):
                        want, scale = f64_dot(wrows[r], xq)
                        got = float(outs[b, r])
                        assert abs(got - want) <= 1e-4 * scale + 1e-6, (dt, n, bsz, b, r, got, want)
                        exact, _ = f64_dot(wrows[r], xs[b])
                        assert abs(got - exact) <= 0.02 * scale + 1e-4


def test_int_kernel_batch_is_bitwise():
    rng = O.Rng(77)
    for dt in [O.Q4_K, O.Q6_K]:
        n, rows = 768, 37
        mat = O.random_matrix(dt, n, rows, rng)
        m = O.Mat(dt, n, rows)
        qs = [O.quantize(rng.fill(-2.0, 2.0, n)) for _ in range(11)]
        batch = O.gemv_int(mat, m, qs)
        for b, q in enumerate(qs):
            one = O.gemv_int(mat, m, [q])[0]
            assert np.array_equal(one.view(np.uint32), batch[b].view(np.uint32))


def test_block_sums_reassemble_kernel():
    # The exported int32 lane sums are the ones the kernel converts: the f64
    # dot of dequantized weights with the dequantized vector equals
    # sum_i d_i*xd_i*sum_l lanes - correction, to rounding.
    rng = O.Rng(5)
    for dt in [O.Q4_K, O.Q6_K]:
        n, rows = 512, 5
        mat = O.random_matrix(dt, n, rows, rng)
        m = O.Mat(dt, n, rows)
        q = O.quantize(rng.fill(-1.0, 1.0, n))
        bs = O.block_sums(mat, m, q, 0, rows)
        assert bs.shape == (rows, 2, 8)
        rb = O.row_bytes(dt, n)
        for r in range(rows):
            blk = mat[r * rb:(r + 1) * rb]
            w = O.dequant_row(dt, blk, n)
            want, scale = f64_dot(w, q.dequant())
            tot = 0.0
            for i in range(2):
                b = blk[i * (rb // 2):(i + 1) * (rb // 2)]
                if dt == O.Q4_K:
                    d = np.frombuffer(b[0:2].tobytes(), np.float16)[0].astype(np.float64)
                    dmin = np.frombuffer(b[2:4].tobytes(), np.float16)[0].astype(np.float64)
                    sc, mn = np.zeros(8, np.int64), np.zeros(8, np.int64)
                    p = b[4:16].astype(np.int64)
                    for j in range(4):
                        sc[j], mn[j] = p[j] & 63, p[j + 4] & 63
                        sc[j + 4] = (p[j + 8] & 15) | ((p[j] >> 6) << 4)
                        mn[j + 4] = (p[j + 8] >> 4) | ((p[j + 4] >> 6) << 4)
                    pairs = q.bsums[i * 16:(i + 1) * 16].astype(np.int64).reshape(8, 2).sum(1)
                    corr = dmin * q.d[i] * float((mn * pairs).sum())
                else:
                    d = np.frombuffer(b[208:210].tobytes(), np.float16)[0].astype(np.float64)
                    sc = b[192:208].view(np.int8).astype(np.int64)
                    corr = d * q.d[i] * float(32 * (sc * q.bsums[i * 16:(i + 1) * 16]).sum())
                tot += d * q.d[i] * float(bs[r, i].sum()) - corr
            # dequant_row rounds every weight to f32, hence a few ulp of slack.
            assert abs(tot - want) <= 1e-6 * scale + 1e-9


FLOAT_TYPES = [O.F32, O.F16, O.BF16, O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K]
ORACLE_FLOAT = {O.F32, O.F16, O.BF16, O.Q8_0, O.Q4_K, O.Q6_K}


def test_simd_kernels_match_scalar_reference():
    # Formats outside the path (Q4_0/Q4_1/Q5_x) still consume their draws.
    rng = O.Rng(0x2545F4914F6CDD1D)
    for dt in FLOAT_TYPES:
        for n in [256, 768, 2048]:
            for rows in [2, 3, 4, 5, 6, 8, 10]:
                mat = np.concatenate([O.random_row(dt, n, rng) for _ in range(rows)])
                x = rng.fill(-1.0, 1.0, n)
                if dt not in ORACLE_FLOAT:
                    continue
                m = O.Mat(dt, n, rows)
                out = O.matvec_rows(mat, m, x, 1, rows - 1)
                rb = O.row_bytes(dt, n)
                for i, got in enumerate(out):
                    r = i + 1
                    w = O.dequant_row(dt, mat[r * rb:(r + 1) * rb], n)
                    want, scale = f64_dot(w, x)
                    assert abs(float(got) - want) <= 1e-4 * scale + 1e-6, (dt, n, r)


def test_multi_matvec_matches_scalar_reference():
    rng = O.Rng(0x9E3779B97F4A7C15)
    for dt in [O.Q4_K, O.Q6_K, O.Q8_0, O.F32, O.Q5_K]:
        for n in [256, 768, 2048]:
            rows = 7
            if dt == O.Q5_K:
                rb = O.row_bytes(dt, n)
                for _ in range(rb * rows):
                    rng.next()
                for _ in range(rb * rows // 176):
                    rng.f(0.001, 0.05)
                    rng.f(0.001, 0.05)
                for bsz in range(1, 12):
                    for _ in range(bsz):
                        rng.fill(-1.0, 1.0, n)
                continue
            mat = O.random_matrix(dt, n, rows, rng)
            m = O.Mat(dt, n, rows)
            rb = O.row_bytes(dt, n)
            wrows = [O.dequant_row(dt, mat[r * rb:(r + 1) * rb], n) for r in range(rows)]
            for bsz in range(1, 12):
                xs = [rng.fill(-1.0, 1.0, n) for _ in range(bsz)]
                a = O.matmul_rows_multi(mat, m, xs, 0, 3)
                b = O.matmul_rows_multi(mat, m, xs, 3, rows)
                outs = np.where(np.isnan(a), b, a)
                for bi in range(bsz):
                    for r in range(rows):
                        want, scale = f64_dot(wrows[r], xs[bi])
                        assert abs(float(outs[bi, r]) - want) <= 1e-4 * scale + 1e-6, (dt, n, bsz, bi, r)


def test_pool_split_matches_single_thread():
    rng = O.Rng(3)
    for dt in [O.Q4_K, O.Q6_K]:
        n, rows = 1024, 301
        mat = O.random_matrix(dt, n, rows, rng)
        m = O.Mat(dt, n, rows)
        xs = np.stack([rng.fill(-1.0, 1.0, n) for _ in range(3)])
        want = O.gemv_int(mat, m, [O.quantize(x) for x in xs])
        O.pool_create(4)
        try:
            got = np.empty((3, rows), np.float32)
            O.pool_matvec_multi(mat, m, xs, got)
        finally:
            O.pool_destroy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_weight_quantizer_round_trip():
    g = np.random.default_rng(0)
    w = g.normal(0, 0.02, (8, 1024)).astype(np.float32)
    for dt, tol in [(O.Q4_K, 0.6), (O.Q6_K, 0.6)]:
        b = O.quantize_weights(dt, w)
        rb = O.row_bytes(dt, 1024)
        dq = np.stack([O.dequant_row(dt, b[r * rb:(r + 1) * rb], 1024) for r in range(8)])
        # Error at most about half a quantization step of each block.
        step = (np.abs(w).max() / (7.5 if dt == O.Q4_K else 31.0))
        assert np.abs(dq - w).max() <= tol * step
