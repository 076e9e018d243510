"""The oracle still reproduces the frozen golden fixtures (tests/golden)."""
import os

import numpy as np

import oracle as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


def test_q8k_fixture():
    q = O.quantize(G["q8k_x"])
    assert same(q.d, G["q8k_d"]) and same(q.qs, G["q8k_qs"]) and same(q.bsums, G["q8k_bsums"])


def test_int_gemv_fixtures():
    for name, dt in [("q4k", O.Q4_K), ("q6k", O.Q6_K)]:
        w, xs = G[name + "_w"], G[name + "_x"]
        qs = [O.quantize(v) for v in xs]
        m = O.Mat(dt, xs.shape[1], G[name + "_out"].shape[1])
        assert same(O.gemv_int(w, m, qs), G[name + "_out"])
        assert same(O.block_sums(w, m, qs[0], 0, m.rows), G[name + "_sums"])


def test_float_matvec_fixtures():
    for name, dt in [("f32", O.F32), ("f16", O.F16), ("q8_0", O.Q8_0), ("fq4k", O.Q4_K), ("fq6k", O.Q6_K)]:
        w, xv, want = G[name + "_w"], G[name + "_x"], G[name + "_out"]
        assert same(O.matvec_rows(w, O.Mat(dt, xv.size, want.size), xv, 0, want.size), want)


def test_float_multi_fixtures():
    for name, dt in [("mf32", O.F32), ("mq8_0", O.Q8_0), ("mq4k", O.Q4_K), ("mq6k", O.Q6_K)]:
        w, xs, want = G[name + "_w"], G[name + "_x"], G[name + "_out"]
        m = O.Mat(dt, xs.shape[1], want.shape[1])
        assert same(O.matmul_rows_multi(w, m, list(xs), 0, m.rows), want)


def test_weight_quantizer_fixtures():
    assert same(O.quantize_weights(O.Q4_K, G["wq_f32"]), G["wq_q4k"])
    assert same(O.quantize_weights(O.Q6_K, G["wq_f32"]), G["wq_q6k"])
