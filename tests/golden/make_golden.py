"""Writes tests/golden/golden.npz: frozen outputs of the CPU oracle on the
reference tests' own generators (quant_q8k.rs:302-336), used as regression
fixtures by tests/test_golden.py (CPU) and tests/test_golden_gpu.py (CUDA).

The reference ships no golden vectors; these pin today's oracle bits so that a
change to the oracle or to the CUDA path that moves a single bit is caught.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def make():
    out = {}
    rng = O.Rng(11)
    x = rng.fill(-3.0, 3.0, 768)
    x[5] = np.float32(np.nan)        # lost inside its MAXPS lane -> quantizes to -128
    x[256:512] = 0.0                 # all-zero block
    q = O.quantize(x)
    out["q8k_x"], out["q8k_d"], out["q8k_qs"], out["q8k_bsums"] = x, q.d, q.qs, q.bsums
    for name, dt in [("q4k", O.Q4_K), ("q6k", O.Q6_K)]:
        rng = O.Rng(0x51ED)
        n, rows, nvec = 768, 37, 3
        w = O.random_matrix(dt, n, rows, rng)
        xs = np.stack([rng.fill(-2.0, 2.0, n) for _ in range(nvec)])
        qs = [O.quantize(v) for v in xs]
        out[name + "_w"], out[name + "_x"] = w, xs
        out[name + "_out"] = O.gemv_int(w, O.Mat(dt, n, rows), qs)
        out[name + "_sums"] = O.block_sums(w, O.Mat(dt, n, rows), qs[0], 0, rows)
    for name, dt in [("f32", O.F32), ("f16", O.F16), ("q8_0", O.Q8_0), ("fq4k", O.Q4_K), ("fq6k", O.Q6_K)]:
        rng = O.Rng(0x2545F4914F6CDD1D)
        n, rows = 512, 6
        w = np.concatenate([O.random_row(dt, n, rng) for _ in range(rows)])
        xv = rng.fill(-1.0, 1.0, n)
        out[name + "_w"], out[name + "_x"] = w, xv
        out[name + "_out"] = O.matvec_rows(w, O.Mat(dt, n, rows), xv, 0, rows)
    for name, dt in [("mf32", O.F32), ("mq8_0", O.Q8_0), ("mq4k", O.Q4_K), ("mq6k", O.Q6_K)]:
        rng = O.Rng(0x9E3779B97F4A7C15)
        n, rows, nvec = 512, 7, 5
        w = O.random_matrix(dt, n, rows, rng)
        xs = np.stack([rng.fill(-1.0, 1.0, n) for _ in range(nvec)])
        out[name + "_w"], out[name + "_x"] = w, xs
        out[name + "_out"] = O.matmul_rows_multi(w, O.Mat(dt, n, rows), list(xs), 0, rows)
    g = np.random.default_rng(5)
    wf = (g.standard_normal((16, 512)) * 0.02).astype(np.float32)
    out["wq_f32"] = wf
    out["wq_q4k"] = O.quantize_weights(O.Q4_K, wf)
    out["wq_q6k"] = O.quantize_weights(O.Q6_K, wf)
    return out


if __name__ == "__main__":
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **make())
    print("wrote", os.path.join(HERE, "golden.npz"))
