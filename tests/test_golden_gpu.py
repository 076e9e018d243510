"""The CUDA path reproduces the frozen golden fixtures (tests/golden) bit for bit."""
import os

import numpy as np
import pytest
import torch

import spindle_b200 as sg

pytestmark = pytest.mark.gpu
G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def dev_t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def same(a, b):
    a = a.cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(b).view(np.uint8))


def test_q8k_fixture_gpu(dev):
    q = sg.quantize(dev_t(G["q8k_x"], dev))
    assert same(q.d, G["q8k_d"]) and same(q.qs, G["q8k_qs"]) and same(q.bsums, G["q8k_bsums"])


def test_int_gemv_fixtures_gpu(dev):
    for name, dt in [("q4k", sg.Q4_K), ("q6k", sg.Q6_K)]:
        w, xs, want = dev_t(G[name + "_w"], dev), G[name + "_x"], G[name + "_out"]
        m = sg.Mat(dt, xs.shape[1], want.shape[1])
        q = sg.quantize(dev_t(xs, dev))
        assert same(sg.gemv(w, m, q), want)
        assert same(sg.block_sums(w, m, q[0], 0, m.rows), G[name + "_sums"])
        t, mt = sg.repack_tiled16(dt, w, m.rows, m.cols)
        assert same(sg.matvec(t, mt, dev_t(xs, dev)), want)


def test_weight_quantizer_fixtures_gpu(dev):
    wf = dev_t(G["wq_f32"], dev)
    assert same(sg.quantize_weights(sg.Q4_K, wf), G["wq_q4k"])
    assert same(sg.quantize_weights(sg.Q6_K, wf), G["wq_q6k"])
