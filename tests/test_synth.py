"""The reference's synthetic benchmark kernels (q4k_gemv.rs, route_moe_top2 in
moe_engine.rs, the int8-KV flash decoding of transformer.rs).

The oracle (oracle/synth.c, the AVX2 code restated) is pinned by the
reference's own tests: test_q4k_avx2_matches_scalar_reference
(transformer.rs:310-349: one block against a scalar dequantize-and-dot, four
vectors, within 1e-2) and test_int8_gqa_flash_decoding_finite_and_causal
(:393-404).  The GPU kernels (spindle_b200/csrc/synth.cu) are then checked
against the oracle bit for bit, rows wrapping modulo 4096 and row offsets
included."""
import ctypes as C

import numpy as np
import pytest

import oracle as O

S = O.SYNTH


def ref_block():
    # the block and activations of test_q4k_avx2_matches_scalar_reference
    blk = np.zeros(144, np.uint8)
    blk[0:2] = [0x00, 0x3C]  # d = 1.0
    blk[2:4] = [0x00, 0x38]  # dmin = 0.5
    blk[4:16] = [3, 5, 7, 9, 2, 4, 6, 8, 0x21, 0x43, 0x65, 0x87]
    blk[16:] = [(i * 73 + 19) & 0xFF for i in range(128)]
    i = np.arange(256, dtype=np.float32)
    acts = [((i - 128.0) * 0.01).astype(np.float32), ((i * 0.5 - 64.0) * 0.01).astype(np.float32),
            ((((np.arange(256) * 3) % 256).astype(np.float32) - 128.0) * 0.01).astype(np.float32),
            ((((np.arange(256) * 7) % 256).astype(np.float32) - 128.0) * 0.01).astype(np.float32)]
    return blk, acts


def scalar_ref(blk, act):
    """q4k_block_dot_scalar_ref (transformer.rs:281-306), in float32 steps."""
    f = np.float32
    d = f(O.synth_f16(int(blk[0]) | (int(blk[1]) << 8)))
    dmin = f(O.synth_f16(int(blk[2]) | (int(blk[3]) << 8)))
    sc = blk[4:16].astype(int)
    s = [sc[j] & 63 for j in range(4)] + [(sc[j + 8] & 15) | ((sc[j] >> 6) << 4) for j in range(4)]
    m = [sc[j + 4] & 63 for j in range(4)] + [(sc[j + 8] >> 4) | ((sc[j + 4] >> 6) << 4) for j in range(4)]
    total = f(0)
    for c in range(4):
        for i in range(32):
            b = int(blk[16 + 32 * c + i])
            wl = f(b & 15) * (d * f(s[2 * c])) - dmin * f(m[2 * c])
            wh = f(b >> 4) * (d * f(s[2 * c + 1])) - dmin * f(m[2 * c + 1])
            total = f(total + f(wl * act[64 * c + i]))
            total = f(total + f(wh * act[64 * c + 32 + i]))
    return float(total)


def test_oracle_block_dot_matches_scalar_reference():
    blk, acts = ref_block()
    for a in acts:
        assert abs(O.q4k_block_dot(blk, a) - scalar_ref(blk, a)) < 1e-2
    # the four-vector slice gives each vector the single dot's bits
    chunk = np.tile(np.concatenate([blk] * 16), 4)
    x4 = np.stack([np.tile(a, 16) for a in acts]).astype(np.float32)
    y4 = np.zeros((4, 4096), np.float32)
    O.q4k_gemm_spec4(chunk, 0, 4, x4, y4)
    for k in range(4):
        want = np.float32(0)
        for _ in range(16):
            want = np.float32(want + np.float32(O.q4k_block_dot(blk, acts[k])))
        assert y4[k, 0] == want and y4[k, 3] == want and y4[k, 4] == 0


def test_oracle_synthetic_f16():
    assert O.synth_f16(0x3C00) == 1.0 and O.synth_f16(0xBC00) == -1.0
    assert O.synth_f16(0x7C00) == 2.0 ** -8  # the Inf code maps to a finite scale
    assert O.synth_f16(0x7800) == 16.0  # exponent 15 clamped to 4
    assert O.synth_f16(0x0001) == 2.0 ** -24  # subnormals kept


def test_oracle_route_top2():
    g = np.random.default_rng(3)
    x = g.standard_normal(4096).astype(np.float32)
    gates = g.standard_normal((8, 4096)).astype(np.float32)
    for layer in range(5):
        ex, w = O.route_moe_top2(x, gates, layer)
        s = [np.float32(sum(np.float32(x[i] * gates[e, i]) for i in range(0, 4096, 16))) for e in range(8)]
        s = [float(np.float32(s[e] + np.float32(np.float32((layer + e) % 8) * np.float32(0.05)))) for e in range(8)]
        order = sorted(range(8), key=lambda e: -s[e])
        assert list(ex) == order[:2]
        assert abs(float(w.sum()) - 1.0) < 1e-6 and w[0] >= w[1]


def test_oracle_flash_finite_and_causal():
    # test_int8_gqa_flash_decoding_finite_and_causal: q = 0.25 everywhere, a
    # 64-position cache, layer 0: every output finite
    q = np.full((4, 4096), 0.25, np.float32)
    cache = O.kvcache_init(64)
    O.flash_gqa_spec4(q, cache, 0)
    assert np.isfinite(q).all()
    # causal: token 0 attends to positions 0..64 only, so changing what token 3
    # appends (position 67) leaves tokens 0..2 unchanged
    g = np.random.default_rng(4)
    qa = g.standard_normal((4, 4096)).astype(np.float32)
    qb = qa.copy()
    qb[3] = g.standard_normal(4096).astype(np.float32)
    ca, cb = O.kvcache_init(64), O.kvcache_init(64)
    O.flash_gqa_spec4(qa, ca, 1)
    O.flash_gqa_spec4(qb, cb, 1)
    assert np.array_equal(qa[:3], qb[:3]) and not np.array_equal(qa[3], qb[3])


# ---- GPU against the oracle, bit for bit -------------------------------------

def _lib():
    import spindle_b200 as sg
    return sg.lib()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def rand_blocks(g, n_rows):
    """Rows of 16 random Q4_K blocks with moderate d / dmin (raw random f16
    codes too: the synthetic f16 clamps them)."""
    b = g.integers(0, 256, (n_rows, 16, 144), dtype=np.uint8)
    if n_rows > 2:
        b[: n_rows // 2, :, 1] = g.integers(0x30, 0x3C, (n_rows // 2, 16), dtype=np.uint8)  # d in a sane range
        b[: n_rows // 2, :, 3] = g.integers(0x30, 0x3C, (n_rows // 2, 16), dtype=np.uint8)
    return b.reshape(-1)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,offset", [(4, 0), (4098, 0), (8200, 4093), (12, 77)])
def test_gpu_gemv_4row_matches_oracle(dev, rows, offset):
    import torch
    g = np.random.default_rng(rows + offset)
    chunk = rand_blocks(g, rows)
    x = (g.standard_normal(4096) * 0.1).astype(np.float32)
    y0 = (g.standard_normal(4096) * 0.01).astype(np.float32)
    want = y0.copy()
    done = O.q4k_gemv_4row(chunk, x, want, offset)
    dc, dx, dy = torch.from_numpy(chunk).to(dev), torch.from_numpy(x).to(dev), torch.from_numpy(y0).to(dev)
    got_rows = C.c_uint64()
    assert _lib().sg_q4k_gemv_4row(C.c_void_p(dc.data_ptr()), chunk.size, C.c_void_p(dx.data_ptr()),
                                   C.c_void_p(dy.data_ptr()), offset, C.byref(got_rows), None) == 0
    torch.cuda.synchronize()
    assert got_rows.value == done == rows // 4 * 4
    assert np.array_equal(bits(dy.cpu().numpy()), bits(want))


@pytest.mark.gpu
@pytest.mark.parametrize("r0,r1,base", [(0, 4, 0), (3, 4099, 10), (100, 200, 4000)])
def test_gpu_gemm_spec4_matches_oracle(dev, r0, r1, base):
    import torch
    g = np.random.default_rng(r1 + base)
    chunk = rand_blocks(g, r1)
    x4 = (g.standard_normal((4, 4096)) * 0.1).astype(np.float32)
    y4 = np.zeros((4, 4096), np.float32)
    want = y4.copy()
    O.q4k_gemm_spec4(chunk, r0, r1, x4, want, base)
    dc, dx, dy = (torch.from_numpy(a).to(dev) for a in (chunk, x4, y4))
    assert _lib().sg_q4k_gemm_spec4(C.c_void_p(dc.data_ptr()), r0, r1, C.c_void_p(dx.data_ptr()),
                                    C.c_void_p(dy.data_ptr()), base, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(dy.cpu().numpy()), bits(want))
    blk, acts = ref_block()  # the reference test's block, through the GPU
    chunk = np.tile(np.concatenate([blk] * 16), 4)
    x4 = np.stack([np.tile(a, 16) for a in acts]).astype(np.float32)
    want = np.zeros((4, 4096), np.float32)
    O.q4k_gemm_spec4(chunk, 0, 4, x4, want)
    dc, dx, dy = (torch.from_numpy(a).to(dev) for a in (chunk, x4, np.zeros((4, 4096), np.float32)))
    assert _lib().sg_q4k_gemm_spec4(C.c_void_p(dc.data_ptr()), 0, 4, C.c_void_p(dx.data_ptr()),
                                    C.c_void_p(dy.data_ptr()), 0, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(dy.cpu().numpy()), bits(want))


@pytest.mark.gpu
def test_gpu_route_top2_matches_oracle(dev):
    import torch
    g = np.random.default_rng(5)
    for layer in range(10):
        x = g.standard_normal(4096).astype(np.float32)
        gates = (g.standard_normal((8, 4096)) * 0.3).astype(np.float32)
        ex, w = O.route_moe_top2(x, gates, layer)
        dx, dg = torch.from_numpy(x).to(dev), torch.from_numpy(gates).to(dev)
        de, dw = torch.zeros(2, dtype=torch.int32, device=dev), torch.zeros(2, device=dev)
        assert _lib().sg_route_moe_top2(C.c_void_p(dx.data_ptr()), C.c_void_p(dg.data_ptr()), layer,
                                        C.c_void_p(de.data_ptr()), C.c_void_p(dw.data_ptr()), None) == 0
        torch.cuda.synchronize()
        assert list(de.cpu().numpy()) == list(ex) and np.array_equal(bits(dw.cpu().numpy()), bits(w))


@pytest.mark.gpu
@pytest.mark.parametrize("ctx,layer", [(64, 0), (300, 33), (600, 7)])
def test_gpu_flash_gqa_matches_oracle(dev, ctx, layer):
    import torch
    g = np.random.default_rng(ctx + layer)
    q = g.standard_normal((4, 4096)).astype(np.float32)
    cache = O.kvcache_init(ctx)
    dq = torch.from_numpy(q).to(dev)
    dk, dv, dks, dvs = (torch.from_numpy(a.copy()).to(dev) for a in cache[:4])
    seq = cache[4]
    O.flash_gqa_spec4(q, cache, layer)
    assert _lib().sg_flash_gqa_spec4(C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()), C.c_void_p(dv.data_ptr()),
                                     C.c_void_p(dks.data_ptr()), C.c_void_p(dvs.data_ptr()), seq, layer,
                                     None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dk.cpu().numpy(), cache[0]) and np.array_equal(dv.cpu().numpy(), cache[1])
    assert np.array_equal(bits(dks.cpu().numpy()), bits(cache[2]))
    assert np.array_equal(bits(dq.cpu().numpy()), bits(q))
