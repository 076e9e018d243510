"""The MoE / fused-FFN oracle against the reference's own MoE test."""
import numpy as np

import oracle as O


def test_moe_forward_matches_reference():
    # smollm_chat.rs:4891-4975: an all-F32 MoE layer (dim 32, ff 24, 6 experts,
    # top 2, shared expert of 16) checked against a loop-by-loop restatement.
    dim, ff, n_exp, k, sh_ff = 32, 24, 6, 2, 16
    buf = []
    seed = [12345]

    def push(n):
        off = len(buf) * 4
        for _ in range(n):
            s = seed[0]
            s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
            s ^= s >> 7
            s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
            seed[0] = s
            buf.append(np.float32(np.float32(s >> 40) / np.float32(1 << 24)) - np.float32(0.5))
        return off

    mat = lambda off, cols, rows: O.Mat(O.F32, cols, rows, off)
    router = mat(push(dim * n_exp), dim, n_exp)
    gate = mat(push(dim * ff * n_exp), dim, ff)
    up = mat(push(dim * ff * n_exp), dim, ff)
    down = mat(push(ff * dim * n_exp), ff, dim)
    shg, shu, shd = mat(push(dim * sh_ff), dim, sh_ff), mat(push(dim * sh_ff), dim, sh_ff), mat(push(sh_ff * dim), sh_ff, dim)
    sh_gate = push(dim)
    W = np.array(buf, np.float32)
    raw = W.view(np.uint8)
    x = np.array([np.sin(np.float32(i) * np.float32(0.37)) for i in range(dim)], np.float32)

    def w(m, e, r, c):
        return W[m.offset // 4 + (e * m.rows + r) * m.cols + c]

    def dot(vals):
        s = np.float32(0.0)
        for v in vals:
            s = np.float32(s + v)
        return s

    for norm, shared in [(True, False), (False, True)]:
        moe = O.Moe(router=router, gate=gate, up=up, down=down, n_expert=n_exp, n_used=k, norm=int(norm),
                    moe_prune=0.0, has_shared=int(shared), has_shared_gate=int(shared), sh_gate=shg, sh_up=shu,
                    sh_down=shd, shared_gate_offset=sh_gate)
        got, chosen, _ = O.moe_forward(raw, moe, x)
        logits = [dot(w(router, 0, e, c) * x[c] for c in range(dim)) for e in range(n_exp)]
        mx = max(logits)
        ex = [np.float32(np.exp(np.float32(l - mx))) for l in logits]
        s = dot(ex)
        probs = [np.float32(e / s) for e in ex]
        order = sorted(range(n_exp), key=lambda e: -probs[e])
        top = order[:k]
        assert list(chosen) == top
        tsum = dot(probs[e] for e in top)

        def ffn_ref(g_, u_, d_, e):
            n = g_.rows
            h = []
            for r in range(n):
                g = dot(w(g_, e, r, c) * x[c] for c in range(dim))
                u = dot(w(u_, e, r, c) * x[c] for c in range(dim))
                h.append(np.float32(np.float32(g / np.float32(1.0 + np.float32(np.exp(-g)))) * u))
            return [dot(w(d_, e, r, c) * h[c] for c in range(n)) for r in range(dim)]

        want = np.zeros(dim, np.float32)
        for e in top:
            wt = probs[e] / tsum if norm else probs[e]
            want += np.float32(wt) * np.array(ffn_ref(gate, up, down, e), np.float32)
        if shared:
            z = dot(W[sh_gate // 4 + c] * x[c] for c in range(dim))
            g = np.float32(1.0) / np.float32(1.0 + np.exp(-z))
            want += g * np.array(ffn_ref(shg, shu, shd, 0), np.float32)
        assert np.all(np.abs(got - want) < 1e-4), (norm, shared)


def test_moe_quantized_route_and_prune():
    # A Q4_K/Q6_K MoE (the Qwen3-30B-A3B layout, scaled down): ffns_fused on the
    # chosen experts equals moe_forward, and pruning keeps the documented count.
    rng = O.Rng(4242)
    dim, ff, n_exp, k = 512, 256, 16, 8
    router = rng.fill(-0.05, 0.05, n_exp * dim)
    g = O.random_matrix(O.Q4_K, dim, ff * n_exp, rng)
    u = O.random_matrix(O.Q4_K, dim, ff * n_exp, rng)
    d = O.random_matrix(O.Q6_K, ff, dim * n_exp, rng)
    raw = np.concatenate([router.view(np.uint8), g, u, d])
    off_g = router.nbytes
    off_u = off_g + g.nbytes
    off_d = off_u + u.nbytes
    moe = O.Moe(router=O.Mat(O.F32, dim, n_exp, 0), gate=O.Mat(O.Q4_K, dim, ff, off_g),
                up=O.Mat(O.Q4_K, dim, ff, off_u), down=O.Mat(O.Q6_K, ff, dim, off_d), n_expert=n_exp, n_used=k,
                norm=1, moe_prune=0.0)
    x = rng.fill(-1.0, 1.0, dim)
    out, chosen, ws = O.moe_forward(raw, moe, x)
    assert len(chosen) == k and abs(float(ws.sum()) - 1.0) < 1e-5
    rb = lambda dt, cols: O.row_bytes(dt, cols)
    gs = [O.Mat(O.Q4_K, dim, ff, off_g + int(e) * ff * rb(O.Q4_K, dim)) for e in chosen]
    us = [O.Mat(O.Q4_K, dim, ff, off_u + int(e) * ff * rb(O.Q4_K, dim)) for e in chosen]
    ds = [O.Mat(O.Q6_K, ff, dim, off_d + int(e) * dim * rb(O.Q6_K, ff)) for e in chosen]
    again = O.ffns_fused(raw, gs, us, ds, ws, x, np.zeros(dim, np.float32))
    assert np.array_equal(again.view(np.uint32), out.view(np.uint32))
    for prune, keep in [(4.0, 4), (1.0, 4), (9.0, 8)]:
        moe.moe_prune = prune
        _, c2, w2 = O.moe_route(raw, moe, x)
        assert len(c2) == keep and list(c2) == list(chosen[:keep])
        assert abs(float(w2.sum()) - 1.0) < 1e-5
    moe.moe_prune = 0.5
    probs, c3, _ = O.moe_route(raw, moe, x)
    assert 4 <= len(c3) <= k
