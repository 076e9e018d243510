"""The oracle's forward pass (oracle/forward.c) pinned without a GPU.

The reference holds no golden vectors for a whole step (its model tests need
model files), so the restatement is checked against an independent float64
implementation of forward_slice (smollm_chat.rs:3371-3552) on the same
dequantized weights, with the oracle on its float kernels (int_on = False):
only fp32 rounding separates them.  The integer path of the matvecs and the
MoE layer are pinned by test_oracle.py and test_oracle_moe.py.
"""
import math
import sys
import os

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import decoder_util as U  # noqa: E402

import oracle as O  # noqa: E402


def test_rmsnorm_is_the_sequential_sum():
    g = np.random.default_rng(3)
    x = g.standard_normal(1000, dtype=np.float32)
    w = g.standard_normal(1000, dtype=np.float32)
    ss = np.float32(0.0)
    for v in x:
        ss = np.float32(ss + np.float32(v * v))
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(1000) + np.float32(1e-6)))
    want = (x * inv).astype(np.float32) * w
    assert np.array_equal(O.rmsnorm(x, w, 1e-6).view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_argmax_ties_pick_the_last():
    assert O.argmax(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 2
    assert O.argmax(np.array([-0.0, 0.0], np.float32)) == 1
    assert O.argmax(np.array([0.0, -0.0], np.float32)) == 0  # total_cmp: -0 < +0
    assert O.argmax(np.array([1.0, np.nan], np.float32)) == 1  # a positive NaN is above every number


def dq(W, dtypes, name, rows, cols):
    dt = dtypes[name]
    rb = O.row_bytes(dt, cols)
    b = W[name]
    return np.stack([O.dequant_row(dt, b[r * rb:(r + 1) * rb], cols) for r in range(rows)]).astype(np.float64)


def ref_forward(cfg, dtypes, W, tokens):
    """forward_slice in float64 over dequantized weights, one token at a time."""
    c = cfg
    dim, hd, H, KV = c["dim"], c["head_dim"], c["n_heads"], c["n_kv_heads"]
    eps = c["rms_eps"]
    E = dq(W, dtypes, "embed", c["vocab"], dim)
    head = dq(W, dtypes, "head", c["vocab"], dim)
    freqs = np.array([1.0 / c["rope_theta"] ** (2 * i / hd) for i in range(hd // 2)])
    L = []
    for i in range(c["n_layers"]):
        p = "l%d." % i
        y = {k: dq(W, dtypes, p + k, r, cc) for k, r, cc in
             [("wq", H * hd, dim), ("wk", KV * hd, dim), ("wv", KV * hd, dim), ("wo", dim, H * hd)]}
        if c.get("moe"):
            m = c["moe"]
            ne, f = m["n_expert"], m["n_ff"]
            y["router"] = W[p + "router"].astype(np.float64)
            y["g"] = dq(W, dtypes, p + "gate_exps", ne * f, dim).reshape(ne, f, dim)
            y["u"] = dq(W, dtypes, p + "up_exps", ne * f, dim).reshape(ne, f, dim)
            y["d"] = dq(W, dtypes, p + "down_exps", ne * dim, f).reshape(ne, dim, f)
        else:
            f = c["n_ff"]
            y["g"] = dq(W, dtypes, p + "gate", f, dim)[None]
            y["u"] = dq(W, dtypes, p + "up", f, dim)[None]
            y["d"] = dq(W, dtypes, p + "down", dim, f)[None]
        L.append(y)

    def norm(x, w):
        return x / np.sqrt(np.mean(x * x) + eps) * w

    def rope(v, pos):
        v = v.reshape(-1, hd).copy()
        a, b = v[:, :hd // 2].copy(), v[:, hd // 2:].copy()
        ang = pos * freqs
        v[:, :hd // 2] = a * np.cos(ang) - b * np.sin(ang)
        v[:, hd // 2:] = a * np.sin(ang) + b * np.cos(ang)
        return v.reshape(-1)

    def silu(z):
        return z / (1 + np.exp(-z))

    K = [[] for _ in range(c["n_layers"])]
    V = [[] for _ in range(c["n_layers"])]
    outs = []
    for pos, t in enumerate(tokens):
        x = E[t].copy()
        for i, y in enumerate(L):
            p = "l%d." % i
            xn = norm(x, W[p + "attn_norm"].astype(np.float64))
            q, k, v = y["wq"] @ xn, y["wk"] @ xn, y["wv"] @ xn
            if p + "q_norm" in W:
                q = np.concatenate([norm(h, W[p + "q_norm"].astype(np.float64)) for h in q.reshape(-1, hd)])
                k = np.concatenate([norm(h, W[p + "k_norm"].astype(np.float64)) for h in k.reshape(-1, hd)])
            q, k = rope(q, pos), rope(k, pos)
            K[i].append(k.astype(np.float16).astype(np.float64))
            V[i].append(v.astype(np.float16).astype(np.float64))
            att = np.zeros(H * hd)
            for h in range(H):
                kv = h // (H // KV)
                ks = np.stack([kk[kv * hd:(kv + 1) * hd] for kk in K[i]])
                vs = np.stack([vv[kv * hd:(kv + 1) * hd] for vv in V[i]])
                s = ks @ q[h * hd:(h + 1) * hd] / math.sqrt(hd)
                pr = np.exp(s - s.max())
                att[h * hd:(h + 1) * hd] = pr @ vs / pr.sum()
            x = x + y["wo"] @ att
            xn = norm(x, W[p + "ffn_norm"].astype(np.float64))
            if c.get("moe"):
                m = c["moe"]
                lg = y["router"] @ xn
                pr = np.exp(lg - lg.max())
                pr /= pr.sum()
                top = np.argsort(-pr, kind="stable")[:m["n_used"]]
                w = pr[top] / pr[top].sum() if m.get("norm", True) else pr[top]
                ffn = sum(wi * (y["d"][e] @ (silu(y["g"][e] @ xn) * (y["u"][e] @ xn))) for wi, e in zip(w, top))
            else:
                ffn = y["d"][0] @ (silu(y["g"][0] @ xn) * (y["u"][0] @ xn))
            x = x + ffn
        xn = norm(x, W["out_norm"].astype(np.float64))
        outs.append(head @ xn)
    return outs


@pytest.mark.parametrize("cfg", [U.DENSE, U.MOE], ids=["dense", "moe"])
def test_forward_matches_float64(cfg):
    c = dict(cfg, n_layers=2, vocab=200)
    dtypes = U.dtypes_for(c)
    W = U.host_weights(c, dtypes, seed=11)
    D = U.oracle_decoder(c, dtypes, W)
    tokens = [3, 17, 199, 42, 0, 7]
    want = ref_forward(c, dtypes, W, tokens)
    for pos, t in enumerate(tokens):
        _, got = D.forward(t, pos, int_on=False)
        scale = np.abs(want[pos]).max()
        err = np.abs(got - want[pos]).max()
        assert err <= 2e-4 * scale, (pos, err, scale)


def test_forward_int_path_close_to_float_path():
    # the integer matvecs quantize activations to int8: close, not equal
    c = dict(U.DENSE, vocab=300)
    dtypes = U.dtypes_for(c)
    W = U.host_weights(c, dtypes, seed=5)
    a, b = U.oracle_decoder(c, dtypes, W), U.oracle_decoder(c, dtypes, W)
    for pos, t in enumerate([1, 2, 3, 4]):
        _, li = a.forward(t, pos, int_on=True)
        _, lf = b.forward(t, pos, int_on=False)
        assert np.abs(li - lf).max() <= 0.05 * np.abs(lf).max()


def _rope_textbook(v, head_dim, pos, theta, neox):
    # rope_reference (smollm_chat.rs:4853-4865): theta^(-2i/hd) per pair
    out = v.copy()
    half = head_dim // 2
    for h in range(v.size // head_dim):
        for i in range(half):
            ang = np.float32(pos) * np.float32(theta) ** np.float32(-(2.0 * i) / head_dim)
            a, b = (h * head_dim + i, h * head_dim + i + half) if neox else (h * head_dim + 2 * i, h * head_dim + 2 * i + 1)
            c, s = np.float32(math.cos(ang)), np.float32(math.sin(ang))
            out[a] = v[a] * c - v[b] * s
            out[b] = v[a] * s + v[b] * c
    return out


@pytest.mark.parametrize("neox", [False, True])
def test_rope_matches_reference_and_composes(neox):
    # rope_matches_reference_and_composes (smollm_chat.rs:4867-4886)
    hd = 64
    v = np.array([((i * 37 % 101) / 50.0) - 1.0 for i in range(3 * hd)], np.float32)
    f = O.rope_freqs(100000.0, hd)
    a = O.rope_rotate(v, hd, f, neox, 17.0)
    assert np.abs(a - _rope_textbook(v, hd, 17.0, 100000.0, neox)).max() < 1e-4
    # the KV-cache shift: rotate(p) then rotate(-d) == rotate(p - d)
    a = O.rope_rotate(a, hd, f, neox, -5.0)
    b = O.rope_rotate(v, hd, f, neox, 12.0)
    assert np.abs(a - b).max() < 1e-4


def test_oracle_kv_shift():
    # shift_kv (smollm_chat.rs:2942-2972) on the oracle's caches: pinned rows
    # untouched, V rows moved verbatim, K rows re-rotated by -n_discard (equal
    # to within f16 rounding to the keys computed at the new positions, since
    # RoPE rotations compose), n_discard clamped, the new position returned
    cfg = dict(U.DENSE, max_seq=32)
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=35)
    a = U.oracle_decoder(cfg, dtypes, W)
    toks = [3, 9, 27, 81, 243, 5, 15, 45, 135, 405, 7, 21]
    for pos, t in enumerate(toks):
        a.forward(t, pos)
    k0, v0 = a.kcache.copy(), a.vcache.copy()
    n_keep, n_discard, cur = 3, 4, len(toks)
    assert a.kv_shift(n_keep, n_discard, cur) == cur - n_discard
    kv_dim = cfg["n_kv_heads"] * cfg["head_dim"]
    kr = lambda c, l, p: c.reshape(cfg["n_layers"], cfg["max_seq"], kv_dim)[l, p]
    for l in range(cfg["n_layers"]):
        for p in range(n_keep):
            assert np.array_equal(kr(a.kcache, l, p), kr(k0, l, p)) and np.array_equal(kr(a.vcache, l, p), kr(v0, l, p))
        for i in range(cur - n_keep - n_discard):
            assert np.array_equal(kr(a.vcache, l, n_keep + i), kr(v0, l, n_keep + n_discard + i))
    # the re-rotated keys of the last layer against the keys a fresh model
    # writes when the kept tokens sit at the new positions (attention of the
    # first layers is unchanged only for pinned rows, so compare one layer-0 row)
    b = U.oracle_decoder(cfg, dtypes, W)
    kept = toks[:n_keep] + toks[n_keep + n_discard:]
    for pos, t in enumerate(kept[:n_keep + 1]):
        b.forward(t, pos)
    got = kr(a.kcache, 0, n_keep).view(np.float16).astype(np.float32)
    want = kr(b.kcache, 0, n_keep).view(np.float16).astype(np.float32)
    assert np.abs(got - want).max() <= 2e-3 * max(np.abs(want).max(), 1.0)
    assert a.kv_shift(cur, 5, cur) == cur and a.kv_shift(0, 99, 3) == 0
