"""Small random decoder models for the forward-pass tests: the same weights as
one host byte buffer with offsets for the oracle (GGUF-like) and as CUDA
tensors for spindle_b200.decoder."""
import numpy as np

import oracle as O

Q4_K, Q6_K, F32, F16 = O.Q4_K, O.Q6_K, O.F32, O.F16


def dtypes_for(cfg, attn_v=Q6_K, down=Q6_K, head=Q6_K, embed=Q6_K, other=Q4_K):
    d = {"embed": embed, "head": head}
    for i in range(cfg["n_layers"]):
        p = "l%d." % i
        d.update({p + "wq": other, p + "wk": other, p + "wv": attn_v, p + "wo": other})
        if cfg.get("moe"):
            d.update({p + "gate_exps": other, p + "up_exps": other, p + "down_exps": down})
        else:
            d.update({p + "gate": other, p + "up": other, p + "down": down})
    return d


def host_weights(cfg, dtypes, seed=0, wscale=0.05):
    """name -> numpy array: uint8 GGUF rows for matrices (the library's
    quantizer, as on the GPU), float32 vectors; norms 1 + 0.1 N(0,1)."""
    g = np.random.default_rng(seed)
    c = cfg
    dim, hd = c["dim"], c["head_dim"]
    q_dim, kv_dim = c["n_heads"] * hd, c["n_kv_heads"] * hd

    def mat(name, rows, cols):
        w = g.standard_normal((rows, cols), dtype=np.float32) * np.float32(wscale)
        dt = dtypes[name]
        if dt == F32:
            return w.reshape(-1).view(np.uint8).copy()
        if dt == F16:
            return w.astype(np.float16).reshape(-1).view(np.uint8).copy()
        return O.quantize_weights(dt, w)

    def norm(n):
        return (np.float32(1.0) + np.float32(0.1) * g.standard_normal(n, dtype=np.float32)).astype(np.float32)

    W = {"embed": mat("embed", c["vocab"], dim), "head": mat("head", c["vocab"], dim), "out_norm": norm(dim)}
    for i in range(c["n_layers"]):
        p = "l%d." % i
        W[p + "attn_norm"], W[p + "ffn_norm"] = norm(dim), norm(dim)
        if c.get("qk_norm", True):
            W[p + "q_norm"], W[p + "k_norm"] = norm(hd), norm(hd)
        W[p + "wq"] = mat(p + "wq", q_dim, dim)
        W[p + "wk"] = mat(p + "wk", kv_dim, dim)
        W[p + "wv"] = mat(p + "wv", kv_dim, dim)
        W[p + "wo"] = mat(p + "wo", dim, q_dim)
        moe = c.get("moe")
        if moe:
            ne, f = moe["n_expert"], moe["n_ff"]
            W[p + "router"] = (g.standard_normal((ne, dim), dtype=np.float32) / np.float32(np.sqrt(dim))).astype(np.float32)
            W[p + "gate_exps"] = mat(p + "gate_exps", ne * f, dim)
            W[p + "up_exps"] = mat(p + "up_exps", ne * f, dim)
            W[p + "down_exps"] = mat(p + "down_exps", ne * dim, f)
        else:
            f = c["n_ff"]
            W[p + "gate"] = mat(p + "gate", f, dim)
            W[p + "up"] = mat(p + "up", f, dim)
            W[p + "down"] = mat(p + "down", dim, f)
    return W


def oracle_decoder(cfg, dtypes, W):
    """The oracle's Decoder over one byte buffer holding W (32-byte aligned).
    W's values may be numpy arrays or torch tensors (CUDA ones are copied
    straight into their slice of the buffer, so a model of many GB is held on
    the host once)."""
    off, pos = {}, 0
    for name, arr in W.items():
        pos += (-pos) % 32
        off[name] = pos
        pos += arr.nbytes if isinstance(arr, np.ndarray) else arr.numel() * arr.element_size()
    buf = np.zeros(pos, np.uint8)
    for name, arr in W.items():
        if isinstance(arr, np.ndarray):
            b = np.ascontiguousarray(arr).reshape(-1).view(np.uint8)
            buf[off[name]:off[name] + b.nbytes] = b
        else:
            import torch
            b = arr.contiguous().reshape(-1).view(torch.uint8)
            torch.from_numpy(buf[off[name]:off[name] + b.numel()]).copy_(b)
    c = cfg
    dim, hd = c["dim"], c["head_dim"]
    q_dim, kv_dim = c["n_heads"] * hd, c["n_kv_heads"] * hd
    mat = lambda name, cols, rows: O.Mat(dtypes[name], cols, rows, off[name])
    layers = []
    for i in range(c["n_layers"]):
        p = "l%d." % i
        y = O.Layer()
        y.attn_norm, y.ffn_norm = off[p + "attn_norm"], off[p + "ffn_norm"]
        y.q_norm = off.get(p + "q_norm", O.NO_NORM)
        y.k_norm = off.get(p + "k_norm", O.NO_NORM)
        y.wq, y.wk = mat(p + "wq", dim, q_dim), mat(p + "wk", dim, kv_dim)
        y.wv, y.wo = mat(p + "wv", dim, kv_dim), mat(p + "wo", q_dim, dim)
        moe = c.get("moe")
        if moe:
            ne, f = moe["n_expert"], moe["n_ff"]
            y.is_moe = 1
            y.moe = O.Moe(router=O.Mat(O.F32, dim, ne, off[p + "router"]), gate=mat(p + "gate_exps", dim, f),
                          up=mat(p + "up_exps", dim, f), down=mat(p + "down_exps", f, dim), n_expert=ne,
                          n_used=moe["n_used"], norm=int(moe.get("norm", True)), moe_prune=moe.get("prune", 0.0))
        else:
            f = c["n_ff"]
            y.is_moe = 0
            y.gate, y.up, y.down = mat(p + "gate", dim, f), mat(p + "up", dim, f), mat(p + "down", f, dim)
        layers.append(y)
    m = O.Model(dim=dim, n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"], head_dim=hd, n_layers=c["n_layers"],
                vocab=c["vocab"], max_seq=c["max_seq"], rope_neox=int(c.get("rope_neox", True)),
                rope_theta=c["rope_theta"], rms_eps=c["rms_eps"], residual_scale=c.get("residual_scale", 1.0),
                embedding_scale=c.get("embedding_scale", 1.0), attn_scale=c.get("attn_scale", 0.0),
                embed=mat("embed", dim, c["vocab"]), lm_head=mat("head", dim, c["vocab"]),
                output_norm=off["out_norm"])
    return O.Decoder(buf, m, layers)


def device_weights(W, dev):
    import torch
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in W.items()}


DENSE = dict(dim=512, n_heads=8, n_kv_heads=4, head_dim=64, n_layers=2, vocab=1000, max_seq=64, rope_theta=1e6,
             rms_eps=1e-6, n_ff=768, rope_neox=True)
MOE = dict(dim=512, n_heads=8, n_kv_heads=2, head_dim=128, n_layers=2, vocab=1200, max_seq=64, rope_theta=1e6,
           rms_eps=1e-6, rope_neox=True, moe=dict(n_expert=16, n_used=4, n_ff=256, norm=True))
