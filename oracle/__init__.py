"""CPU oracle for spindle's quantized matvec path — TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes front end over oracle/_build/libsg_oracle.so, a C restatement
of the reference Rust kernels (WiseHax/spindle 1.1.0: quant_q8k.rs, quant.rs,
quant_multi.rs, q4k_gemv.rs, worker_pool.rs) with bit-identical fp32 results.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use it,
and only as the checker / the timed reference — never as the product path.

Parity anchoring: the reference ships no golden vectors; the oracle is checked
against all of its own tests' known-answer comparators (tests/test_oracle.py).
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 3, 6, 7, 8, 12, 13, 14, 30
QK = 256

_lib = None


class Mat(C.Structure):
    """`Mat` of quant.rs:914-935: dtype, byte offset, cols, rows."""
    _fields_ = [("dtype", C.c_int32), ("_pad", C.c_uint32), ("offset", C.c_uint64),
                ("cols", C.c_uint64), ("rows", C.c_uint64)]

    def __init__(self, dtype, cols, rows, offset=0):
        super().__init__(dtype, 0, offset, cols, rows)


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        P, S, U64, I32 = C.c_void_p, C.c_size_t, C.c_uint64, C.c_int32
        sig = {
            "or_rng_next": (U64, [C.POINTER(U64)]),
            "or_rng_f": (C.c_float, [C.POINTER(U64), C.c_float, C.c_float]),
            "or_rng_fill_f32": (None, [C.POINTER(U64), C.c_float, C.c_float, P, S]),
            "or_f16_trunc": (C.c_uint16, [C.c_float]),
            "or_f16_trunc_flush": (C.c_uint16, [C.c_float]),
            "or_random_matrix": (C.c_int, [I32, S, S, C.POINTER(U64), P]),
            "or_random_row": (C.c_int, [I32, S, C.POINTER(U64), P]),
            "or_row_bytes": (C.c_int64, [I32, U64]),
            "or_f16_to_f32": (C.c_float, [C.c_uint16]),
            "or_dequant_row": (C.c_int, [I32, P, S, P]),
            "or_q8k_quantize": (None, [P, S, P, P, P]),
            "or_matmul_rows": (C.c_int, [P, C.POINTER(Mat), S, P, P, P, P, S, S]),
            "or_block_sums": (C.c_int, [P, C.POINTER(Mat), P, S, S, P]),
            "or_matvec_rows": (C.c_int, [P, C.POINTER(Mat), P, P, S, S]),
            "or_matmul_rows_multi": (C.c_int, [P, C.POINTER(Mat), S, P, P, S, S]),
            "or_pool_create": (C.c_int, [C.c_int]),
            "or_pool_destroy": (None, []),
            "or_pool_threads": (C.c_int, []),
            "or_pool_matvec_multi": (C.c_int, [P, C.POINTER(Mat), S, P, P]),
            "or_cpu_has_avx2": (C.c_int, []),
            "or_quantize_q4k": (None, [P, S, P]),
            "or_quantize_q6k": (None, [P, S, P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        if not L.or_cpu_has_avx2():
            raise RuntimeError("oracle needs a CPU with AVX2, FMA and F16C")
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


class Rng:
    """The tests' xorshift64 generator (quant_q8k.rs:302-313)."""

    def __init__(self, seed):
        self.s = C.c_uint64(seed)

    def next(self):
        return lib().or_rng_next(C.byref(self.s))

    def f(self, lo, hi):
        return lib().or_rng_f(C.byref(self.s), lo, hi)

    def fill(self, lo, hi, n):
        out = np.empty(n, np.float32)
        lib().or_rng_fill_f32(C.byref(self.s), lo, hi, _p(out), n)
        return out


def row_bytes(dtype, cols):
    r = lib().or_row_bytes(dtype, cols)
    if r < 0:
        raise ValueError("unsupported dtype %d / width %d" % (dtype, cols))
    return r


def random_matrix(dtype, cols, rows, rng):
    """quant_q8k.rs:323-336 (+ Q8_0 / F32 from quant_multi.rs:301-322)."""
    out = np.empty(row_bytes(dtype, cols) * rows, np.uint8)
    if lib().or_random_matrix(dtype, cols, rows, C.byref(rng.s), _p(out)):
        raise ValueError("random_matrix: unsupported dtype %d" % dtype)
    return out


def random_row(dtype, cols, rng):
    """quant.rs:1693-1723."""
    out = np.empty(row_bytes(dtype, cols), np.uint8)
    if lib().or_random_row(dtype, cols, C.byref(rng.s), _p(out)):
        raise ValueError("random_row: unsupported dtype %d" % dtype)
    return out


def dequant_row(dtype, row, cols):
    row = np.ascontiguousarray(row, np.uint8)
    out = np.empty(cols, np.float32)
    if lib().or_dequant_row(dtype, _p(row), cols, _p(out)):
        raise ValueError("dequant_row: unsupported dtype %d" % dtype)
    return out


class Q8K:
    """One quantized activation vector (quant_q8k.rs:61-65)."""

    def __init__(self, d, qs, bsums):
        self.d, self.qs, self.bsums = d, qs, bsums

    def dequant(self):
        return (self.d.repeat(QK) * self.qs.astype(np.float32)).astype(np.float32)


def quantize(x):
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    if n % QK:
        raise ValueError("length must be a multiple of 256")
    d = np.empty(n // QK, np.float32)
    qs = np.empty(n, np.int8)
    bs = np.empty(n // 16, np.int16)
    lib().or_q8k_quantize(_p(x), n, _p(d), _p(qs), _p(bs))
    return Q8K(d, qs, bs)


def _ptrs(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def matmul_rows(w, mat, qs, outs, r0, r1):
    """quant_q8k::matmul_rows: rows r0..r1 of outs[b] = W * qs[b]."""
    w = np.ascontiguousarray(w, np.uint8)
    rc = lib().or_matmul_rows(_p(w), C.byref(mat), len(qs), _ptrs([q.d for q in qs]),
                              _ptrs([q.qs for q in qs]), _ptrs([q.bsums for q in qs]),
                              _ptrs(outs), r0, r1)
    if rc:
        raise ValueError("matmul_rows: unsupported matrix")


def gemv_int(w, mat, qs):
    """All rows for a list of Q8K vectors -> float32 [n_vec, rows]."""
    out = np.full((len(qs), mat.rows), np.nan, np.float32)
    matmul_rows(w, mat, qs, [out[b] for b in range(len(qs))], 0, mat.rows)
    return out


def block_sums(w, mat, q, r0, r1):
    """int32 [r1-r0, nb, 8] lane sums of quant_q8k.rs:235-242 for one vector."""
    w = np.ascontiguousarray(w, np.uint8)
    nb = mat.cols // QK
    out = np.empty((r1 - r0, nb, 8), np.int32)
    if lib().or_block_sums(_p(w), C.byref(mat), _p(q.qs), r0, r1, _p(out)):
        raise ValueError("block_sums: unsupported matrix")
    return out


def matvec_rows(w, mat, x, r0, n_rows):
    """quant::matvec_rows_avx2 (float kernels)."""
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    if lib().or_matvec_rows(_p(w), C.byref(mat), _p(x), _p(out), r0, n_rows):
        raise ValueError("matvec_rows: unsupported dtype %d" % mat.dtype)
    return out


def matmul_rows_multi(w, mat, xs, r0, r1):
    """quant_multi::matmul_rows_avx2 -> float32 [n_vec, rows] (rows outside r0..r1 NaN)."""
    w = np.ascontiguousarray(w, np.uint8)
    xs = [np.ascontiguousarray(x, np.float32) for x in xs]
    out = np.full((len(xs), mat.rows), np.nan, np.float32)
    rc = lib().or_matmul_rows_multi(_p(w), C.byref(mat), len(xs), _ptrs(xs),
                                    _ptrs([out[b] for b in range(len(xs))]), r0, r1)
    if rc:
        raise ValueError("matmul_rows_multi: unsupported dtype %d" % mat.dtype)
    return out


def pool_create(n_threads):
    return lib().or_pool_create(n_threads)


def pool_destroy():
    lib().or_pool_destroy()


def pool_matvec_multi(w, mat, xs, out):
    """matvec / matvec_multi on the worker pool; xs [n_vec, cols] -> out [n_vec, rows]."""
    rc = lib().or_pool_matvec_multi(_p(w), C.byref(mat), xs.shape[0], _p(xs), _p(out))
    if rc:
        raise RuntimeError("pool_matvec_multi failed (%d)" % rc)


def quantize_weights(dtype, w):
    """The build's f32 -> Q4_K / Q6_K quantizer (kquant.c); w is [rows, cols]."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    out = np.empty(row_bytes(dtype, cols) * rows, np.uint8)
    if dtype == Q4_K:
        lib().or_quantize_q4k(_p(w), w.size, _p(out))
    elif dtype == Q6_K:
        lib().or_quantize_q6k(_p(w), w.size, _p(out))
    else:
        raise ValueError("quantize_weights: dtype %d" % dtype)
    return out


class Moe(C.Structure):
    """`Moe` of smollm_chat.rs:152-169 (without residency): router and expert-0 views."""
    _fields_ = [("router", Mat), ("gate", Mat), ("up", Mat), ("down", Mat), ("n_expert", C.c_uint32),
                ("n_used", C.c_uint32), ("norm", C.c_int32), ("moe_prune", C.c_float), ("has_shared", C.c_int32),
                ("has_shared_gate", C.c_int32), ("sh_gate", Mat), ("sh_up", Mat), ("sh_down", Mat),
                ("shared_gate_offset", C.c_uint64)]


def _moe_sigs():
    L = lib()
    if not hasattr(L, "_moe_ready"):
        P, S = C.c_void_p, C.c_size_t
        L.or_moe_forward.restype = C.c_int
        L.or_moe_forward.argtypes = [P, C.POINTER(Moe), P, P, C.c_int, P, P, C.POINTER(C.c_uint32)]
        L.or_moe_route.restype = C.c_int
        L.or_moe_route.argtypes = [P, C.POINTER(Moe), P, P, P, P, C.POINTER(C.c_uint32)]
        L.or_ffns_fused.restype = C.c_int
        L.or_ffns_fused.argtypes = [P, P, P, P, P, S, P, P, C.c_int]
        L._moe_ready = True
    return L


def moe_forward(buf, moe, x, int_on=True):
    """moe_forward (smollm_chat.rs:1178-1392): returns (out, chosen experts, weights)."""
    L = _moe_sigs()
    buf = np.ascontiguousarray(buf, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(moe.down.rows, np.float32)
    chosen = np.empty(moe.n_used, np.int32)
    ws = np.empty(moe.n_used, np.float32)
    n = C.c_uint32()
    if L.or_moe_forward(_p(buf), C.byref(moe), _p(x), _p(out), int(int_on), _p(chosen), _p(ws), C.byref(n)):
        raise RuntimeError("moe_forward failed")
    return out, chosen[:n.value].copy(), ws[:n.value].copy()


def moe_route(buf, moe, x):
    """Router + softmax + top-k + prune: (probs, chosen, weights)."""
    L = _moe_sigs()
    buf = np.ascontiguousarray(buf, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    probs = np.empty(moe.n_expert, np.float32)
    chosen = np.empty(moe.n_used, np.int32)
    ws = np.empty(moe.n_used, np.float32)
    n = C.c_uint32()
    if L.or_moe_route(_p(buf), C.byref(moe), _p(x), _p(probs), _p(chosen), _p(ws), C.byref(n)):
        raise RuntimeError("moe_route failed")
    return probs, chosen[:n.value].copy(), ws[:n.value].copy()


def ffns_fused(buf, gates, ups, downs, weights, x, out, int_on=True):
    """ffns_fused (smollm_chat.rs:382-442): out += sum_e w_e * FFN_e(x), in order."""
    L = _moe_sigs()
    k = len(gates)
    arr = lambda ms: (Mat * k)(*ms)
    w = np.ascontiguousarray(weights, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    if L.or_ffns_fused(_p(np.ascontiguousarray(buf, np.uint8)), arr(gates), arr(ups), arr(downs), _p(w), k, _p(x),
                       _p(out), int(int_on)):
        raise RuntimeError("ffns_fused failed")
    return out


# ---- decoder forward pass (smollm_chat.rs:3371-3552) ----

NO_NORM = 0xFFFFFFFFFFFFFFFF


class Layer(C.Structure):
    """One decoder layer: norm offsets, attention matrices, dense FFN or MoE."""
    _fields_ = [("attn_norm", C.c_uint64), ("ffn_norm", C.c_uint64), ("q_norm", C.c_uint64),
                ("k_norm", C.c_uint64), ("wq", Mat), ("wk", Mat), ("wv", Mat), ("wo", Mat),
                ("is_moe", C.c_int32), ("moe", Moe), ("gate", Mat), ("up", Mat), ("down", Mat)]


class Model(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("n_layers", C.c_uint32), ("vocab", C.c_uint32),
                ("max_seq", C.c_uint32), ("rope_neox", C.c_int32), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("residual_scale", C.c_float), ("embedding_scale", C.c_float),
                ("attn_scale", C.c_float), ("embed", Mat), ("lm_head", Mat), ("output_norm", C.c_uint64),
                ("layers", C.POINTER(Layer))]


def _fwd_sigs():
    L = lib()
    if not hasattr(L, "_fwd_ready"):
        P = C.c_void_p
        L.or_forward.restype = C.c_int
        L.or_forward.argtypes = [P, C.POINTER(Model), P, P, C.c_int64, P, C.c_uint32, C.c_int, P, P]
        L.or_argmax.restype = C.c_int64
        L.or_argmax.argtypes = [P, C.c_size_t]
        L.or_rmsnorm.restype = None
        L.or_rmsnorm.argtypes = [P, P, P, C.c_size_t, C.c_float]
        L.or_rope_freqs.restype = None
        L.or_rope_freqs.argtypes = [C.c_float, C.c_uint32, P]
        L.or_kv_shift.restype = C.c_uint32
        L.or_kv_shift.argtypes = [C.POINTER(Model), P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.or_rope_rotate.restype = None
        L.or_rope_rotate.argtypes = [P, C.c_size_t, C.c_uint32, P, C.c_int32, C.c_float]
        L._fwd_ready = True
    return L


class Decoder:
    """A model (weights in one byte buffer, GGUF-like offsets) with its own f16 KV cache."""

    def __init__(self, buf, model, layers):
        self.buf = np.ascontiguousarray(buf, np.uint8)
        self.layers = (Layer * len(layers))(*layers)
        model.layers = self.layers
        self.model = model
        kv = model.n_layers * model.max_seq * model.n_kv_heads * model.head_dim
        self.kcache = np.zeros(kv, np.uint16)
        self.vcache = np.zeros(kv, np.uint16)

    def forward(self, token, pos, int_on=True, logits=True):
        """One token (id, or an fp32 hidden vector) at pos: (output-normed hidden, logits or None)."""
        L = _fwd_sigs()
        m = self.model
        hidden = np.empty(m.dim, np.float32)
        out = np.empty(m.vocab, np.float32) if logits else None
        tok, xin = (int(token), None) if np.isscalar(token) else (-1, np.ascontiguousarray(token, np.float32))
        rc = L.or_forward(_p(self.buf), C.byref(m), _p(self.kcache), _p(self.vcache), tok,
                          None if xin is None else _p(xin), pos, int(int_on), _p(hidden),
                          None if out is None else _p(out))
        if rc:
            raise RuntimeError("or_forward failed (%d)" % rc)
        return hidden, out

    def kv_shift(self, n_keep, n_discard, cur_pos, l0=0, l1=None):
        """shift_kv (smollm_chat.rs:2942-2972) on layers [l0, l1); returns the new position."""
        l1 = self.model.n_layers if l1 is None else l1
        return int(_fwd_sigs().or_kv_shift(C.byref(self.model), _p(self.kcache), _p(self.vcache), l0, l1, n_keep,
                                           n_discard, cur_pos))


def argmax(logits):
    """Greedy token: largest under f32::total_cmp, the last one on ties."""
    a = np.ascontiguousarray(logits, np.float32)
    return int(_fwd_sigs().or_argmax(_p(a), a.size))


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    _fwd_sigs().or_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def rope_freqs(theta, head_dim):
    out = np.empty(head_dim // 2, np.float32)
    _fwd_sigs().or_rope_freqs(theta, head_dim, _p(out))
    return out


def rope_rotate(v, head_dim, inv_freq, neox, pos):
    """Rope::rotate (smollm_chat.rs:1409-1419) on a copy of v."""
    v = np.array(v, np.float32, copy=True)
    f = np.ascontiguousarray(inv_freq, np.float32)
    _fwd_sigs().or_rope_rotate(_p(v), v.size, head_dim, _p(f), int(neox), pos)
    return v



# ---- the reference's synthetic benchmark kernels (synth.c) -------------------

SYNTH = dict(hidden=4096, row_bytes=2304, n_expert=8, layers=32, max_seq=512, kv_dim=1024, kv_heads=8, spec=4)


def _synth_sigs():
    L = lib()
    if not hasattr(L, "_synth_ready"):
        P, U64 = C.c_void_p, C.c_uint64
        L.or_synth_f16.restype = C.c_float
        L.or_synth_f16.argtypes = [C.c_uint16]
        L.or_q4k_block_dot.restype = C.c_float
        L.or_q4k_block_dot.argtypes = [P, P]
        L.or_q4k_gemv_4row.restype = U64
        L.or_q4k_gemv_4row.argtypes = [P, U64, P, P, U64]
        L.or_q4k_gemm_spec4.restype = None
        L.or_q4k_gemm_spec4.argtypes = [P, U64, U64, P, P, U64]
        L.or_route_moe_top2.restype = None
        L.or_route_moe_top2.argtypes = [P, P, U64, P, P]
        L.or_kvcache_init.restype = None
        L.or_kvcache_init.argtypes = [P, P, P, P, U64]
        L.or_flash_gqa_spec4.restype = None
        L.or_flash_gqa_spec4.argtypes = [P, P, P, P, P, U64, U64]
        L._synth_ready = True
    return L


def synth_f16(h):
    """q4k_gemv.rs's f16_to_f32 (non-IEEE: exponents clamped, 0x7C00.. finite)."""
    return float(_synth_sigs().or_synth_f16(int(h)))


def q4k_block_dot(blk, act):
    """q4k_block_dot_avx2: one 144-byte block against 256 floats."""
    blk = np.ascontiguousarray(blk, np.uint8)
    act = np.ascontiguousarray(act, np.float32)
    return float(_synth_sigs().or_q4k_block_dot(_p(blk), _p(act)))


def q4k_gemv_4row(chunk, x, y, row_offset=0):
    """q4k_gemv_4row_avx2 into y (float32 [4096], updated in place); rows done."""
    chunk = np.ascontiguousarray(chunk, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    return int(_synth_sigs().or_q4k_gemv_4row(_p(chunk), chunk.size, _p(x), _p(y), row_offset))


def q4k_gemm_spec4(chunk, r0, r1, x4, y4, base=0):
    """q4k_gemm_spec4_slice_avx2: rows [r0, r1) for x4 [4][4096] into y4 [4][4096] (in place)."""
    chunk = np.ascontiguousarray(chunk, np.uint8)
    x4 = np.ascontiguousarray(x4, np.float32)
    _synth_sigs().or_q4k_gemm_spec4(_p(chunk), r0, r1, _p(x4), _p(y4), base)


def route_moe_top2(x, gates, layer):
    """route_moe_top2: (experts [2], weights [2])."""
    x = np.ascontiguousarray(x, np.float32)
    gates = np.ascontiguousarray(gates, np.float32)
    ex = np.zeros(2, np.int32)
    w = np.zeros(2, np.float32)
    _synth_sigs().or_route_moe_top2(_p(x), _p(gates), layer, _p(ex), _p(w))
    return ex, w


def kvcache_init(init_ctx):
    """QuantizedKvCache::new(init_ctx): (k, v, k_scale, v_scale, seq_len)."""
    S = SYNTH
    k = np.zeros(S["layers"] * S["max_seq"] * S["kv_dim"], np.int8)
    v = np.zeros_like(k)
    ks = np.zeros(S["layers"] * S["max_seq"] * S["kv_heads"], np.float32)
    vs = np.zeros_like(ks)
    _synth_sigs().or_kvcache_init(_p(k), _p(v), _p(ks), _p(vs), init_ctx)
    return k, v, ks, vs, min(init_ctx, S["max_seq"] - S["spec"])


def flash_gqa_spec4(q_spec, cache, layer):
    """flash_decoding_gqa_spec4_avx2 on q_spec [4][4096] (updated in place) and
    the cache of kvcache_init (updated: the four new K/V rows)."""
    k, v, ks, vs, seq = cache
    _synth_sigs().or_flash_gqa_spec4(_p(q_spec), _p(k), _p(v), _p(ks), _p(vs), seq, layer)
