"""Decoder step on the GPU (forward_slice, smollm_chat.rs:3371-3552, greedy
sampling :3661-3671) through the C ABI: sg_model_*, sg_forward.

A model is a dict of weights named like the GGUF tensors of one architecture
(Qwen3 / Qwen3-MoE): `embed` [vocab][dim] and `head` [vocab][dim] (K-quant or
F32/F16 GGUF rows), `out_norm` [dim]; per layer i `l{i}.attn_norm`,
`l{i}.ffn_norm`, optional `l{i}.q_norm` / `l{i}.k_norm` [head_dim], `l{i}.wq`
[q_dim][dim], `l{i}.wk` / `l{i}.wv` [kv_dim][dim], `l{i}.wo` [dim][q_dim], and
either the dense FFN `l{i}.gate` / `l{i}.up` [n_ff][dim], `l{i}.down`
[dim][n_ff] or the MoE `l{i}.router` F32 [n_expert][dim], `l{i}.gate_exps`,
`l{i}.up_exps` [n_expert * n_ff][dim], `l{i}.down_exps` [n_expert * dim][n_ff].
"""
import ctypes as C

import torch

from . import _lib, lib, _stream, repack_tiled16, tiled16_bytes, Q4_K, Q6_K, F32, F16
from . import quantize_weights as _quantize_weights
from ._lib import SgError, SgMoe


class SgLayer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
                ("wq_dtype", C.c_int32), ("wk_dtype", C.c_int32), ("wv_dtype", C.c_int32), ("wo_dtype", C.c_int32),
                ("is_moe", C.c_int32), ("moe", SgMoe), ("ffn_gate_up", C.c_void_p), ("ffn_down", C.c_void_p),
                ("ffn_gate_up_dtype", C.c_int32), ("ffn_down_dtype", C.c_int32), ("n_ff", C.c_uint64)]


class SgModel(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("n_layers", C.c_uint32), ("vocab", C.c_uint32), ("max_seq", C.c_uint32), ("rope_neox", C.c_int32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("residual_scale", C.c_float),
                ("embedding_scale", C.c_float), ("attn_scale", C.c_float), ("embed", C.c_void_p),
                ("embed_dtype", C.c_int32), ("lm_head", C.c_void_p), ("lm_head_dtype", C.c_int32),
                ("output_norm", C.c_void_p), ("layers", C.POINTER(SgLayer))]


def _sigs():
    L = lib()
    if not hasattr(L, "_dec_ready"):
        P = C.c_void_p
        L.sg_model_scratch_bytes.restype = C.c_uint64
        L.sg_model_scratch_bytes.argtypes = [C.POINTER(SgModel)]
        L.sg_model_kv_bytes.restype = C.c_uint64
        L.sg_model_kv_bytes.argtypes = [C.POINTER(SgModel)]
        L.sg_model_prepare.restype = C.c_int32
        L.sg_model_prepare.argtypes = [C.POINTER(SgModel), P, C.c_uint64, P]
        L.sg_forward.restype = C.c_int32
        L.sg_forward.argtypes = [C.POINTER(SgModel), P, P, P, C.c_uint64, P, P, P, P]
        L.sg_model_ep_scratch_bytes.restype = C.c_uint64
        L.sg_model_ep_scratch_bytes.argtypes = [C.POINTER(SgModel)]
        L.sg_forward_ep.restype = C.c_int32
        L.sg_forward_ep.argtypes = [C.POINTER(SgModel), P, P, P, P, C.c_uint64, P, P, P, P]
        L.sg_model_batch_scratch_bytes.restype = C.c_uint64
        L.sg_model_batch_scratch_bytes.argtypes = [C.POINTER(SgModel), C.c_uint64]
        L.sg_model_batch_prepare.restype = C.c_int32
        L.sg_model_batch_prepare.argtypes = [C.POINTER(SgModel), C.c_uint64, P, C.c_uint64, P]
        L.sg_forward_batch_range.restype = C.c_int32
        L.sg_forward_batch_range.argtypes = [C.POINTER(SgModel), C.c_uint32, C.c_uint32, P, P, C.c_uint64, P, P, P,
                                             C.c_uint64, C.c_uint64, P, P, C.c_uint64, P, P]
        L.sg_forward_batch.restype = C.c_int32
        L.sg_forward_batch.argtypes = [C.POINTER(SgModel), P, C.c_uint64, P, P, P, C.c_uint64, C.c_uint64, P,
                                       C.c_uint64, P, P]
        L._dec_ready = True
    return L


def _ptr(t):
    return None if t is None else t.data_ptr()


class Decoder:
    """Device weights, KV cache, scratch and the {token, pos} state of one model."""

    def __init__(self, cfg, weights, dtypes, device, qk_adjacent=True, ep=None):
        """weights: name -> CUDA tensor (uint8 GGUF rows for matrices, float32
        vectors); dtypes: name -> GGML dtype of each matrix.  qk_adjacent: store
        each layer's wk right after its wq when both have one format, which lets
        sg_forward compute q and k in one launch.  ep: a spindle_b200.tp.TpGroup
        to spread every MoE layer's experts over its ranks (sg_forward_ep; every
        rank builds the Decoder with the same weights, in the same order, and
        steps it with the same state); the batch forms are then unavailable."""
        self.cfg, self.dev, self.ep = dict(cfg), device, ep
        c = self.cfg
        self.keep = []  # every device buffer the model points at
        dim, hd = c["dim"], c["head_dim"]
        q_dim, kv_dim = c["n_heads"] * hd, c["n_kv_heads"] * hd

        def tiled(name, rows, cols):
            t, _ = repack_tiled16(dtypes[name], weights[name], rows, cols)
            self.keep.append(t)
            return t.data_ptr()

        def tiled_pair(a, rows_a, b, rows_b, cols):
            # both matrices in one buffer, b's tiles right after a's
            na, nb = tiled16_bytes(dtypes[a], rows_a, cols), tiled16_bytes(dtypes[b], rows_b, cols)
            t = torch.empty(na + nb, dtype=torch.uint8, device=device)
            for name, rows, off in [(a, rows_a, 0), (b, rows_b, na)]:
                _lib.check(lib().sg_repack_tiled16(dtypes[name], C.c_void_p(weights[name].data_ptr()), rows, cols,
                                                   C.c_void_p(t.data_ptr() + off), _stream()), "repack_tiled16")
            self.keep.append(t)
            return t.data_ptr(), t.data_ptr() + na

        def vec(name):
            t = weights.get(name)
            if t is None:
                return None
            t = t.contiguous()
            self.keep.append(t)
            return t.data_ptr()

        layers = []
        moe = c.get("moe")
        self._eps = []
        for i in range(c["n_layers"]):
            p = "l%d." % i
            y = SgLayer()
            y.attn_norm, y.ffn_norm = vec(p + "attn_norm"), vec(p + "ffn_norm")
            y.q_norm, y.k_norm = vec(p + "q_norm"), vec(p + "k_norm")
            if qk_adjacent and dtypes[p + "wq"] == dtypes[p + "wk"]:
                y.wq, y.wk = tiled_pair(p + "wq", q_dim, p + "wk", kv_dim, dim)
            else:
                y.wq, y.wk = tiled(p + "wq", q_dim, dim), tiled(p + "wk", kv_dim, dim)
            y.wq_dtype, y.wk_dtype = dtypes[p + "wq"], dtypes[p + "wk"]
            y.wv, y.wv_dtype = tiled(p + "wv", kv_dim, dim), dtypes[p + "wv"]
            y.wo, y.wo_dtype = tiled(p + "wo", dim, q_dim), dtypes[p + "wo"]
            if moe and ep is not None:
                # this rank's experts only; the router and the choice stay whole
                from .tp import EpMoe
                em = EpMoe(ep, weights[p + "router"].float(), weights[p + "gate_exps"], weights[p + "up_exps"],
                           weights[p + "down_exps"], dtypes[p + "gate_exps"], dtypes[p + "down_exps"],
                           moe["n_expert"], moe["n_used"], dim, moe["n_ff"], n_tok_max=1,
                           norm=moe.get("norm", True), moe_prune=moe.get("prune", 0.0))
                self.keep.append(em)
                y.is_moe, y.moe = 1, em.moe.c()
                self._eps.append(em.c())
            elif moe:
                from . import Moe
                m = Moe.pack(weights[p + "router"].float(), weights[p + "gate_exps"], weights[p + "up_exps"],
                             weights[p + "down_exps"], dtypes[p + "gate_exps"], dtypes[p + "down_exps"],
                             moe["n_expert"], moe["n_used"], dim, moe["n_ff"], norm=moe.get("norm", True),
                             moe_prune=moe.get("prune", 0.0))
                self.keep.append(m)
                y.is_moe, y.moe = 1, m.c()
            else:
                from . import Moe
                f = c["n_ff"]
                one = Moe.pack(torch.zeros(1, dim, device=device), weights[p + "gate"], weights[p + "up"],
                               weights[p + "down"], dtypes[p + "gate"], dtypes[p + "down"], 1, 1, dim, f)
                self.keep.append(one)
                y.is_moe = 0
                y.ffn_gate_up, y.ffn_down = one.gate_up.data_ptr(), one.down.data_ptr()
                y.ffn_gate_up_dtype, y.ffn_down_dtype, y.n_ff = dtypes[p + "gate"], dtypes[p + "down"], f
            if ep is not None and not moe:
                from ._lib import SgMoeEp
                self._eps.append(SgMoeEp())  # not read for a dense layer
            layers.append(y)
        self.layers = (SgLayer * len(layers))(*layers)
        m = SgModel()
        m.dim, m.n_heads, m.n_kv_heads, m.head_dim = dim, c["n_heads"], c["n_kv_heads"], hd
        m.n_layers, m.vocab, m.max_seq = c["n_layers"], c["vocab"], c["max_seq"]
        m.rope_neox, m.rope_theta, m.rms_eps = int(c.get("rope_neox", True)), c["rope_theta"], c["rms_eps"]
        m.residual_scale, m.embedding_scale = c.get("residual_scale", 1.0), c.get("embedding_scale", 1.0)
        m.attn_scale = c.get("attn_scale", 0.0)
        emb = weights["embed"].contiguous()
        self.keep.append(emb)
        m.embed, m.embed_dtype = emb.data_ptr(), dtypes["embed"]
        m.lm_head, m.lm_head_dtype = tiled("head", c["vocab"], dim), dtypes["head"]
        m.output_norm = vec("out_norm")
        m.layers = self.layers
        self.model = m
        L = _sigs()
        if ep is not None:
            from ._lib import SgMoeEp
            self.eps = (SgMoeEp * len(self._eps))(*self._eps)
        nbytes = L.sg_model_ep_scratch_bytes(C.byref(m)) if ep is not None else L.sg_model_scratch_bytes(C.byref(m))
        if not nbytes:
            raise SgError(1, "sg_model_scratch_bytes (invalid model)")
        self.scratch = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.kv = torch.zeros(L.sg_model_kv_bytes(C.byref(m)), dtype=torch.uint8, device=device)
        self.state = torch.zeros(2, dtype=torch.int32, device=device)
        self.logits = torch.empty(c["vocab"], dtype=torch.float32, device=device)
        self.hidden = torch.empty(dim, dtype=torch.float32, device=device)
        self.token = torch.zeros(1, dtype=torch.int64, device=device)
        _lib.check(L.sg_model_prepare(C.byref(m), C.c_void_p(self.scratch.data_ptr()), self.scratch.numel(),
                                      _stream()), "sg_model_prepare")

    def set_state(self, token, pos, stream=None):
        self.state.copy_(torch.tensor([token, pos], dtype=torch.int32), non_blocking=False)

    def step(self, stream=None, hidden=True, logits=True):
        """One decoder step on the device state; the state then holds the greedy
        token and the next position."""
        L = _sigs()
        args = (C.c_void_p(self.state.data_ptr()), C.c_void_p(self.kv.data_ptr()), C.c_void_p(self.scratch.data_ptr()),
                self.scratch.numel(), C.c_void_p(self.hidden.data_ptr()) if hidden else None,
                C.c_void_p(self.logits.data_ptr()) if logits else None, C.c_void_p(self.token.data_ptr()),
                _stream(stream))
        if self.ep is not None:
            _lib.check(L.sg_forward_ep(C.byref(self.model), C.cast(self.eps, C.c_void_p), *args), "sg_forward_ep")
        else:
            _lib.check(L.sg_forward(C.byref(self.model), *args), "sg_forward")

    def shift_kv(self, n_keep, n_discard, cur_pos, l0=0, l1=None, stream=None):
        """shift_kv (smollm_chat.rs:2942-2972) on the device caches of layers
        [l0, l1) (a pipeline stage shifts its own): positions [n_keep +
        n_discard, cur_pos) move down by n_discard, K re-rotated by -n_discard.
        Returns the new position, cur_pos - n_discard (n_discard clamped to
        cur_pos - n_keep); the caller continues from it (set_state)."""
        l1 = self.cfg["n_layers"] if l1 is None else l1
        n_discard = min(n_discard, max(cur_pos - n_keep, 0))
        _lib.check(lib().sg_kv_shift(C.byref(self.model), C.c_void_p(self.kv.data_ptr()),
                                     C.c_void_p(self.scratch.data_ptr()), l0, l1, n_keep, n_discard, cur_pos,
                                     _stream(stream)), "sg_kv_shift")
        return cur_pos - n_discard

    def kv_room(self, cur_pos, needed, n_keep):
        """ensure_kv_room's choice (smollm_chat.rs:2924-2940): 0 when needed
        more positions fit, else how many to discard (at least the overflow,
        rounded up to half of the unpinned window, at most all of it)."""
        if cur_pos + needed <= self.cfg["max_seq"]:
            return 0
        n_ctx = cur_pos - n_keep
        want = max(cur_pos + needed - self.cfg["max_seq"], n_ctx // 2)
        return min(want, n_ctx)

    def ensure_kv_room(self, cur_pos, needed, n_keep, stream=None):
        """ensure_kv_room (smollm_chat.rs:2924-2940): shifts when cur_pos +
        needed would pass max_seq; returns the position to continue from."""
        n_discard = self.kv_room(cur_pos, needed, n_keep)
        return self.shift_kv(n_keep, n_discard, cur_pos, stream=stream) if n_discard else cur_pos

    def forward_batch(self, tokens, pos0, logits=True, n_max=64, stream=None):
        """forward_batch_slice + compute_logits_batch: tokens at positions
        pos0 .. pos0 + n - 1 in one call (their K/V rows enter the cache).
        Returns (logits [n, vocab] or None, greedy next tokens int64 [n]); per
        token bit for bit the one-token step."""
        if self.ep is not None:
            raise ValueError("the batch forward is not expert-parallel; build the Decoder without ep")
        L = _sigs()
        n = len(tokens)
        n_max = max(n_max, n)
        if getattr(self, "_bscratch", None) is None or self._bn < n_max:
            nbytes = L.sg_model_batch_scratch_bytes(C.byref(self.model), n_max)
            if not nbytes:
                raise SgError(3, "sg_model_batch_scratch_bytes")
            self._bscratch = torch.empty(nbytes, dtype=torch.uint8, device=self.dev)
            self._bn = n_max
            _lib.check(L.sg_model_batch_prepare(C.byref(self.model), n_max, C.c_void_p(self._bscratch.data_ptr()),
                                                nbytes, _stream(stream)), "sg_model_batch_prepare")
        toks = torch.tensor(list(tokens), dtype=torch.int32, device=self.dev)
        pos = torch.tensor([pos0], dtype=torch.int32, device=self.dev)
        lg = torch.empty(n, self.cfg["vocab"], dtype=torch.float32, device=self.dev) if logits else None
        greedy = torch.empty(n, dtype=torch.int64, device=self.dev)
        _lib.check(L.sg_forward_batch(C.byref(self.model), C.c_void_p(toks.data_ptr()), n, C.c_void_p(pos.data_ptr()),
                                      C.c_void_p(self.kv.data_ptr()), C.c_void_p(self._bscratch.data_ptr()),
                                      self._bscratch.numel(), self._bn,
                                      C.c_void_p(lg.data_ptr()) if logits else None, self.cfg["vocab"],
                                      C.c_void_p(greedy.data_ptr()), _stream(stream)), "sg_forward_batch")
        return lg, greedy

    def forward_batch_range(self, pos0, l0, l1, tokens=None, hidden=None, n_max=64, stream=None, head=True):
        """A pipeline stage: layers [l0, l1) for positions pos0 .. pos0 + n - 1.
        The first stage takes tokens, later ones the raw residual `hidden`
        (float32 CUDA [n, dim]); a middle stage returns the raw residual, the
        last one (logits [n, vocab], greedy tokens int64 [n]), or with
        head=False the output-normed hidden states (forward_batch_slice's
        return value) and no LM head."""
        if self.ep is not None:
            raise ValueError("the batch forward is not expert-parallel; build the Decoder without ep")
        L = _sigs()
        n = len(tokens) if tokens is not None else hidden.shape[0]
        n_max = max(n_max, n)
        if getattr(self, "_bscratch", None) is None or self._bn < n_max:
            nbytes = L.sg_model_batch_scratch_bytes(C.byref(self.model), n_max)
            if not nbytes:
                raise SgError(3, "sg_model_batch_scratch_bytes")
            self._bscratch = torch.empty(nbytes, dtype=torch.uint8, device=self.dev)
            self._bn = n_max
            _lib.check(L.sg_model_batch_prepare(C.byref(self.model), n_max, C.c_void_p(self._bscratch.data_ptr()),
                                                nbytes, _stream(stream)), "sg_model_batch_prepare")
        toks = None if tokens is None else torch.tensor(list(tokens), dtype=torch.int32, device=self.dev)
        pos = torch.tensor([pos0], dtype=torch.int32, device=self.dev)
        last = l1 == self.cfg["n_layers"]
        with_head = last and head
        out = None if with_head else torch.empty(n, self.cfg["dim"], dtype=torch.float32, device=self.dev)
        lg = torch.empty(n, self.cfg["vocab"], dtype=torch.float32, device=self.dev) if with_head else None
        greedy = torch.empty(n, dtype=torch.int64, device=self.dev) if with_head else None
        ptr = lambda t: None if t is None else C.c_void_p(t.data_ptr())
        _lib.check(L.sg_forward_batch_range(C.byref(self.model), l0, l1, ptr(toks), ptr(hidden), n, ptr(pos),
                                            ptr(self.kv), ptr(self._bscratch), self._bscratch.numel(), self._bn,
                                            ptr(out), ptr(lg), self.cfg["vocab"], ptr(greedy), _stream(stream)),
                   "sg_forward_batch_range")
        return (lg, greedy) if with_head else (out,)

    def feed(self, tokens, pos0=0, chunk=128, stream=None):
        """feed (smollm_chat.rs:3042-3106): the prompt in chunks of `chunk`
        positions (128 as the reference's, at most SG_MOE_MAX_BATCH = 128),
        K/V rows into the caches, no LM head; returns the last position's
        output-normed hidden state (float32 CUDA [dim])."""
        tokens = list(tokens)
        last = None
        for c0 in range(0, len(tokens), chunk):
            part = tokens[c0:c0 + chunk]
            (last,) = self.forward_batch_range(pos0 + c0, 0, self.cfg["n_layers"], tokens=part,
                                               n_max=max(chunk, getattr(self, "_bn", 0) or 0), stream=stream,
                                               head=False)
        return None if last is None else last[-1]

    def feed_overlapped(self, tokens, pos0=0, chunk=128, streams=None, in_flight=2):
        """feed with in_flight chunks in flight: chunk c runs a layer at a
        time on stream c % in_flight with its own scratch
        (sg_forward_batch_range continuing on that scratch), its layer l after
        chunk c - 1's layer l (whose K/V rows it reads), so one chunk's
        latency-bound kernels overlap the others'.  Every layer's arithmetic
        is feed's, so the caches and the returned hidden state are bit for
        bit feed's.  streams: in_flight torch.cuda.Streams (made here if None;
        the caller's current stream waits for all of them before this
        returns)."""
        if self.ep is not None:
            raise ValueError("the batch forward is not expert-parallel; build the Decoder without ep")
        L = _sigs()
        tokens = list(tokens)
        nl = self.cfg["n_layers"]
        if streams is None:
            streams = [torch.cuda.Stream(device=self.dev) for _ in range(in_flight)]
        k = len(streams)
        if k < 1:
            raise ValueError("feed_overlapped needs at least one stream")
        cur = torch.cuda.current_stream(self.dev)
        for st in streams:
            st.wait_stream(cur)
        if getattr(self, "_ovl", None) is None or self._ovl[0] < chunk or len(self._ovl[1]) < k:
            nbytes = L.sg_model_batch_scratch_bytes(C.byref(self.model), chunk)
            if not nbytes:
                raise SgError(3, "sg_model_batch_scratch_bytes")
            bufs = [torch.empty(nbytes, dtype=torch.uint8, device=self.dev) for _ in range(k)]
            for b in bufs:
                _lib.check(L.sg_model_batch_prepare(C.byref(self.model), chunk, C.c_void_p(b.data_ptr()), nbytes,
                                                    _stream(cur)), "sg_model_batch_prepare")
            self._ovl = (chunk, bufs)
        n_max, bufs = self._ovl
        starts = list(range(0, len(tokens), chunk))
        toks = torch.tensor(tokens, dtype=torch.int32, device=self.dev)
        pos = torch.tensor([pos0 + c0 for c0 in starts], dtype=torch.int32, device=self.dev)
        out = torch.empty(chunk, self.cfg["dim"], dtype=torch.float32, device=self.dev)
        for st in streams:
            st.wait_stream(cur)  # the token and position copies above
        prev = None
        ptr = lambda t, off=0: C.c_void_p(t.data_ptr() + off)
        for c, c0 in enumerate(starts):
            st, buf, n = streams[c % k], bufs[c % k], min(chunk, len(tokens) - c0)
            evs = []
            for l in range(nl):
                if prev is not None:
                    st.wait_event(prev[l])
                last = l == nl - 1
                _lib.check(L.sg_forward_batch_range(
                    C.byref(self.model), l, l + 1, ptr(toks, 4 * c0) if l == 0 else None, None, n, ptr(pos, 4 * c),
                    ptr(self.kv), ptr(buf), buf.numel(), n_max, ptr(out) if last else None, None,
                    self.cfg["vocab"], None, _stream(st)), "sg_forward_batch_range")
                ev = torch.cuda.Event()
                ev.record(st)
                evs.append(ev)
            prev = evs
        for st in streams:
            cur.wait_stream(st)
        return out[n - 1] if starts else None

    def generate(self, prompt, n_new):
        """Greedy decode: feed the prompt, then n_new tokens; returns the new tokens."""
        out = []
        for i, t in enumerate(prompt):
            self.set_state(t, i)
            self.step(hidden=False, logits=False)
        for _ in range(n_new):
            out.append(int(self.token.item()))
            self.step(hidden=False, logits=False)
        return out


def random_weights(cfg, dtypes, device, seed=0):
    """Random-init weights of the architecture in cfg, made on the GPU with the
    library's quantizer (N(0, 0.02) matrices, router N(0, 1/dim), norms 1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    c = cfg
    dim, hd = c["dim"], c["head_dim"]
    q_dim, kv_dim = c["n_heads"] * hd, c["n_kv_heads"] * hd

    def mat(name, rows, cols):
        w = torch.randn(rows, cols, device=device, generator=g) * 0.02
        return _quantize_weights(dtypes[name], w)

    W = {"embed": mat("embed", c["vocab"], dim), "head": mat("head", c["vocab"], dim),
         "out_norm": torch.ones(dim, device=device)}
    for i in range(c["n_layers"]):
        p = "l%d." % i
        W[p + "attn_norm"] = torch.ones(dim, device=device)
        W[p + "ffn_norm"] = torch.ones(dim, device=device)
        if c.get("qk_norm", True):
            W[p + "q_norm"] = torch.ones(hd, device=device)
            W[p + "k_norm"] = torch.ones(hd, device=device)
        W[p + "wq"] = mat(p + "wq", q_dim, dim)
        W[p + "wk"] = mat(p + "wk", kv_dim, dim)
        W[p + "wv"] = mat(p + "wv", kv_dim, dim)
        W[p + "wo"] = mat(p + "wo", dim, q_dim)
        moe = c.get("moe")
        if moe:
            ne, f = moe["n_expert"], moe["n_ff"]
            W[p + "router"] = torch.randn(ne, dim, device=device, generator=g) / dim ** 0.5
            W[p + "gate_exps"] = mat(p + "gate_exps", ne * f, dim)
            W[p + "up_exps"] = mat(p + "up_exps", ne * f, dim)
            W[p + "down_exps"] = mat(p + "down_exps", ne * dim, f)
        else:
            f = c["n_ff"]
            W[p + "gate"] = mat(p + "gate", f, dim)
            W[p + "up"] = mat(p + "up", f, dim)
            W[p + "down"] = mat(p + "down", dim, f)
    return W


def qwen3_dtypes(cfg, attn_v=Q6_K, down=Q6_K, head=Q6_K, embed=Q6_K, other=Q4_K):
    """The Q4_K_M mix of the BASELINE configs: Q6_K for attn_v, ffn_down and
    the embedding/head, Q4_K elsewhere."""
    d = {"embed": embed, "head": head}
    for i in range(cfg["n_layers"]):
        p = "l%d." % i
        d.update({p + "wq": other, p + "wk": other, p + "wv": attn_v, p + "wo": other})
        if cfg.get("moe"):
            d.update({p + "gate_exps": other, p + "up_exps": other, p + "down_exps": down})
        else:
            d.update({p + "gate": other, p + "up": other, p + "down": down})
    return d
