"""spindle-b200: spindle's quantized matvec path on B200 (sm_100a).

Host-side mirror of the reference's kernel API (WiseHax/spindle 1.1.0, src/):
  Mat                      quant.rs:914-935
  row_bytes                quant.rs:1527-1542
  supports / set_enabled   quant_q8k.rs:22-57
  Q8K, Q8K.quantize        quant_q8k.rs:61-81
  matmul_rows              quant_q8k.rs:255-295
  matmul_batch             smollm_chat.rs:447-512 (matvec_multi, 9..64 vectors, one pass)
  matvec_rows_float        quant.rs:939-1094 (float path, one vector at a time)
  matmul_rows_float        quant_multi.rs:232-273 (float path, shared decode)
  Moe, moe_forward         smollm_chat.rs:1178-1382
  moe_forward_batch        smollm_chat.rs:928-1174
Every call goes through the C ABI of include/spindle_gpu.h (libspindle_b200.so);
torch tensors are only the device-memory plumbing.  There is no CPU path: a
missing library or a failed call raises.
"""
import ctypes as C

import torch

from . import _lib
from ._lib import SgError, SgMat, SgQ8K

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
GGUF, TILED16 = 0, 1  # weight layouts (sg_mat.layout)
QK = 256
DTYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def lib():
    return _lib.load()


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class Mat:
    """A weight matrix inside a device byte buffer (quant.rs:914-935 `Mat`)."""

    def __init__(self, dtype, cols, rows, offset=0, layout=GGUF):
        self.dtype, self.cols, self.rows, self.offset, self.layout = dtype, cols, rows, offset, layout

    def c(self):
        return SgMat(self.dtype, self.layout, self.offset, self.cols, self.rows)

    def expert(self, e):
        """View of expert e of a 3D tensor (quant.rs:929-934)."""
        return Mat(self.dtype, self.cols, self.rows, self.offset + e * self.rows * row_bytes(self.dtype, self.cols))


def row_bytes(dtype, cols):
    out = C.c_uint64()
    _lib.check(lib().sg_row_bytes(dtype, cols, C.byref(out)), "row_bytes")
    return out.value


def supports(m):
    return bool(lib().sg_supports(C.byref(m.c())))


def set_enabled(on):
    """The --float-kernels switch (quant_q8k.rs:22-24)."""
    lib().sg_set_int_kernels(1 if on else 0)


def enabled():
    return bool(lib().sg_int_kernels_enabled())


class Q8K:
    """One Q8_K activation vector in device memory (quant_q8k.rs:61-65),
    carved from one 16-byte aligned buffer."""

    def __init__(self, n, device=None):
        if n % QK:
            raise ValueError("Q8K length must be a multiple of 256")
        self.n = n
        nbytes = lib().sg_q8k_bytes(n)
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device or "cuda")
        self.desc = SgQ8K()
        _lib.check(lib().sg_q8k_view(C.c_void_p(self.buf.data_ptr()), n, C.byref(self.desc)), "q8k_view")
        nb = n // QK
        self.d = self.buf[:nb * 4].view(torch.float32)
        off_qs = self.desc.qs - self.desc.d
        off_bs = self.desc.bsums - self.desc.d
        self.qs = self.buf[off_qs:off_qs + n].view(torch.int8)
        self.bsums = self.buf[off_bs:off_bs + nb * 32].view(torch.int16)

    def quantize(self, x, stream=None):
        """Q8K::quantize (quant_q8k.rs:73-81) of a float32 CUDA vector."""
        quantize_into(x.reshape(1, -1), [self], stream)
        return self


def quantize_into(xs, outs, stream=None):
    """Quantizes the rows of xs [n_vec, n] (float32, CUDA) into outs (Q8K list)."""
    if xs.dtype != torch.float32 or not xs.is_cuda:
        raise TypeError("expected a float32 CUDA tensor")
    if xs.stride(-1) != 1:
        raise ValueError("rows must be contiguous")
    n_vec, n = xs.shape
    descs = (SgQ8K * n_vec)(*[q.desc for q in outs])
    _lib.check(lib().sg_q8k_quantize(C.c_void_p(xs.data_ptr()), n, n_vec, xs.stride(0), descs, _stream(stream)),
               "q8k_quantize")


def quantize(xs, stream=None):
    """Float32 CUDA [n] or [n_vec, n] -> Q8K (or list of Q8K)."""
    single = xs.dim() == 1
    xs2 = xs.reshape(1, -1) if single else xs
    outs = [Q8K(xs2.shape[1], xs2.device) for _ in range(xs2.shape[0])]
    quantize_into(xs2, outs, stream)
    return outs[0] if single else outs


def matmul_rows(base, m, xq, outs, r0, r1, stream=None):
    """quant_q8k::matmul_rows (quant_q8k.rs:255-295): rows r0..r1 of
    outs[b] = W * xq[b].  base: uint8 CUDA tensor holding the GGUF bytes;
    outs[b]: float32 CUDA tensors of m.rows entries (row r -> outs[b][r])."""
    n = len(xq)
    if len(outs) != n:
        raise ValueError("one output per vector")
    for o in outs:
        if o.dtype != torch.float32 or o.numel() < m.rows:
            raise ValueError("each output must be float32 with m.rows entries")
    descs = (SgQ8K * n)(*[q.desc for q in xq])
    ptrs = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    _lib.check(lib().sg_matmul_rows(C.c_void_p(base.data_ptr()), C.byref(m.c()), descs, ptrs, n, r0, r1,
                                    _stream(stream)), "matmul_rows")


def matvec(base, m, xs, out=None, r0=0, r1=None, stream=None):
    """matvec / matvec_multi (smollm_chat.rs:309, :447) on the integer path:
    fp32 CUDA xs [n_vec, cols] (or [cols]) -> out [n_vec, rows]; the Q8_K
    quantization runs inside the GEMV kernel.  TILED16 weights."""
    single = xs.dim() == 1
    xs2 = xs.reshape(1, -1) if single else xs
    if xs2.dtype != torch.float32 or xs2.stride(-1) != 1:
        raise ValueError("xs must be float32 with contiguous rows")
    r1 = m.rows if r1 is None else r1
    if out is None:
        out = torch.empty((xs2.shape[0], m.rows), dtype=torch.float32, device=xs2.device)
    out2 = out.reshape(1, -1) if out.dim() == 1 else out
    _lib.check(lib().sg_matvec(C.c_void_p(base.data_ptr()), C.byref(m.c()), C.c_void_p(xs2.data_ptr()),
                               xs2.stride(0), C.c_void_p(out2.data_ptr()), out2.stride(0), xs2.shape[0], r0, r1,
                               _stream(stream)), "matvec")
    return out


def matvec_list(entries, outs=None, stream=None):
    """Several matvecs in one launch (sg_matvec_list): entries is a list of
    (base, Mat, x) with x an fp32 CUDA vector of Mat.cols values; returns (or
    fills) one [rows] output per entry, bit for bit matvec's."""
    n = len(entries)
    if outs is None:
        outs = [torch.empty(m.rows, dtype=torch.float32, device=x.device) for _, m, x in entries]
    for _, m, x in entries:
        if x.dtype != torch.float32 or not x.is_contiguous():
            raise ValueError("every x must be a contiguous float32 vector")
    P = C.c_void_p
    bases = (P * n)(*[b.data_ptr() for b, _, _ in entries])
    mats = (_lib.SgMat * n)(*[m.c() for _, m, _ in entries])
    xs = (P * n)(*[x.data_ptr() for _, _, x in entries])
    os_ = (P * n)(*[o.data_ptr() for o in outs])
    _lib.check(lib().sg_matvec_list(bases, mats, xs, os_, n, _stream(stream)), "matvec_list")
    return outs


def q8k_images(xs, imgs=None, stream=None):
    """Q8_K images of fp32 vectors (sg_q8k_images, one launch): a list of uint8
    CUDA tensors of sg_q8k_image_bytes(cols) bytes each."""
    n = len(xs)
    for x in xs:
        if x.dtype != torch.float32 or not x.is_contiguous():
            raise ValueError("every x must be a contiguous float32 vector")
    if imgs is None:
        imgs = [torch.empty(lib().sg_q8k_image_bytes(x.numel()), dtype=torch.uint8, device=x.device) for x in xs]
    P = C.c_void_p
    _lib.check(lib().sg_q8k_images((P * n)(*[x.data_ptr() for x in xs]), (C.c_uint64 * n)(*[x.numel() for x in xs]),
                                   (P * n)(*[t.data_ptr() for t in imgs]), n, _stream(stream)), "q8k_images")
    return imgs


def matvec_list_q8k(entries, outs=None, stream=None):
    """matvec_list on Q8_K images (sg_matvec_list_q8k): entries is a list of
    (base, Mat, img) with img from q8k_images."""
    n = len(entries)
    if outs is None:
        outs = [torch.empty(m.rows, dtype=torch.float32, device=b.device) for b, m, _ in entries]
    P = C.c_void_p
    _lib.check(lib().sg_matvec_list_q8k((P * n)(*[b.data_ptr() for b, _, _ in entries]),
                                        (_lib.SgMat * n)(*[m.c() for _, m, _ in entries]),
                                        (P * n)(*[i.data_ptr() for _, _, i in entries]),
                                        (P * n)(*[o.data_ptr() for o in outs]), n, _stream(stream)), "matvec_list_q8k")
    return outs


def matvec_scratch(base, m, xs, out=None, r0=0, r1=None, scratch=None, stream=None):
    """matvec for either layout, Q8_K images in caller scratch (a uint8 CUDA
    tensor of at least sg_matvec_scratch_bytes bytes; allocated if None)."""
    single = xs.dim() == 1
    xs2 = xs.reshape(1, -1) if single else xs
    if xs2.dtype != torch.float32 or xs2.stride(-1) != 1:
        raise ValueError("xs must be float32 with contiguous rows")
    r1 = m.rows if r1 is None else r1
    if out is None:
        out = torch.empty((xs2.shape[0], m.rows), dtype=torch.float32, device=xs2.device)
    out2 = out.reshape(1, -1) if out.dim() == 1 else out
    need = lib().sg_matvec_scratch_bytes(m.cols, xs2.shape[0])
    if scratch is None:
        scratch = torch.empty(need, dtype=torch.uint8, device=xs2.device)
    _lib.check(lib().sg_matvec_scratch(C.c_void_p(base.data_ptr()), C.byref(m.c()), C.c_void_p(xs2.data_ptr()),
                                       xs2.stride(0), C.c_void_p(out2.data_ptr()), out2.stride(0), xs2.shape[0], r0,
                                       r1, C.c_void_p(scratch.data_ptr()), scratch.numel(), _stream(stream)),
               "matvec_scratch")
    return out


def _float_call(fn, what, base, m, xs, out, r0, r1, stream):
    single = xs.dim() == 1
    xs2 = xs.reshape(1, -1) if single else xs
    if xs2.dtype != torch.float32 or xs2.stride(-1) != 1:
        raise ValueError("xs must be float32 with contiguous rows")
    r1 = m.rows if r1 is None else r1
    if out is None:
        out = torch.full((xs2.shape[0], m.rows), float("nan"), dtype=torch.float32, device=xs2.device)
    out2 = out.reshape(1, -1) if out.dim() == 1 else out
    _lib.check(fn(C.c_void_p(base.data_ptr()), C.byref(m.c()), C.c_void_p(xs2.data_ptr()), xs2.stride(0),
                  C.c_void_p(out2.data_ptr()), out2.stride(0), xs2.shape[0], r0, r1, _stream(stream)), what)
    return out


def matvec_rows_float(base, m, xs, out=None, r0=0, r1=None, stream=None):
    """quant::matvec_rows_avx2 (quant.rs:939-1094) for every vector: fp32 CUDA
    xs [n_vec, cols] (or [cols]) -> out [n_vec, rows] (rows outside r0..r1
    untouched).  GGUF rows of F32, F16, Q8_0, Q4_K or Q6_K."""
    return _float_call(lib().sg_matvec_rows_float, "matvec_rows_float", base, m, xs, out, r0, r1, stream)


def matmul_batch(base, m, xs, out=None, r0=0, r1=None, stream=None):
    """matvec_multi (smollm_chat.rs:447-512) for up to 128 vectors in one pass
    over a TILED16 Q4_K / Q6_K matrix: fp32 CUDA xs [n_vec, cols] -> out
    [n_vec, rows] (rows outside r0..r1 untouched), bit for bit the GEMV's."""
    xs2 = xs.reshape(1, -1) if xs.dim() == 1 else xs
    if xs2.dtype != torch.float32 or xs2.stride(-1) != 1:
        raise ValueError("xs must be float32 with contiguous rows")
    r1 = m.rows if r1 is None else r1
    if out is None:
        out = torch.full((xs2.shape[0], m.rows), float("nan"), dtype=torch.float32, device=xs2.device)
    out2 = out.reshape(1, -1) if out.dim() == 1 else out
    L = lib()
    nbytes = L.sg_matmul_batch_scratch_bytes(C.byref(m.c()), xs2.shape[0])
    if not nbytes:
        raise SgError(3, "matmul_batch_scratch_bytes")
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=xs2.device)
    _lib.check(L.sg_matmul_batch(C.c_void_p(base.data_ptr()), C.byref(m.c()), C.c_void_p(xs2.data_ptr()),
                                 xs2.stride(0), C.c_void_p(out2.data_ptr()), out2.stride(0), xs2.shape[0], r0, r1,
                                 C.c_void_p(scratch.data_ptr()), nbytes, _stream(stream)), "matmul_batch")
    return out


def matmul_rows_float(base, m, xs, out=None, r0=0, r1=None, stream=None):
    """quant_multi::matmul_rows_avx2 (quant_multi.rs:232-273): the shared-decode
    rows_multi kernels for several vectors, matvec_rows for one."""
    return _float_call(lib().sg_matmul_rows_float, "matmul_rows_float", base, m, xs, out, r0, r1, stream)


def gemv(base, m, xq, stream=None):
    """All rows for a list of Q8K vectors -> float32 CUDA [n_vec, rows]."""
    out = torch.empty((len(xq), m.rows), dtype=torch.float32, device=base.device)
    matmul_rows(base, m, xq, [out[b] for b in range(len(xq))], 0, m.rows, stream)
    return out


def block_sums(base, m, q, r0, r1, stream=None):
    """int32 [r1-r0, nb, 8] lane sums of quant_q8k.rs:235-242, as the kernel computes them."""
    out = torch.empty((r1 - r0, m.cols // QK, 8), dtype=torch.int32, device=base.device)
    _lib.check(lib().sg_block_sums(C.c_void_p(base.data_ptr()), C.byref(m.c()), C.byref(q.desc),
                                   C.c_void_p(out.data_ptr()), r0, r1, _stream(stream)), "block_sums")
    return out


def quantize_weights(dtype, w, stream=None):
    """f32 [rows, cols] CUDA -> uint8 CUDA bytes of Q4_K / Q6_K rows (own quantizer)."""
    w = w.contiguous()
    rows, cols = w.shape
    out = torch.empty(rows * row_bytes(dtype, cols), dtype=torch.uint8, device=w.device)
    _lib.check(lib().sg_quantize_weights(dtype, C.c_void_p(w.data_ptr()), rows, cols, C.c_void_p(out.data_ptr()),
                                         _stream(stream)), "quantize_weights")
    return out


def tiled16_bytes(dtype, rows, cols):
    out = C.c_uint64()
    _lib.check(lib().sg_tiled16_bytes(dtype, rows, cols, C.byref(out)), "tiled16_bytes")
    return out.value


def repack_tiled16(dtype, w, rows, cols, stream=None):
    """GGUF-row bytes (uint8 CUDA) -> TILED16 bytes; returns (buffer, Mat)."""
    out = torch.empty(tiled16_bytes(dtype, rows, cols), dtype=torch.uint8, device=w.device)
    _lib.check(lib().sg_repack_tiled16(dtype, C.c_void_p(w.data_ptr()), rows, cols, C.c_void_p(out.data_ptr()),
                                       _stream(stream)), "repack_tiled16")
    return out, Mat(dtype, cols, rows, layout=TILED16)


def unpack_tiled16(dtype, t, rows, cols, stream=None):
    """TILED16 bytes -> GGUF-row bytes (uint8 CUDA)."""
    out = torch.empty(rows * row_bytes(dtype, cols), dtype=torch.uint8, device=t.device)
    _lib.check(lib().sg_unpack_tiled16(dtype, C.c_void_p(t.data_ptr()), rows, cols, C.c_void_p(out.data_ptr()),
                                       _stream(stream)), "unpack_tiled16")
    return out


def device_status():
    """Raises SgError if a bounded device wait gave up since the last check."""
    _lib.check(lib().sg_device_status(), "device status")


# ---- MoE layer (smollm_chat.rs:1178-1382 moe_forward, with ffns_fused :382-442)

MOE_MAX_USED = _lib.MOE_MAX_USED


class Moe:
    """Device weights of one MoE layer (smollm_chat.rs:152-167 `Moe`).

    Built by `Moe.pack` from the GGUF expert tensors (uint8 CUDA buffers of
    GGUF rows: ffn_gate_exps / ffn_up_exps [n_expert][n_ff][dim], ffn_down_exps
    [n_expert][dim][n_ff]) and the F32 router [n_expert][dim].  The tensors the
    layer holds stay referenced by this object for as long as it lives."""

    def __init__(self, **kw):
        self.__dict__.update(kw)

    @classmethod
    def pack(cls, router, gate_exps, up_exps, down_exps, gate_up_dtype, down_dtype, n_expert, n_used, dim, n_ff,
             norm=True, moe_prune=0.0, shared=None, shared_gate=None, stream=None):
        """shared: optional (gate, up, down, gate_up_dtype, down_dtype, n_ff) of GGUF
        rows (one expert); shared_gate: optional F32 [dim] CUDA tensor."""
        dev = router.device
        gu_stride = tiled16_bytes(gate_up_dtype, 2 * n_ff, dim)
        dn_stride = tiled16_bytes(down_dtype, dim, n_ff)
        gu = torch.empty(gu_stride * n_expert, dtype=torch.uint8, device=dev)
        dn = torch.empty(dn_stride * n_expert, dtype=torch.uint8, device=dev)
        s = _stream(stream)
        _lib.check(lib().sg_moe_pack_gate_up(gate_up_dtype, C.c_void_p(gate_exps.data_ptr()),
                                             C.c_void_p(up_exps.data_ptr()), n_expert, n_ff, dim,
                                             C.c_void_p(gu.data_ptr()), s), "moe_pack_gate_up")
        _lib.check(lib().sg_moe_pack_down(down_dtype, C.c_void_p(down_exps.data_ptr()), n_expert, dim, n_ff,
                                          C.c_void_p(dn.data_ptr()), s), "moe_pack_down")
        m = cls(router=router.contiguous(), gate_up=gu, down=dn, gate_up_dtype=gate_up_dtype,
                down_dtype=down_dtype, gate_up_stride=gu_stride, down_stride=dn_stride, dim=dim, n_ff=n_ff,
                n_expert=n_expert, n_used=n_used, norm=bool(norm), moe_prune=float(moe_prune),
                shared_gate_up=None, shared_down=None, shared_gate_up_dtype=0, shared_down_dtype=0,
                shared_n_ff=0, shared_gate=None)
        if shared is not None:
            sg_, su, sd, sgu_dt, sd_dt, sh_ff = shared
            sgu = torch.empty(tiled16_bytes(sgu_dt, 2 * sh_ff, dim), dtype=torch.uint8, device=dev)
            sdn = torch.empty(tiled16_bytes(sd_dt, dim, sh_ff), dtype=torch.uint8, device=dev)
            _lib.check(lib().sg_moe_pack_gate_up(sgu_dt, C.c_void_p(sg_.data_ptr()), C.c_void_p(su.data_ptr()), 1,
                                                 sh_ff, dim, C.c_void_p(sgu.data_ptr()), s), "moe_pack_gate_up")
            _lib.check(lib().sg_moe_pack_down(sd_dt, C.c_void_p(sd.data_ptr()), 1, dim, sh_ff,
                                              C.c_void_p(sdn.data_ptr()), s), "moe_pack_down")
            m.shared_gate_up, m.shared_down = sgu, sdn
            m.shared_gate_up_dtype, m.shared_down_dtype, m.shared_n_ff = sgu_dt, sd_dt, sh_ff
            m.shared_gate = None if shared_gate is None else shared_gate.contiguous()
        return m

    def c(self):
        ptr = lambda t: None if t is None else t.data_ptr()
        return _lib.SgMoe(ptr(self.router), ptr(self.gate_up), ptr(self.down), self.gate_up_dtype, self.down_dtype,
                          self.gate_up_stride, self.down_stride, self.dim, self.n_ff, self.n_expert, self.n_used,
                          int(self.norm), self.moe_prune, ptr(self.shared_gate_up), ptr(self.shared_down),
                          self.shared_gate_up_dtype, self.shared_down_dtype, self.shared_n_ff,
                          ptr(self.shared_gate))

    def scratch_bytes(self):
        n = lib().sg_moe_scratch_bytes(C.byref(self.c()))
        if not n:
            raise SgError(1, "moe_scratch_bytes")
        return n


def moe_forward(m, x, out=None, scratch=None, choice=None, probs=None, stream=None):
    """out[dim] = moe_forward(x[dim]) (smollm_chat.rs:1178).  choice: optional
    int32 CUDA tensor of 36 words receiving sg_moe_choice (n, pad, id[16],
    weight bits[16]); probs: optional float32 [n_expert] for the softmax."""
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be contiguous float32")
    if out is None:
        out = torch.empty(m.dim, dtype=torch.float32, device=x.device)
    if scratch is None:
        scratch = torch.empty(m.scratch_bytes(), dtype=torch.uint8, device=x.device)
    ptr = lambda t: None if t is None else C.c_void_p(t.data_ptr())
    _lib.check(lib().sg_moe_forward(C.byref(m.c()), ptr(x), ptr(out), ptr(scratch), scratch.numel(), ptr(choice),
                                    ptr(probs), _stream(stream)), "moe_forward")
    return out


def moe_forward_batch(m, xs, out=None, scratch=None, choices=None, stream=None):
    """moe_forward_batch (smollm_chat.rs:928-1174): out[t] = moe_forward(xs[t])
    for xs float32 CUDA [n_tok, dim], bit for bit the one-token results.
    choices: optional int32 CUDA [n_tok, 36] receiving each token's choice."""
    if xs.dtype != torch.float32 or xs.dim() != 2 or xs.stride(-1) != 1:
        raise ValueError("xs must be float32 [n_tok, dim] with contiguous rows")
    n_tok = xs.shape[0]
    if out is None:
        out = torch.empty(n_tok, m.dim, dtype=torch.float32, device=xs.device)
    if scratch is None:
        n = lib().sg_moe_batch_scratch_bytes(C.byref(m.c()), n_tok)
        if not n:
            raise SgError(1, "moe_batch_scratch_bytes")
        scratch = torch.empty(n, dtype=torch.uint8, device=xs.device)
    ptr = lambda t: None if t is None else C.c_void_p(t.data_ptr())
    _lib.check(lib().sg_moe_forward_batch(C.byref(m.c()), ptr(xs), xs.stride(0), n_tok, ptr(out), out.stride(0),
                                          ptr(scratch), scratch.numel(), ptr(choices), _stream(stream)),
               "moe_forward_batch")
    return out


def decode_choice(choice):
    """(ids, weights) of the kept experts from a choice tensor filled by moe_forward."""
    c = choice.cpu()
    n = int(c[0])
    ids = [int(v) for v in c[4:4 + n]]
    w = c[4 + MOE_MAX_USED:4 + MOE_MAX_USED + n].view(torch.float32).tolist()
    return ids, w
