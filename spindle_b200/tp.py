"""Row-split tensor parallelism over NVLink: sg_matvec_tp and its set-up.

One process per GPU.  par_rows (smollm_chat.rs:332-337) splits a matvec's rows
[0, R) across worker threads as [R*t/T, R*(t+1)/T); here rank p of P owns that
slice of every matrix, and the GEMV kernel stores each row of its slice
straight into the output buffer of every rank (CUDA IPC mappings, NVLink peer
stores), so that after the call every rank holds the whole output: the matvec
and the all-gather that follows it are one kernel.  Rows travel as 8-byte (epoch, value) pairs, so the receiving
blocks know a row has arrived without any memory fence.

Receive buffers that other ranks write into are plain cudaMalloc allocations
(IPC handles name whole allocations), made by the library (sg_alloc).
"""
import ctypes as C

import torch

from . import _lib, lib, _stream, repack_tiled16, row_bytes
from ._lib import SgTpGroup, TP_MAX_RANKS


def shard_rows(rows, n_ranks, rank):
    """par_rows's split (smollm_chat.rs:334): rank p owns rows [R*p/P, R*(p+1)/P)."""
    return rows * rank // n_ranks, rows * (rank + 1) // n_ranks


def _dist_on():
    import torch.distributed as dist
    return dist.is_available() and dist.is_initialized()


def exchange(obj, group=None):
    """Every rank's obj, in rank order (an all-gather over the process group;
    a group of one without torch.distributed)."""
    import torch.distributed as dist
    if not _dist_on():
        return [obj]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


class _DeviceArray:
    """A raw device allocation as seen by torch.as_tensor (no copy)."""

    def __init__(self, ptr, shape, device):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}
        self.device = device


class TpBuffer:
    """One row-split output: .tensor [n_vec, rows] is this rank's plain copy
    (every rank gets the whole output); .recv[q] addresses rank q's receive
    buffer of epoch-tagged rows."""

    def __init__(self, tensor, recv, n_vec, rows):
        self.tensor, self.recv, self.n_vec, self.rows = tensor, recv, n_vec, rows


class TpGroup:
    """This rank's comm block and the shared receive buffers made through it.
    Every rank constructs it and its buffers in the same order (each is a
    collective over the process group)."""

    def __init__(self, group=None, device=None):
        import torch.distributed as dist
        self.group = group
        self.rank, self.n = (dist.get_rank(group), dist.get_world_size(group)) if _dist_on() else (0, 1)
        if self.n > TP_MAX_RANKS:
            raise ValueError("at most %d ranks" % TP_MAX_RANKS)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._own, self._opened = [], []
        self.comm = self._alloc(lib().sg_tp_comm_bytes())
        _lib.check(lib().sg_tp_comm_init(C.c_void_p(self.comm), None), "sg_tp_comm_init")
        torch.cuda.synchronize(self.device)

    def _alloc(self, nbytes):
        p = C.c_void_p()
        _lib.check(lib().sg_alloc(nbytes, C.byref(p)), "sg_alloc")
        self._own.append(p.value)
        return p.value

    def _share(self, ptr):
        n = lib().sg_ipc_handle_bytes()
        h = (C.c_ubyte * n)()
        _lib.check(lib().sg_ipc_get_handle(C.c_void_p(ptr), h), "sg_ipc_get_handle")
        handles = exchange(bytes(h), self.group)
        ptrs = []
        for q, hq in enumerate(handles):
            if q == self.rank:
                ptrs.append(ptr)
                continue
            p = C.c_void_p()
            _lib.check(lib().sg_ipc_open((C.c_ubyte * n).from_buffer_copy(hq), C.byref(p)), "sg_ipc_open")
            self._opened.append(p.value)
            ptrs.append(p.value)
        return ptrs

    def buffer(self, n_vec, rows):
        nbytes = lib().sg_tp_recv_bytes(n_vec, rows)
        ptr = self._alloc(nbytes)
        # epoch 0 never runs: a zeroed buffer holds no row of any call
        torch.as_tensor(_DeviceArray(ptr, (nbytes // 4,), self.device), device=self.device).zero_()
        torch.cuda.synchronize(self.device)
        out = torch.empty(n_vec, rows, dtype=torch.float32, device=self.device)
        return TpBuffer(out, self._share(ptr), n_vec, rows)

    def c(self, buf):
        g = SgTpGroup()
        g.n_ranks, g.rank = self.n, self.rank
        for q in range(self.n):
            g.recv[q] = buf.recv[q]
        g.comm = self.comm
        return g

    def close(self):
        """Unmaps the other ranks' memory, waits for every rank to do the same,
        then frees this rank's."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            _lib.check(lib().sg_ipc_close(C.c_void_p(p)), "sg_ipc_close")
        self._opened = []
        if _dist_on():
            dist.barrier(group=self.group)
        for p in self._own:
            _lib.check(lib().sg_free(C.c_void_p(p)), "sg_free")
        self._own = []


class ShardedMatrix:
    """This rank's row shard of a GGUF-row matrix, repacked to TILED16."""

    def __init__(self, dtype, w_full, rows, cols, n_ranks, rank):
        self.r0, self.r1 = shard_rows(rows, n_ranks, rank)
        rb = row_bytes(dtype, cols)
        part = w_full[self.r0 * rb:self.r1 * rb]
        self.w, self.m = repack_tiled16(dtype, part, self.r1 - self.r0, cols)
        self.rows, self.cols = rows, cols


def matvec_tp(shard, xs, grp, buf, stream=None):
    """buf.tensor[b, r] = (W x_b)[r] for every row r of the full matrix, on
    every rank; xs fp32 CUDA [n_vec, cols] (or [cols]), the same on all ranks."""
    xs2 = xs.reshape(1, -1) if xs.dim() == 1 else xs
    if xs2.dtype != torch.float32 or xs2.stride(-1) != 1:
        raise ValueError("xs must be float32 with contiguous rows")
    g = grp.c(buf)
    out = buf.tensor
    _lib.check(lib().sg_matvec_tp(C.c_void_p(shard.w.data_ptr()), C.byref(shard.m.c()), C.c_void_p(xs2.data_ptr()),
                                  xs2.stride(0), xs2.shape[0], shard.r0, buf.rows, C.c_void_p(out.data_ptr()),
                                  out.stride(0), C.byref(g), _stream(stream)), "sg_matvec_tp")
    return out


def gather_layout(rows, n_ranks):
    """Where every rank's shard outputs sit in a row-split list's all-gather
    (matvec_list_tp): each rank's block holds matrix j's shard rows at
    offset off[j], with room for the largest shard of j over the ranks, so
    that all blocks have the same size, chunk floats (a multiple of 64).
    rows: the matrices' full row counts.  Returns (off, chunk)."""
    maxrows = [max(b - a for a, b in (shard_rows(r, n_ranks, q) for q in range(n_ranks))) for r in rows]
    off = [sum(maxrows[:j]) for j in range(len(rows))]
    return off, -(-sum(maxrows) // 64) * 64


def split_gathered(gathered, rows, n_ranks, off, chunk):
    """Matrix j's whole output, rows in order, from the all-gathered blocks
    of a row-split list (rank q's block at q * chunk): one tensor per matrix."""
    outs = []
    for j, r in enumerate(rows):
        parts = []
        for q in range(n_ranks):
            a, b = shard_rows(r, n_ranks, q)
            parts.append(gathered[q * chunk + off[j]:q * chunk + off[j] + (b - a)])
        outs.append(torch.cat(parts))
    return outs


class ListTp:
    """A row-split list of independent matvecs: this rank's shards
    (ShardedMatrix, up to SG_LIST_MAX of them), one local block of their
    outputs and the buffer the blocks are all-gathered into (layout of
    gather_layout)."""

    def __init__(self, shards, n_ranks, device):
        self.shards, self.n_ranks = list(shards), n_ranks
        self.rows = [sh.rows for sh in self.shards]
        self.off, self.chunk = gather_layout(self.rows, n_ranks)
        self.local = torch.zeros(self.chunk, dtype=torch.float32, device=device)
        self.gathered = torch.empty(n_ranks * self.chunk, dtype=torch.float32, device=device)
        self.outs = [self.local[o:o + sh.r1 - sh.r0] for o, sh in zip(self.off, self.shards)]

    def gather(self, group=None):
        """The NCCL all-gather of the ranks' blocks (on torch's current stream)."""
        import torch.distributed as dist
        if _dist_on():
            dist.all_gather_into_tensor(self.gathered, self.local, group=group)
        else:
            self.gathered.copy_(self.local)

    def outputs(self):
        """Every matrix's whole output (copies taken from the gathered buffer)."""
        return split_gathered(self.gathered, self.rows, self.n_ranks, self.off, self.chunk)


def matvec_list_tp(lt, imgs, group=None, stream=None, gather=True):
    """Row-split matvecs of a list on every rank: sg_matvec_list_q8k over this
    rank's shards (imgs: the vectors' Q8_K images, sg.q8k_images, the same on
    every rank) into lt.local, then (gather=True) one all-gather of the
    blocks: afterwards lt.gathered holds every matrix's whole output on every
    rank (lt.outputs() for them in row order).  The rows are bit for bit
    those of matvec_tp and of one-GPU sg_matvec."""
    from . import matvec_list_q8k
    matvec_list_q8k([(sh.w, sh.m, im) for sh, im in zip(lt.shards, imgs)], lt.outs, stream=stream)
    if gather:
        if stream is None:
            lt.gather(group)
        else:
            with torch.cuda.stream(stream):
                lt.gather(group)
    return lt.gathered


class EpMoe:
    """This rank's part of an expert-parallel MoE layer (sg_moe_forward_batch_ep).

    Rank p of P keeps experts [E*p/P, E*(p+1)/P) (par_rows's split over the
    experts) and the whole router; every rank computes every token's choice,
    runs the slots of its own experts, and their outputs reach every rank's
    receive buffer over NVLink, where each rank's combine sums them in router
    order: each rank ends with the whole layer output, bit for bit the one-GPU
    result.  Build it on every rank, in the same order as the group's other
    buffers (its set-up is collective)."""

    def __init__(self, grp, router, gate_exps, up_exps, down_exps, gate_up_dtype, down_dtype, n_expert, n_used, dim,
                 n_ff, n_tok_max=16, norm=True, moe_prune=0.0):
        from . import Moe
        self.grp, self.n_tok_max = grp, n_tok_max
        self.lo, self.hi = shard_rows(n_expert, grp.n, grp.rank)
        rg, rd = row_bytes(gate_up_dtype, dim), row_bytes(down_dtype, n_ff)
        sl = lambda t, rb, rows: t[self.lo * rows * rb:self.hi * rows * rb]
        n_loc = self.hi - self.lo
        self.moe = Moe.pack(router, sl(gate_exps, rg, n_ff), sl(up_exps, rg, n_ff), sl(down_exps, rd, dim),
                            gate_up_dtype, down_dtype, max(n_loc, 1), n_used, dim, n_ff, norm=norm,
                            moe_prune=moe_prune) if n_loc else None
        if self.moe is None:  # a rank without experts still takes part
            self.moe = Moe.pack(router, gate_exps[:rg * n_ff], up_exps[:rg * n_ff], down_exps[:rd * dim],
                                gate_up_dtype, down_dtype, 1, n_used, dim, n_ff, norm=norm, moe_prune=moe_prune)
        self.moe.n_expert = n_expert  # the router and the choice span every expert
        self.comm = grp._alloc(lib().sg_tp_comm_bytes())
        _lib.check(lib().sg_tp_comm_init(C.c_void_p(self.comm), None), "sg_tp_comm_init")
        nbytes = lib().sg_moe_ep_recv_bytes(C.byref(self.moe.c()), n_tok_max)
        if not nbytes:
            raise ValueError("sg_moe_ep_recv_bytes: unsupported layer or batch")
        recv = grp._alloc(nbytes)
        torch.as_tensor(_DeviceArray(recv, (nbytes // 4,), grp.device), device=grp.device).zero_()
        torch.cuda.synchronize(grp.device)
        self.recv = grp._share(recv)
        self._scratch = {}

    def c(self):
        from ._lib import SgMoeEp
        e = SgMoeEp()
        e.n_ranks, e.rank = self.grp.n, self.grp.rank
        e.expert_lo, e.expert_hi = self.lo, self.hi
        e.recv_slots = self.n_tok_max * self.moe.n_used
        for q in range(self.grp.n):
            e.recv[q] = self.recv[q]
        e.comm = self.comm
        return e

    def forward(self, xs, out=None, stream=None):
        """out[t] = the layer on xs[t] (float32 CUDA [n_tok, dim]), on every rank."""
        n_tok = xs.shape[0]
        if out is None:
            out = torch.empty(n_tok, self.moe.dim, dtype=torch.float32, device=xs.device)
        sc = self._scratch.get(n_tok)
        if sc is None:
            nb = lib().sg_moe_batch_scratch_bytes(C.byref(self.moe.c()), n_tok)
            sc = self._scratch[n_tok] = torch.empty(nb, dtype=torch.uint8, device=xs.device)
        m, e = self.moe.c(), self.c()
        _lib.check(lib().sg_moe_forward_batch_ep(C.byref(m), C.byref(e), C.c_void_p(xs.data_ptr()), xs.stride(0),
                                                 n_tok, C.c_void_p(out.data_ptr()), out.stride(0),
                                                 C.c_void_p(sc.data_ptr()), sc.numel(), None, _stream(stream)),
                   "sg_moe_forward_batch_ep")
        return out


class PipeLink:
    """A one-way link src -> dst for up to n_max floats per call: the residual
    between pipeline stages (sg_pipe_send / sg_pipe_recv).  Every rank of the
    group builds it (the set-up is collective); only src sends, only dst
    receives, each call of one matched by a call of the other."""

    def __init__(self, grp, src, dst, n_max):
        self.grp, self.src, self.dst, self.n_max = grp, src, dst, n_max
        self.comm = grp._alloc(lib().sg_tp_comm_bytes())
        _lib.check(lib().sg_tp_comm_init(C.c_void_p(self.comm), None), "sg_tp_comm_init")
        nbytes = lib().sg_pipe_recv_bytes(n_max)
        recv = grp._alloc(nbytes)
        torch.as_tensor(_DeviceArray(recv, (nbytes // 4,), grp.device), device=grp.device).zero_()
        torch.cuda.synchronize(grp.device)
        self.comms = grp._share(self.comm)
        self.recvs = grp._share(recv)

    def send(self, x, stream=None):
        x = x.contiguous()
        _lib.check(lib().sg_pipe_send(C.c_void_p(x.data_ptr()), x.numel(), self.n_max,
                                      C.c_void_p(self.recvs[self.dst]), C.c_void_p(self.comm), _stream(stream)),
                   "sg_pipe_send")

    def recv(self, out, stream=None):
        _lib.check(lib().sg_pipe_recv(C.c_void_p(out.data_ptr()), out.numel(), self.n_max,
                                      C.c_void_p(self.recvs[self.dst]), C.c_void_p(self.comm),
                                      C.c_void_p(self.comms[self.src]), _stream(stream)), "sg_pipe_recv")
        return out


class PipelineStage:
    """One rank's stage of a layer split over the ranks of a group: the two-PC
    mode of cluster_net.rs (layers 0..split on one machine, the rest and the
    head on the other) as a chain of GPUs.  Stage p runs layers [L*p/P,
    L*(p+1)/P) of its Decoder (par_rows's split over the layers), receives the
    residual from stage p-1 and sends it to stage p+1 over NVLink (PipeLink:
    the STEP / PREFILL frames' activations).  The last stage holds the head and
    owns the sliding window, as the reference's master does:

      kv_info()        FRAME_KV_INFO: every stage's KV capacity; the pipeline's
                       context is the smallest (attach_cluster clamps the
                       master's max_seq to the worker's).
      ensure_kv_room() ensure_kv_room on the last stage, then FRAME_KV_SHIFT:
                       (n_keep, n_discard, cur_pos) reach every stage, each
                       shifts its own layers' caches (shift_kv), so all stages
                       keep identical positions.

    Every rank builds its stage in the same order (the set-up is collective)
    and calls forward / ensure_kv_room with the same arguments."""

    def __init__(self, decoder, grp, n_max=64):
        self.dec, self.grp, self.n_max = decoder, grp, n_max
        self.rank, self.n = grp.rank, grp.n
        self.l0, self.l1 = shard_rows(decoder.cfg["n_layers"], self.n, self.rank)
        dim = decoder.cfg["dim"]
        self.links = [PipeLink(grp, p, p + 1, n_max * dim) for p in range(self.n - 1)]
        self.max_seq = self.kv_info()

    def kv_info(self):
        return min(exchange(int(self.dec.cfg["max_seq"]), self.grp.group))

    def _broadcast(self, obj):
        return exchange(obj, self.grp.group)[self.n - 1]  # the last stage's value

    def forward(self, tokens, pos0, stream=None):
        """The stage's layers for positions pos0 .. pos0 + len(tokens) - 1; the
        last stage returns (logits [n, vocab], greedy tokens), the others None."""
        n = len(tokens)
        if pos0 + n > self.max_seq:
            raise ValueError("positions past the pipeline's context: call ensure_kv_room first")
        dim = self.dec.cfg["dim"]
        if self.rank == 0:
            out = self.dec.forward_batch_range(pos0, self.l0, self.l1, tokens=tokens, n_max=self.n_max,
                                               stream=stream)
        else:
            h = self.links[self.rank - 1].recv(torch.empty(n, dim, device=self.dec.dev), stream=stream)
            out = self.dec.forward_batch_range(pos0, self.l0, self.l1, hidden=h, n_max=self.n_max, stream=stream)
        if self.rank < self.n - 1:
            self.links[self.rank].send(out[0], stream=stream)
            return None
        return out

    def ensure_kv_room(self, cur_pos, needed, n_keep, stream=None):
        """Room for `needed` more positions: the last stage decides as
        ensure_kv_room does (against the pipeline's context), every stage
        applies the same shift to its layers; returns the position to go on
        from (the same on every stage)."""
        if self.rank == self.n - 1:
            if cur_pos + needed <= self.max_seq:
                decision = (n_keep, 0, cur_pos)
            else:
                n_ctx = cur_pos - n_keep
                decision = (n_keep, min(max(cur_pos + needed - self.max_seq, n_ctx // 2), n_ctx), cur_pos)
        else:
            decision = None
        n_keep, n_discard, pos = self._broadcast(decision)
        if n_discard == 0:
            return pos
        return self.dec.shift_kv(n_keep, n_discard, pos, l0=self.l0, l1=self.l1, stream=stream)
