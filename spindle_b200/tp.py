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
