"""sg_matvec_tp, the row-split GEMV with the gather fused in (peer stores over
NVLink): the gathered output equals the whole-matrix sg_matvec bit for bit,
over repeated calls and CUDA-graph replays.  One rank runs on any GPU box;
two ranks (two processes, NCCL for the set-up only) need two GPUs."""
import os
import socket
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import tp_util  # noqa: E402

import spindle_b200 as sg  # noqa: E402
from spindle_b200.tp import ShardedMatrix, TpGroup, matvec_tp  # noqa: E402

pytestmark = pytest.mark.gpu


def bits(t):
    return t.cpu().numpy().view(np.uint32)


def test_tp_one_rank(dev):
    grp = TpGroup(device=dev)
    try:
        g = torch.Generator(device=dev).manual_seed(5)
        for dt, rows, cols in tp_util.SHAPES:
            w = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=g) * 0.02)
            full, mf = sg.repack_tiled16(dt, w, rows, cols)
            shard = ShardedMatrix(dt, w, rows, cols, 1, 0)
            for nv in [1, 2, 8]:
                buf = grp.buffer(nv, rows)
                for _ in range(3):
                    xs = torch.randn(nv, cols, device=dev, generator=g)
                    got = matvec_tp(shard, xs, grp, buf)
                    assert np.array_equal(bits(got), bits(sg.matvec(full, mf, xs))), (dt, rows, nv)
        xs = torch.randn(1, 4096, device=dev, generator=g)
        w = sg.quantize_weights(sg.Q4_K, torch.randn(4096, 4096, device=dev, generator=g) * 0.02)
        full, mf = sg.repack_tiled16(sg.Q4_K, w, 4096, 4096)
        shard = ShardedMatrix(sg.Q4_K, w, 4096, 4096, 1, 0)
        buf = grp.buffer(1, 4096)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                matvec_tp(shard, xs, grp, buf, stream=s)
            want = sg.matvec(full, mf, xs, stream=s)
            for _ in range(5):
                buf.tensor.fill_(float("nan"))
                graph.replay()
                torch.cuda.synchronize()
                assert np.array_equal(bits(buf.tensor), bits(want))
        torch.cuda.current_stream().wait_stream(s)
        del graph
        sg.device_status()
    finally:
        grp.close()


def test_tp_bad_args(dev):
    import ctypes as C
    grp = TpGroup(device=dev)
    try:
        w = sg.quantize_weights(sg.Q4_K, torch.randn(64, 256, device=dev) * 0.02)
        shard = ShardedMatrix(sg.Q4_K, w, 64, 256, 1, 0)
        buf = grp.buffer(1, 64)
        x = torch.randn(256, device=dev)
        lib = sg.lib()

        def call(m, wptr, row0, rows, g):
            return lib.sg_matvec_tp(C.c_void_p(wptr), C.byref(m.c()), C.c_void_p(x.data_ptr()), 256, 1, row0, rows,
                                    C.c_void_p(buf.tensor.data_ptr()), 64, C.byref(g), None)

        g = grp.c(buf)
        g.rank = 1  # outside the group
        assert call(shard.m, shard.w.data_ptr(), 0, 64, g) == 1
        g = grp.c(buf)
        assert call(shard.m, shard.w.data_ptr(), 8, 64, g) == 1  # rows past the whole matrix
        assert call(sg.Mat(sg.Q4_K, 256, 64), w.data_ptr(), 0, 64, g) == 1  # GGUF layout
        g.comm = None
        assert call(shard.m, shard.w.data_ptr(), 0, 64, g) == 1
        sg.device_status()
    finally:
        grp.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_ranks(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=tp_util.gpu_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=900)
        res.setdefault(r, []).append(msg)
    for p in procs:
        p.join(timeout=120)
    assert res == {r: ["ok"] for r in range(world)}, res
