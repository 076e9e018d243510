"""The layer split over two GPUs (sg_forward_batch_range + sg_pipe_send /
sg_pipe_recv): stage 0 runs the first half of the layers on each prompt
chunk and sends the raw residual over NVLink, stage 1 runs the rest and the
head; its logits and greedy tokens equal the whole model's on one GPU bit
for bit.  One GPU checks the stages back to back on the same device."""
import os
import socket
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import decoder_util as U  # noqa: E402
import tp_util  # noqa: E402

from spindle_b200.decoder import Decoder  # noqa: E402
from spindle_b200.tp import TpGroup  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_stages_on_one_gpu(dev, kind):
    cfg = dict(U.DENSE if kind == "dense" else U.MOE, n_layers=4, max_seq=128)
    dtypes = U.dtypes_for(cfg)
    W = U.device_weights(U.host_weights(cfg, dtypes, seed=62), dev)
    a, b, whole = Decoder(cfg, W, dtypes, dev), Decoder(cfg, W, dtypes, dev), Decoder(cfg, W, dtypes, dev)
    toks = np.random.default_rng(4).integers(0, cfg["vocab"], 30).tolist()
    pos = 0
    for c in [1, 9, 20]:
        (h,) = a.forward_batch_range(pos, 0, 1, tokens=toks[pos:pos + c])
        (h2,) = a.forward_batch_range(pos, 1, 3, hidden=h)
        lg, gr = b.forward_batch_range(pos, 3, 4, hidden=h2)
        wl, wg = whole.forward_batch(toks[pos:pos + c], pos)
        torch.cuda.synchronize()
        assert np.array_equal(lg.cpu().numpy().view(np.uint32), wl.cpu().numpy().view(np.uint32)), pos
        assert torch.equal(gr, wg)
        pos += c


@pytest.mark.parametrize("world", [2, 4, 8])
def test_pipeline_ranks(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=tp_util.pipe_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=900)
        res.setdefault(r, []).append(msg)
    for p in procs:
        p.join(timeout=120)
    assert res == {r: ["ok"] for r in range(world)}, res


def test_pipeline_kv_shift_one_stage(dev):
    # a pipeline of one stage (all layers): the KV window slides as on the
    # plain decoder, logits bit for bit through several shifts
    import decoder_util as U
    from spindle_b200.decoder import Decoder
    from spindle_b200.tp import PipelineStage
    grp = TpGroup(device=dev)
    try:
        cfg = dict(U.MOE, n_layers=2, max_seq=40)
        dtypes = U.dtypes_for(cfg)
        W = U.device_weights(U.host_weights(cfg, dtypes, seed=63), dev)
        stage = PipelineStage(Decoder(cfg, W, dtypes, dev), grp, n_max=8)
        assert stage.max_seq == 40
        bad, shifts = tp_util.pipe_shift_loop(stage, Decoder(cfg, W, dtypes, dev), 3, 100, dev)
        assert not bad and shifts >= 3, (bad, shifts)
        with pytest.raises(ValueError):
            stage.forward([1], 40)
    finally:
        grp.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_pipeline_kv_shift_ranks(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=tp_util.pipe_kv_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=900)
        res.setdefault(r, []).append(msg)
    for p in procs:
        p.join(timeout=120)
    assert res == {r: ["ok"] for r in range(world)}, res
