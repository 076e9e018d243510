"""Expert parallelism of the batched MoE layer (sg_moe_forward_batch_ep):
each rank keeps a slice of the experts, the slot outputs travel to every rank
over NVLink peer stores, and every rank's output equals the whole layer on
one GPU bit for bit.  One rank runs on any GPU box; two ranks need two GPUs."""
import os
import socket
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import tp_util  # noqa: E402

from spindle_b200.tp import TpGroup  # noqa: E402

pytestmark = pytest.mark.gpu


def test_ep_one_rank(dev):
    grp = TpGroup(device=dev)
    try:
        assert tp_util.ep_check(dev, grp, None) == []
    finally:
        grp.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_ranks(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=tp_util.ep_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=900)
        res.setdefault(r, []).append(msg)
    for p in procs:
        p.join(timeout=120)
    assert res == {r: ["ok"] for r in range(world)}, res


def test_decoder_ep_one_rank(dev):
    # a group of one: every expert is local, sg_forward_ep == sg_forward bit for bit
    import numpy as np
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import decoder_util as U
    from spindle_b200.decoder import Decoder
    grp = TpGroup(device=dev)
    try:
        cfg = dict(U.MOE, n_layers=2, max_seq=32)
        dtypes = U.dtypes_for(cfg)
        W = U.device_weights(U.host_weights(cfg, dtypes, seed=71), dev)
        full, epd = Decoder(cfg, W, dtypes, dev), Decoder(cfg, W, dtypes, dev, ep=grp)
        for pos, t in enumerate([5, 77, 130, 9, 400, 11]):
            full.set_state(t, pos)
            full.step()
            epd.set_state(t, pos)
            epd.step()
            torch.cuda.synchronize()
            assert np.array_equal(full.logits.cpu().numpy().view(np.uint32), epd.logits.cpu().numpy().view(np.uint32))
            assert torch.equal(full.state, epd.state)
        with pytest.raises(ValueError):
            epd.forward_batch([1, 2], 6)
        del full, epd
    finally:
        grp.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decoder_ep_ranks(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=tp_util.decoder_ep_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=900)
        res.setdefault(r, []).append(msg)
    for p in procs:
        p.join(timeout=120)
    assert res == {r: ["ok"] for r in range(world)}, res
