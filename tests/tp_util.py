"""Rank bodies for the multi-process tests of spindle_b200.tp (run under
torch.multiprocessing spawn; 127.0.0.1 rendezvous)."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def init(rank, world, port, backend):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = {}
    if backend == "nccl":
        import torch
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device("cuda", rank)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), **kw)


def cpu_rank(rank, world, port, out):
    # host logic only: the shard split, the rank-ordered exchange and the
    # row-split list's gather layout
    import torch.distributed as dist
    from spindle_b200.tp import exchange, shard_rows
    init(rank, world, port, "gloo")
    try:
        got = exchange(("rank", rank, b"\x01" * 64), None)
        assert got == [("rank", q, b"\x01" * 64) for q in range(world)]
        for rows in [1, 7, 16, 1000, 4096, 151936]:
            parts = exchange(shard_rows(rows, world, rank), None)
            assert parts[0][0] == 0 and parts[-1][1] == rows
            assert all(parts[q][1] == parts[q + 1][0] for q in range(world - 1))
        # the row-split list's gather layout: blocks of equal size, each
        # matrix's shard at its offset, reassembled in row order
        import torch
        from spindle_b200.tp import gather_layout, split_gathered
        rows = [1, 7, 16, 1000, 4096, 151936, 33]
        off, chunk = gather_layout(rows, world)
        assert chunk % 64 == 0 and chunk >= off[-1] + max(b - a for a, b in
                                                          (shard_rows(rows[-1], world, q) for q in range(world)))
        local = torch.full((chunk,), -1.0)
        for j, r in enumerate(rows):
            a, b = shard_rows(r, world, rank)
            local[off[j]:off[j] + b - a] = torch.arange(a, b, dtype=torch.float32) + 1e6 * j
        blocks = [torch.empty(chunk) for _ in range(world)]
        dist.all_gather(blocks, local)
        outs = split_gathered(torch.cat(blocks), rows, world, off, chunk)
        for j, r in enumerate(rows):
            assert torch.equal(outs[j], torch.arange(r, dtype=torch.float32) + 1e6 * j), j
        out.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        out.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


SHAPES = [(12, 4096, 4096), (14, 1000, 1024), (12, 14336, 2048), (14, 2048, 768 * 4)]


def gpu_rank(rank, world, port, out):
    # the fused row-split GEMV against the whole matrix on one GPU, bit for bit
    import numpy as np
    import torch
    import torch.distributed as dist
    import spindle_b200 as sg
    from spindle_b200.tp import ShardedMatrix, TpGroup, matvec_tp
    init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    grp = None
    try:
        grp = TpGroup(device=dev)
        g = torch.Generator(device=dev).manual_seed(3)
        for dt, rows, cols in SHAPES:
            w = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=g) * 0.02)
            full, mf = sg.repack_tiled16(dt, w, rows, cols)
            shard = ShardedMatrix(dt, w, rows, cols, world, rank)
            for nv in [1, 3]:
                buf = grp.buffer(nv, rows)
                for it in range(4):
                    xs = torch.randn(nv, cols, device=dev, generator=g)
                    got = matvec_tp(shard, xs, grp, buf)
                    want = sg.matvec(full, mf, xs)
                    torch.cuda.synchronize(dev)
                    ok = np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32))
                    dist.barrier()  # no rank writes the next call's rows while another still reads these
                    assert ok, (dt, rows, cols, nv, it)
                # a captured call replayed: the epoch lives on the device
                xs = torch.randn(nv, cols, device=dev, generator=g)
                s = torch.cuda.Stream(device=dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(s):
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=s):
                        matvec_tp(shard, xs, grp, buf, stream=s)
                    want = sg.matvec(full, mf, xs, stream=s)
                    for _ in range(3):
                        buf.tensor.fill_(float("nan"))
                        torch.cuda.synchronize(dev)
                        dist.barrier()  # every rank's buffer is cleared before any rank writes
                        graph.replay()
                        torch.cuda.synchronize(dev)
                        ok = np.array_equal(buf.tensor.cpu().numpy().view(np.uint32),
                                            want.cpu().numpy().view(np.uint32))
                        dist.barrier()
                        assert ok, (dt, rows, "graph")
                del graph
                torch.cuda.synchronize(dev)
                dist.barrier()
        sg.device_status()
        out.put((rank, "ok"))
    except Exception as e:
        out.put((rank, repr(e)))
    finally:
        if grp is not None:
            try:
                grp.close()
            except Exception as e:
                out.put((rank, "close: " + repr(e)))
        dist.destroy_process_group()


def ep_layer(dev, seed=9, ne=32, k=4, dim=512, ff=256):
    """A random MoE layer, the same on every rank (GGUF expert tensors)."""
    import torch
    import spindle_b200 as sg
    g = torch.Generator(device=dev).manual_seed(seed)
    router = torch.randn(ne, dim, device=dev, generator=g) / dim ** 0.5
    gq = sg.quantize_weights(sg.Q4_K, torch.randn(ne * ff, dim, device=dev, generator=g) * 0.02)
    uq = sg.quantize_weights(sg.Q4_K, torch.randn(ne * ff, dim, device=dev, generator=g) * 0.02)
    dq = sg.quantize_weights(sg.Q6_K, torch.randn(ne * dim, ff, device=dev, generator=g) * 0.02)
    return router, gq, uq, dq, ne, k, dim, ff


def ep_check(dev, grp, out_fail):
    """EpMoe against the whole layer on this GPU, bit for bit, over batches,
    repeated calls and a graph replay; returns a list of failures."""
    import numpy as np
    import torch
    import spindle_b200 as sg
    from spindle_b200.tp import EpMoe
    router, gq, uq, dq, ne, k, dim, ff = ep_layer(dev)
    full = sg.Moe.pack(router, gq, uq, dq, sg.Q4_K, sg.Q6_K, ne, k, dim, ff)
    ep = EpMoe(grp, router, gq, uq, dq, sg.Q4_K, sg.Q6_K, ne, k, dim, ff, n_tok_max=17)
    g = torch.Generator(device=dev).manual_seed(21)
    bad = []
    for it, nt in enumerate([1, 9, 17, 3, 9]):
        xs = torch.randn(nt, dim, device=dev, generator=g)
        got = ep.forward(xs)
        want = sg.moe_forward_batch(full, xs)
        torch.cuda.synchronize(dev)
        if not np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32)):
            bad.append(("batch", it, nt))
    xs = torch.randn(9, dim, device=dev, generator=g)
    out = torch.empty(9, dim, device=dev)
    want = sg.moe_forward_batch(full, xs)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        ep.forward(xs, out, stream=s)  # allocates its scratch outside the capture
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            ep.forward(xs, out, stream=s)
        for r in range(3):
            out.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize(dev)
            if not np.array_equal(out.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32)):
                bad.append(("graph", r))
    del graph
    sg.device_status()
    return bad


def ep_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from spindle_b200.tp import TpGroup
    init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    grp = None
    try:
        grp = TpGroup(device=dev)
        bad = ep_check(dev, grp, out)
        out.put((rank, "ok" if not bad else repr(bad)))
    except Exception as e:
        out.put((rank, repr(e)))
    finally:
        if grp is not None:
            try:
                grp.close()
            except Exception as e:
                out.put((rank, "close: " + repr(e)))
        dist.destroy_process_group()


def pipe_rank(rank, world, port, out):
    # a pipeline of `world` stages: stage p runs layers [L*p/P, L*(p+1)/P) of
    # each prompt chunk (par_rows's split over the layers), receiving the
    # residual from stage p-1 and sending it to stage p+1; the last stage runs
    # the head and compares with the whole model on its own GPU
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import decoder_util as U
    from spindle_b200.decoder import Decoder
    from spindle_b200.tp import PipeLink, TpGroup, shard_rows
    init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    grp = None
    try:
        grp = TpGroup(device=dev)
        msgs = []
        for kind, cfg in [("moe", dict(U.MOE, n_layers=8, max_seq=128)), ("dense", dict(U.DENSE, n_layers=8))]:
            dtypes = U.dtypes_for(cfg)
            W = U.device_weights(U.host_weights(cfg, dtypes, seed=61), dev)
            stage = Decoder(cfg, W, dtypes, dev)
            links = [PipeLink(grp, p, p + 1, 32 * cfg["dim"]) for p in range(world - 1)]
            toks = np.random.default_rng(3).integers(0, cfg["vocab"], 50).tolist()
            chunks = [9, 32, 1, 8]
            L = cfg["n_layers"]
            l0, l1 = shard_rows(L, world, rank)
            whole = Decoder(cfg, W, dtypes, dev) if rank == world - 1 else None
            pos = 0
            for c in chunks:
                if rank == 0:
                    (h,) = stage.forward_batch_range(pos, l0, l1, tokens=toks[pos:pos + c])
                else:
                    h = links[rank - 1].recv(torch.empty(c, cfg["dim"], device=dev))
                    if rank < world - 1:
                        (h,) = stage.forward_batch_range(pos, l0, l1, hidden=h)
                if rank < world - 1:
                    links[rank].send(h)
                else:
                    lg, gr = stage.forward_batch_range(pos, l0, l1, hidden=h)
                    wl, wg = whole.forward_batch(toks[pos:pos + c], pos)
                    torch.cuda.synchronize(dev)
                    if not (np.array_equal(lg.cpu().numpy().view(np.uint32), wl.cpu().numpy().view(np.uint32))
                            and torch.equal(gr, wg)):
                        msgs.append((kind, pos, c))
                pos += c
            torch.cuda.synchronize(dev)
            dist.barrier()
        __import__("spindle_b200").device_status()
        out.put((rank, "ok" if not msgs else repr(msgs)))
    except Exception as e:
        out.put((rank, repr(e)))
    finally:
        if grp is not None:
            try:
                grp.close()
            except Exception as e:
                out.put((rank, "close: " + repr(e)))
        dist.destroy_process_group()


def decoder_ep_rank(rank, world, port, out):
    # the decoder step with expert parallelism (sg_forward_ep) against the
    # whole model on this GPU (sg_forward): logits bit for bit and the same
    # greedy tokens, eager and replayed as a CUDA graph, on a small MoE model
    # and on two layers of the Qwen3-30B-A3B shape
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import decoder_util as U
    from spindle_b200.decoder import Decoder, qwen3_dtypes, random_weights
    from spindle_b200.tp import TpGroup
    init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    grp = None
    try:
        grp = TpGroup(device=dev)
        msgs = []
        small = dict(U.MOE, n_layers=3, max_seq=64)
        big = dict(dim=2048, n_heads=32, n_kv_heads=4, head_dim=128, n_layers=2, vocab=151936, max_seq=64,
                   rope_theta=1e6, rms_eps=1e-6, rope_neox=True,
                   moe=dict(n_expert=128, n_used=8, n_ff=768, norm=True))
        for kind, cfg in [("small", small), ("qwen3_30b_a3b_2layers", big)]:
            if kind == "small":
                dtypes = U.dtypes_for(cfg)
                W = U.device_weights(U.host_weights(cfg, dtypes, seed=71), dev)
            else:
                dtypes = qwen3_dtypes(cfg, embed=U.Q4_K)
                W = random_weights(cfg, dtypes, dev, seed=72)
            full = Decoder(cfg, W, dtypes, dev)
            epd = Decoder(cfg, W, dtypes, dev, ep=grp)
            seq = [5, 77, 130, 9]
            for pos in range(16):
                t = seq[pos]
                full.set_state(t, pos)
                full.step()
                epd.set_state(t, pos)
                epd.step()
                torch.cuda.synchronize(dev)
                if not (np.array_equal(full.logits.cpu().numpy().view(np.uint32),
                                       epd.logits.cpu().numpy().view(np.uint32))
                        and int(full.token.item()) == int(epd.token.item())
                        and torch.equal(full.state, epd.state)):
                    msgs.append((kind, "eager", pos))
                if len(seq) == pos + 1:
                    seq.append(int(full.token.item()))
            # one captured step replayed token after token: the epoch counters live on the device
            want = full.generate(seq[:4], 8)
            for i, t in enumerate(seq[:4]):
                epd.set_state(t, i)
                epd.step(hidden=False, logits=False)
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            got = []
            with torch.cuda.stream(s):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    epd.step(stream=s, hidden=False, logits=False)
                for _ in range(8):
                    got.append(int(epd.state[0].item()))
                    graph.replay()
                    torch.cuda.synchronize(dev)
            torch.cuda.current_stream(dev).wait_stream(s)
            del graph
            if got != want:
                msgs.append((kind, "graph", got, want))
            del full, epd, W
            torch.cuda.synchronize(dev)
            dist.barrier()
        __import__("spindle_b200").device_status()
        out.put((rank, "ok" if not msgs else repr(msgs)))
    except Exception as e:
        out.put((rank, repr(e)))
    finally:
        if grp is not None:
            try:
                grp.close()
            except Exception as e:
                out.put((rank, "close: " + repr(e)))
        dist.destroy_process_group()


def pipe_shift_loop(stage, whole, n_keep, n_steps, dev):
    """Greedy decode through a PipelineStage past its context, shifting the KV
    window on every stage when needed; the last stage checks every step's
    logits against `whole` (the model on one GPU, shifted alike).  Returns
    (failures, shifts); every rank calls it with the same arguments."""
    import numpy as np
    import torch
    from spindle_b200.tp import exchange
    tok, pos, shifts, bad = 17, 0, 0, []
    last = stage.rank == stage.n - 1
    for _ in range(n_steps):
        new = stage.ensure_kv_room(pos, 1, n_keep)
        if new != pos:
            shifts += 1
            if last:
                assert whole.shift_kv(n_keep, pos - new, pos) == new
            pos = new
        out = stage.forward([tok], pos)
        nxt = None
        if last:
            lg, gr = out
            wl, wg = whole.forward_batch([tok], pos)
            torch.cuda.synchronize(dev)
            if not (np.array_equal(lg.cpu().numpy().view(np.uint32), wl.cpu().numpy().view(np.uint32))
                    and torch.equal(gr, wg)):
                bad.append((pos, shifts))
            nxt = int(gr[0].item())
        tok = exchange(nxt, stage.grp.group)[stage.n - 1]
        pos += 1
    return bad, shifts


def pipe_kv_rank(rank, world, port, out):
    # KV_SHIFT / KV_INFO across a pipeline of `world` stages: decoding past the
    # context keeps every stage's window in step, bit for bit the one-GPU model
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import decoder_util as U
    from spindle_b200.decoder import Decoder
    from spindle_b200.tp import PipelineStage, TpGroup
    init(rank, world, port, "nccl")
    dev = torch.device("cuda", rank)
    grp = None
    try:
        grp = TpGroup(device=dev)
        # the last stage has the smaller cache: kv_info clamps the pipeline to it
        cfg = dict(U.MOE, n_layers=8, max_seq=48 if rank == world - 1 else 64)
        dtypes = U.dtypes_for(cfg)
        W = U.device_weights(U.host_weights(cfg, dtypes, seed=62), dev)
        stage = PipelineStage(Decoder(cfg, W, dtypes, dev), grp, n_max=8)
        whole = Decoder(dict(cfg, max_seq=48), W, dtypes, dev) if rank == world - 1 else None
        msgs = []
        if stage.max_seq != 48:
            msgs.append(("kv_info", stage.max_seq))
        bad, shifts = pipe_shift_loop(stage, whole, 4, 120, dev)
        if bad or shifts < 3:
            msgs.append(("shift", bad, shifts))
        torch.cuda.synchronize(dev)
        dist.barrier()
        __import__("spindle_b200").device_status()
        out.put((rank, "ok" if not msgs else repr(msgs)))
    except Exception as e:
        out.put((rank, repr(e)))
    finally:
        if grp is not None:
            try:
                grp.close()
            except Exception as e:
                out.put((rank, "close: " + repr(e)))
        dist.destroy_process_group()
