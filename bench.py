#!/usr/bin/env python
"""Headline benchmark: K-quant GEMV HBM GB/s on B200 (BASELINE.json metric and
Q4_K and Q6_K weights x Q8_K activations at 4096x4096,
14336x4096, 4096x14336 and the 151936x1024 Q6_K LM head).

One step = the hot path of `matvec` (smollm_chat.rs:309-318) over every matrix
of the sweep: Q8_K-quantize that step's activation, then the integer GEMV
(quant_q8k::matmul_rows).  N(0, 0.02) weights quantized by the library's own
quantizer, N(0, 1) activations, all seeded; synthetic data.  The 7 matrices
hold 314 MB, more than the 126 MB L2, so every matrix is evicted before it is
read again.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--nvec B] [--impl reference]

N > 1 (under torchrun): strong scaling.  Every matrix of the sweep is split
by rows over the ranks (par_rows's split, smollm_chat.rs:332-337); one
sg_matvec_tp per matrix leaves the whole output on every rank, its rows
stored by each rank's GEMV epilogue straight into every peer's receive buffer
over NVLink (no NCCL call on the data path).  value = the whole sweep's
algorithmic bytes / max-over-ranks step time.
--impl reference: the reference's CPU algorithm (the oracle's C restatement
of the AVX2 kernels with its worker pool) on all host cores, same metric.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q4_K, Q6_K = 12, 14
SHAPES = [(Q4_K, 4096, 4096), (Q6_K, 4096, 4096), (Q4_K, 14336, 4096), (Q6_K, 14336, 4096),
          (Q4_K, 4096, 14336), (Q6_K, 4096, 14336), (Q6_K, 151936, 1024)]
BLK = {Q4_K: 144, Q6_K: 210}
L2_BYTES = 126 * 1024 * 1024
NAME = {Q4_K: "Q4_K", Q6_K: "Q6_K"}
METRIC = "K-quant GEMV HBM GB/s (Q4_K/Q6_K x Q8_K sweep)"


def cpu_model():
    """The host CPU's model name (the cpu_baseline's hardware)."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def alg_bytes(dt, rows, cols, n):
    """Algorithmic bytes of one GEMV: weights + Q8_K activations + fp32 out."""
    return rows * (cols // 256) * BLK[dt] + n * (cols + 4 * cols // 256 + 2 * cols // 16) + n * rows * 4


def step_bytes(n):
    return sum(alg_bytes(dt, r, c, n) for dt, r, c in SHAPES)


def profiled_traffic(args):
    """DRAM bytes (read + write) of one sweep step's GEMV launches, from the
    committed ncu launch list of this workload (N = 1 vector, tiled layout,
    all seven matrices); None for any other configuration."""
    if args.nvec != 1 or getattr(args, "layout", "tiled") != "tiled" or args.shape is not None:
        return None
    import re
    try:
        text = open(os.path.join(ROOT, "profiles", "bench_launch_list.md")).read()
        m = re.search(r"^\| step \| \| [\d.]+ \| ([\d.]+) \|", text, re.M)
        return int(float(m.group(1)) * 1e6) if m else None
    except OSError:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x1: "gpu_idle", 0x2: "applications_clocks_setting"}

    def __init__(self, index, period=0.01):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        names = sorted(n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle")
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "NVML, 10 ms period, during the timed region"}


def rank_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def cpu_sample(shapes_host, nvec, budget_s, threads):
    """Times the oracle's pooled matvec (the reference's CPU algorithm) on
    full sweeps until budget_s is spent (at least one sweep after warm-up)."""
    import numpy as np
    import oracle as O
    O.pool_create(threads)
    try:
        g = np.random.default_rng(7)
        xs = [g.standard_normal((nvec, c), dtype=np.float32) for _, _, c in SHAPES]
        outs = [np.empty((nvec, r), np.float32) for _, r, _ in SHAPES]
        mats = [O.Mat(dt, c, r) for dt, r, c in SHAPES]

        def sweep(frac=1.0):
            for k, (dt, r, c) in enumerate(SHAPES):
                m = mats[k] if frac >= 1.0 else O.Mat(dt, c, max(1, int(r * frac)))
                O.pool_matvec_multi(shapes_host[k], m, xs[k], outs[k])

        sweep()  # warm-up
        t0 = time.perf_counter()
        n = 0
        while True:
            sweep()
            n += 1
            if time.perf_counter() - t0 >= budget_s:
                break
        dt = (time.perf_counter() - t0) / n
    finally:
        O.pool_destroy()
    return dt, n


def host_weights(rank):
    """The sweep's weights as host bytes, made the same way as on the GPU."""
    import numpy as np
    import oracle as O
    g = np.random.default_rng(1000 + rank)
    out = []
    for dt, r, c in SHAPES:
        w = (g.standard_normal((r, c), dtype=np.float32) * np.float32(0.02))
        out.append(O.quantize_weights(dt, w))
    return out


def run_reference(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    wh = host_weights(0)
    # Size each step so that warm-up + steps stay within about two minutes.
    probe, _ = cpu_sample(wh, args.nvec, 0.0, threads)
    total = args.steps + args.warmup
    frac = min(1.0, 120.0 / max(total * probe, 1e-9))
    import numpy as np
    import oracle as O
    O.pool_create(threads)
    try:
        g = np.random.default_rng(7)
        xs = [g.standard_normal((args.nvec, c), dtype=np.float32) for _, _, c in SHAPES]
        outs = [np.empty((args.nvec, r), np.float32) for _, r, _ in SHAPES]
        mats = [O.Mat(dt, c, max(1, int(r * frac))) for dt, r, c in SHAPES]
        bytes_step = sum(alg_bytes(dt, m.rows, c, args.nvec) for (dt, _, c), m in zip(SHAPES, mats))
        for _ in range(args.warmup):
            for k in range(len(SHAPES)):
                O.pool_matvec_multi(wh[k], mats[k], xs[k], outs[k])
        t0 = time.perf_counter()
        for _ in range(args.steps):
            for k in range(len(SHAPES)):
                O.pool_matvec_multi(wh[k], mats[k], xs[k], outs[k])
        el = time.perf_counter() - t0
    finally:
        O.pool_destroy()
    value = bytes_step * args.steps / el / 1e9
    sample = "each step: rows [0, %.4g x rows) of every sweep matrix" % frac if frac < 1 else "each step: the full sweep"
    tp = getattr(args, "workload", "gemv") == "gemv_tp"
    line = {"impl": "reference", "metric": TP_METRIC if tp else METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8/int32 + fp32",
            "data": "synthetic", "config": config_block(args, 1),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                             "sample": sample + "; oracle = C restatement of quant_q8k.rs with the worker pool"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_block(args, world):
    return {"workload": "gemv_sweep_n%d" % args.nvec, "layout": getattr(args, "layout", "tiled"),
            "shapes": ["%s %dx%d" % (NAME[dt], r, c) for dt, r, c in SHAPES],
            "n_vec": args.nvec, "global_batch": args.nvec,
            "parallelism": "single GPU" if world == 1 else "row-split x%d (strong)" % world,
            "l2": "314 MB of weights per step > 126 MB L2: each matrix is evicted before its next read",
            "weights": "N(0,0.02) seeded, own Q4_K/Q6_K quantizer", "activations": "N(0,1) seeded"}


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200 import _lib

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    lib = sg.lib()
    nvec = args.nvec

    # ---- resident inputs: weights, activations, Q8_K buffers, outputs ------
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    W, WG, X, XQ, OUT, M = [], [], [], [], [], []
    for dt, r, c in SHAPES:
        wf = torch.randn(r, c, device=dev, generator=gen) * 0.02
        wq = sg.quantize_weights(dt, wf)
        del wf
        WG.append(wq)
        if args.layout == "tiled":
            t, m = sg.repack_tiled16(dt, wq, r, c)
            W.append(t)
            M.append(m)
        else:
            W.append(wq)
            M.append(sg.Mat(dt, c, r))
        X.append(torch.randn(nvec, c, device=dev, generator=gen))
        XQ.append([sg.Q8K(c, dev) for _ in range(nvec)])
        OUT.append(torch.empty(nvec, r, device=dev))
    torch.cuda.synchronize()
    # One vector on TILED16: the step is the list form, the activations' Q8_K
    # images in one launch (sg_q8k_images) and the 7 GEMVs in one persistent
    # launch (sg_matvec_list_q8k); otherwise one launch (or two) per matrix.
    as_list = nvec == 1 and args.layout == "tiled" and args.form == "list"
    XS = [X[k][0] for k in range(len(SHAPES))]
    IMGS = sg.q8k_images(XS) if as_list else None
    EQ = [(W[k], M[k], IMGS[k]) for k in range(len(SHAPES))] if as_list else None
    OUTS = [OUT[k][0] for k in range(len(SHAPES))]

    def gemv(k):
        if args.layout == "tiled":
            sg.matvec(W[k], M[k], X[k], OUT[k])  # Q8_K quantization fused into the GEMV kernel
        else:
            sg.quantize_into(X[k], XQ[k])
            sg.matmul_rows(W[k], M[k], XQ[k], [OUT[k][b] for b in range(nvec)], 0, M[k].rows)

    def per_matrix():
        for k in range(len(SHAPES)):
            gemv(k)

    def step():
        if as_list:
            sg.q8k_images(XS, IMGS)
            sg.matvec_list_q8k(EQ, OUTS)
        else:
            per_matrix()

    # Warm-up outside capture (plans, function attributes), then capture.
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        g_step = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=stream):
            step()
        g_gemv = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_gemv, stream=stream):
            if as_list:
                sg.matvec_list_q8k(EQ, OUTS)
            else:
                per_matrix()
        g_per = None
        if as_list:
            # the same 7 GEMVs one launch per matrix, reported beside the list
            # form; its outputs must be the list form's bit for bit
            want = [o.clone() for o in OUTS]
            per_matrix()
            torch.cuda.synchronize()
            if not all(torch.equal(a.view(torch.int32), b.view(torch.int32)) for a, b in zip(want, OUTS)):
                raise RuntimeError("list form and per-matrix GEMVs differ")
            g_per = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_per, stream=stream):
                per_matrix()
    launches_per_step = 2 if as_list else (1 if args.layout == "tiled" else 2) * len(SHAPES)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g_step.replay()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                g_step.replay()
            e1.record(stream)
            e1.synchronize()
            # a soak of about a second of the same step right after, still
            # sampled, so that the clock record holds many samples under load
            n_soak = 0
            if not args.profile:
                s0.record(stream)
                t_end = time.time() + 1.0
                while time.time() < t_end:
                    for _ in range(200):
                        g_step.replay()
                    n_soak += 200
                    s1.record(stream)
                    s1.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        soak_ms = s0.elapsed_time(s1) / n_soak if n_soak else None
        if args.profile:
            if rank == 0:
                print(json.dumps({"profile": True, "shapes": [list(s) for s in SHAPES], "ms_per_step": ms}))
            return None, WG

        # Roofline of the dominant kernel: the 7 GEMV launches alone, replayed.
        reps = max(args.warmup, min(args.steps, 2000))
        for _ in range(args.warmup):
            g_gemv.replay()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(reps):
            g_gemv.replay()
        f1.record(stream)
        f1.synchronize()
        gemv_ms = f0.elapsed_time(f1) / reps  # the list launch, or the 7 launches
        per_ms = None
        if g_per is not None:
            for _ in range(args.warmup):
                g_per.replay()
            f0.record(stream)
            for _ in range(reps):
                g_per.replay()
            f1.record(stream)
            f1.synchronize()
            per_ms = f0.elapsed_time(f1) / reps

        # Per-shape GEMV time: one launch, timed right after the whole sweep
        # has streamed 314 MB through L2, so the matrix is read from HBM.
        per_shape = []
        for k, (dt, r, c) in enumerate(SHAPES):
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1, stream=stream):
                gemv(k)
            tot = 0.0
            n_rep = 20
            for _ in range(n_rep):
                g_gemv.replay()           # evicts matrix k from L2 (314 MB streamed)
                a0.record(stream)
                g1.replay()
                a1.record(stream)
                a1.synchronize()
                tot += a0.elapsed_time(a1)
            us = tot / n_rep * 1e3
            per_shape.append({"shape": "%s %dx%d" % (NAME[dt], r, c), "us": round(us, 2),
                              "GB_s": round(alg_bytes(dt, r, c, nvec) / (us * 1e-6) / 1e9, 1)})

        # Per shape as a throughput: the shape alone through the list kernel,
        # over distinct copies that hold 2.5x the L2 (each read from HBM), in
        # lists of up to 16 on the same Q8_K image.
        per_shape_list = []
        if as_list:
            peak_ = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"] \
                if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 6650.0
            for k, (dt, r, c) in enumerate(SHAPES):
                ncp = max(2, -(-int(2.5 * L2_BYTES) // W[k].numel()))
                cps = [W[k]] + [W[k].clone() for _ in range(ncp - 1)]
                o_ = [torch.empty(r, device=dev) for _ in range(min(ncp, 16))]
                lists = [[(w_, M[k], IMGS[k]) for w_ in cps[i:i + 16]] for i in range(0, ncp, 16)]

                def run_lists():
                    for L_ in lists:
                        sg.matvec_list_q8k(L_, o_[:len(L_)])

                run_lists()
                torch.cuda.synchronize()
                gl_ = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gl_, stream=stream):
                    run_lists()
                for _ in range(3):
                    gl_.replay()
                q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                q0.record(stream)
                for _ in range(10):
                    gl_.replay()
                q1.record(stream)
                q1.synchronize()
                per = q0.elapsed_time(q1) / 10 / ncp
                gbs = alg_bytes(dt, r, c, 1) / (per * 1e-3) / 1e9
                per_shape_list.append({"shape": "%s %dx%d" % (NAME[dt], r, c), "copies": ncp,
                                       "launches": len(lists), "us_per_matrix": round(per * 1e3, 2),
                                       "GB_s": round(gbs, 1), "frac": round(gbs / peak_, 4)})
                del gl_, cps, o_, lists

        # one Q4_K 3072 x 1024 GEMV (1.78 MB).  Its
        # single-launch latency, read from HBM after the sweep has evicted it,
        # and a chain of launches over copies that hold 2.5x the L2 (each read
        # from HBM), for an aggregate rate.
        c1 = {}
        if args.nvec == 1 and args.layout == "tiled":
            w1 = sg.quantize_weights(Q4_K, torch.randn(3072, 1024, device=dev, generator=gen) * 0.02)
            t1, m1 = sg.repack_tiled16(Q4_K, w1, 3072, 1024)
            x1 = torch.randn(1, 1024, device=dev, generator=gen)
            o1 = torch.empty(1, 3072, device=dev)
            cb = alg_bytes(Q4_K, 3072, 1024, 1)
            ncp = -(-int(2.5 * L2_BYTES) // t1.numel())
            cps = [t1] + [t1.clone() for _ in range(ncp - 1)]
            gs = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gs, stream=stream):
                sg.matvec(t1, m1, x1, o1)
            gc = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gc, stream=stream):
                for w_ in cps:
                    sg.matvec(w_, m1, x1, o1)
            tot = 0.0
            for _ in range(20):
                g_gemv.replay()
                a0.record(stream)
                gs.replay()
                a1.record(stream)
                a1.synchronize()
                tot += a0.elapsed_time(a1)
            for _ in range(2):
                gc.replay()
            a0.record(stream)
            for _ in range(10):
                gc.replay()
            a1.record(stream)
            a1.synchronize()
            per = a0.elapsed_time(a1) / 10 / ncp
            c1 = {"shape": "Q4_K 3072x1024 (configs[0])", "us_single_launch": round(tot / 20 * 1e3, 2),
                  "GB_s_single_launch": round(cb / (tot / 20 * 1e-3) / 1e9, 1),
                  "us_per_launch_in_chain": round(per * 1e3, 2),
                  "GB_s_in_chain": round(cb / (per * 1e-3) / 1e9, 1),
                  "chain": "%d launches over %d copies (%.0f MB > 2.5 x L2), one graph" % (ncp, ncp, ncp * cb / 1e6)}
            del cps, gc, gs
        # BASELINE configs[1]'s vector counts (speculative-verify batches):
        # the same sweep with N = 2, 4, 8 and 16 vectors per matrix
        nvec_sweep = []
        if args.nvec == 1 and args.layout == "tiled":
            for nv in (2, 4, 8, 16):
                Xn = [torch.randn(nv, c, device=dev, generator=gen) for _, _, c in SHAPES]
                On = [torch.empty(nv, r, device=dev) for _, r, _ in SHAPES]
                SCn = [torch.empty(lib.sg_matmul_batch_scratch_bytes(C.byref(M[k].c()), nv), dtype=torch.uint8,
                                   device=dev) for k in range(len(SHAPES))]
                sp_ = C.c_void_p(stream.cuda_stream)

                def tiled_n():  # sg_matvec: the tiled GEMV, up to 8 vectors per launch
                    for k in range(len(SHAPES)):
                        sg.matvec(W[k], M[k], Xn[k], On[k])

                def batch_n():  # sg_matmul_batch: one Q8_K batch image, then the batch GEMM
                    for k in range(len(SHAPES)):
                        _lib.check(lib.sg_matmul_batch(C.c_void_p(W[k].data_ptr()), C.byref(M[k].c()),
                                                       C.c_void_p(Xn[k].data_ptr()), Xn[k].stride(0),
                                                       C.c_void_p(On[k].data_ptr()), On[k].stride(0), nv, 0,
                                                       M[k].rows, C.c_void_p(SCn[k].data_ptr()), SCn[k].numel(),
                                                       sp_), "matmul_batch")

                entry = {"n_vec": nv}
                for label, fn in [("matvec", tiled_n), ("matmul_batch", batch_n)]:
                    fn()
                    torch.cuda.synchronize()
                    gn = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gn, stream=stream):
                        fn()
                    for _ in range(3):
                        gn.replay()
                    a0.record(stream)
                    for _ in range(30):
                        gn.replay()
                    a1.record(stream)
                    a1.synchronize()
                    t_ = a0.elapsed_time(a1) / 30
                    entry[label] = {"us": round(t_ * 1e3, 2), "GB_s": round(step_bytes(nv) / (t_ * 1e-3) / 1e9, 1)}
                    del gn
                nvec_sweep.append(entry)
                del Xn, On, SCn

        # ---- e2e through the C ABI with host buffers -----------------------
        # All activations of a step sit in one pinned host buffer and go up in
        # one copy; each output comes back as soon as its GEMV is done, on a
        # side stream, so the copies overlap the remaining GEMVs (the matrix
        # with the largest output runs first).
        xsz = [nvec * c for _, _, c in SHAPES]
        osz = [nvec * r for _, r, _ in SHAPES]
        xoff = [sum(xsz[:k]) for k in range(len(SHAPES))]
        ooff = [sum(osz[:k]) for k in range(len(SHAPES))]
        XC = torch.empty(sum(xsz), device=dev)
        OC = torch.empty(sum(osz), device=dev)
        h_x = torch.empty(sum(xsz), dtype=torch.float32).pin_memory()
        h_o = torch.empty(sum(osz), dtype=torch.float32).pin_memory()
        for k in range(len(SHAPES)):
            h_x[xoff[k]:xoff[k] + xsz[k]].copy_(X[k].reshape(-1).cpu())
        XV = [XC[xoff[k]:xoff[k] + xsz[k]].view(nvec, -1) for k in range(len(SHAPES))]
        OV = [OC[ooff[k]:ooff[k] + osz[k]].view(nvec, -1) for k in range(len(SHAPES))]
        order = sorted(range(len(SHAPES)), key=lambda k: -osz[k])
        side = torch.cuda.Stream(device=dev)
        evs = [torch.cuda.Event() for _ in range(len(SHAPES) + 1)]
        sp, ssp = C.c_void_p(stream.cuda_stream), C.c_void_p(side.cuda_stream)

        if as_list:
            XE = [XV[k][0] for k in range(len(SHAPES))]
            IE = sg.q8k_images(XE)
            EE = [(W[k], M[k], IE[k]) for k in range(len(SHAPES))]
            OE = [OV[k][0] for k in range(len(SHAPES))]

        def e2e_step():
            _lib.check(lib.sg_memcpy_h2d(C.c_void_p(XC.data_ptr()), C.c_void_p(h_x.data_ptr()), h_x.numel() * 4,
                                         sp), "h2d")
            if as_list:
                # the matrix with the largest output (the LM head) first, as a
                # list of its own: its output goes back on the side stream
                # while the other GEMVs run in a second list; then theirs
                big, rest = order[0], sorted(order[1:])
                sg.q8k_images(XE, IE)
                sg.matvec_list_q8k([EE[big]], [OE[big]])
                evs[0].record(stream)
                side.wait_event(evs[0])
                _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o.data_ptr() + 4 * ooff[big]),
                                             C.c_void_p(OV[big].data_ptr()), osz[big] * 4, ssp), "d2h")
                sg.matvec_list_q8k([EE[k] for k in rest], [OE[k] for k in rest])
                if rest == list(range(len(rest))) and big == len(rest):  # the others' outputs are contiguous
                    _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o.data_ptr()), C.c_void_p(OC.data_ptr()),
                                                 ooff[big] * 4, sp), "d2h")
                else:
                    for k in rest:
                        _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o.data_ptr() + 4 * ooff[k]),
                                                     C.c_void_p(OV[k].data_ptr()), osz[k] * 4, sp), "d2h")
                evs[-1].record(side)
                stream.wait_event(evs[-1])
                return
            for i, k in enumerate(order):
                if args.layout == "tiled":
                    sg.matvec(W[k], M[k], XV[k], OV[k])
                else:
                    sg.quantize_into(XV[k], XQ[k])
                    sg.matmul_rows(W[k], M[k], XQ[k], [OV[k][b] for b in range(nvec)], 0, M[k].rows)
                evs[i].record(stream)
                side.wait_event(evs[i])
                _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o.data_ptr() + 4 * ooff[k]), C.c_void_p(OV[k].data_ptr()),
                                             osz[k] * 4, ssp), "d2h")
            evs[-1].record(side)
            stream.wait_event(evs[-1])

        e2e_step()
        torch.cuda.synchronize()
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=stream):
            e2e_step()
        for _ in range(args.warmup):
            g_e2e.replay()
        barrier()
        reps_e2e = max(3, min(args.steps, 2000))
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        for _ in range(reps_e2e):
            g_e2e.replay()
        b1.record(stream)
        b1.synchronize()
        barrier()
        e2e_ms = max_over_ranks(b0.elapsed_time(b1)) / reps_e2e
    sg.device_status()

    bytes_rank = step_bytes(nvec)
    value = bytes_rank * world / (ms * 1e-3) / 1e9
    gemv_bytes = bytes_rank
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    peak, peak_src = None, "MEASURED_PEAKS.json hbm_gbs"
    try:
        peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
    except Exception:
        peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    h2d = h_x.numel() * 4
    d2h = h_o.numel() * 4
    line = None
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8 x int4/int6 -> int32, fp32 epilogue", "data": "synthetic",
                "config": config_block(args, world),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args),
                             "traffic_source": "profiles/bench_launch_list.md: ncu dram__bytes_read.sum + "
                                               "dram__bytes_write.sum of the step's launches (committed capture)",
                             "algorithmic_bytes": gemv_bytes, "peak_source": peak_src,
                             "kernel": ("gemv_list_kernel" if as_list else "gemv_tiled_kernel") if args.layout == "tiled"
                             else "gemv_q8k_kernel",
                             "how": ("algorithmic bytes of the 7 GEMVs / the replayed duration of the one list "
                                     "launch" if as_list else "algorithmic bytes of the 7 GEMV launches / their "
                                     "replayed duration") + " (CUDA events on the launch stream); traffic = DRAM "
                                    "read + write of the same launches from the committed ncu launch list"},
                "form": ("list: sg_q8k_images (the 7 activations to Q8_K images, one launch) + sg_matvec_list_q8k "
                         "(the 7 GEMVs in one persistent launch)") if as_list else "one sg_matvec launch per matrix",
                "per_matrix_launches": {"us": round(per_ms * 1e3, 2),
                                        "GB_s": round(gemv_bytes / (per_ms * 1e-3) / 1e9, 1),
                                        "how": "the same 7 GEMVs as 7 sg_matvec launches (Q8_K quantization fused "
                                               "in each), replayed; outputs checked equal to the list form's"}
                if per_ms else None,
                "per_shape": per_shape,
                "per_shape_list": {"entries": per_shape_list,
                                   "how": "each shape alone: distinct copies holding 2.5x the L2, as lists of up "
                                          "to 16 GEMVs (sg_matvec_list_q8k) on one Q8_K image, replayed; "
                                          "per matrix = time / copies"} if per_shape_list else None,
                "config1": c1,
                "nvec_sweep": [dict(e, best_frac=round(max(e["matvec"]["GB_s"], e["matmul_batch"]["GB_s"]) / peak, 4))
                               for e in nvec_sweep],
                "soak": {"seconds": round(soak_ms * n_soak / 1e3, 2) if soak_ms else None,
                         "value": round(bytes_rank / (soak_ms * 1e-3) / 1e9, 1) if soak_ms else None,
                         "how": "the step replayed for about a second right after the timed region, inside the "
                                "clock record (same graph, same bytes per step)"},
                "e2e": {"value": round(bytes_rank * world / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "how": ("every step: one sg_memcpy_h2d of all fp32 activations from pinned host, "
                                "sg_q8k_images, sg_matvec_list_q8k on the matrix with the largest output (the "
                                "LM head), whose sg_memcpy_d2h runs on a side stream while sg_matvec_list_q8k "
                                "does the other six, then one sg_memcpy_d2h of their outputs")
                        if as_list else
                               ("every step: one sg_memcpy_h2d of all fp32 activations from pinned host, "
                                "sg_matvec (quantize + GEMV) per matrix, sg_memcpy_d2h of each fp32 output "
                                "on a side stream as soon as its GEMV ends (overlapping the next GEMVs)")},
                "gpu_launches": launches_per_step * args.steps,
                "clocks": clk.summary()}
    if world > 1:
        dist.barrier()
        del g_step, g_gemv, g_e2e, g_per
        dist.destroy_process_group()
    return line, WG


# ---- MoE layer workload (--workload moe) -------------------------------------
# One step = one token through MOE_LAYERS distinct MoE layers of the
# Qwen3-30B-A3B shape (128 experts, top 8, hidden 2048,
# FFN 768, Q4_K gate/up, Q6_K down, F32 router with logits about N(0,1)),
# each layer moe_forward (smollm_chat.rs:1178): router, softmax/top-k, the
# chosen experts' SwiGLU FFNs, the weighted sum.  8 layers hold 3.1 GB of
# experts, so the 24.5 MB a token reads per layer is not left in L2 by the
# step before.

MOE = dict(dim=2048, n_ff=768, n_expert=128, n_used=8, gu=Q4_K, dn=Q6_K)
MOE_LAYERS = 8
MOE_METRIC = "MoE layer decode: chosen-expert weight GB/s (Qwen3-30B-A3B layer, top-8 of 128)"


def moe_layer_bytes(n_chosen):
    """Algorithmic bytes of one token through one layer: F32 router, the chosen
    experts' gate/up/down rows, the input and the output."""
    d, f, ne = MOE["dim"], MOE["n_ff"], MOE["n_expert"]
    per_expert = 2 * f * (d // 256) * BLK[MOE["gu"]] + d * (f // 256) * BLK[MOE["dn"]]
    return ne * d * 4 + n_chosen * per_expert + 2 * d * 4


def moe_host_layers(n_layers, seed=2000):
    """Host weights of the MoE layers (numpy), seeded: router N(0, 1/dim) so
    that logits of an N(0,1) input are about N(0,1); experts N(0, 0.02)."""
    import numpy as np
    import oracle as O
    d, f, ne = MOE["dim"], MOE["n_ff"], MOE["n_expert"]
    g = np.random.default_rng(seed)
    layers = []
    for _ in range(n_layers):
        router = (g.standard_normal((ne, d), dtype=np.float32) / np.float32(np.sqrt(d))).astype(np.float32)
        gate = O.quantize_weights(MOE["gu"], g.standard_normal((ne * f, d), dtype=np.float32) * np.float32(0.02))
        up = O.quantize_weights(MOE["gu"], g.standard_normal((ne * f, d), dtype=np.float32) * np.float32(0.02))
        down = O.quantize_weights(MOE["dn"], g.standard_normal((ne * d, f), dtype=np.float32) * np.float32(0.02))
        layers.append((router, gate, up, down))
    return layers


def moe_oracle(layer):
    import numpy as np
    import oracle as O
    router, gate, up, down = layer
    d, f, ne = MOE["dim"], MOE["n_ff"], MOE["n_expert"]
    parts = [np.ascontiguousarray(router, np.float32).reshape(-1).view(np.uint8), gate, up, down]
    off = np.cumsum([0] + [p.nbytes for p in parts])
    moe = O.Moe(router=O.Mat(O.F32, d, ne, 0), gate=O.Mat(MOE["gu"], d, f, int(off[1])),
                up=O.Mat(MOE["gu"], d, f, int(off[2])), down=O.Mat(MOE["dn"], f, d, int(off[3])), n_expert=ne,
                n_used=MOE["n_used"], norm=1, moe_prune=0.0)
    return np.concatenate(parts), moe


def moe_cpu_sample(layers_host, budget_s):
    """Times the oracle's moe_forward (one thread) token-layers for budget_s."""
    import numpy as np
    import oracle as O
    bufs = [moe_oracle(l) for l in layers_host]
    g = np.random.default_rng(11)
    xs = [g.standard_normal(MOE["dim"], dtype=np.float32) for _ in range(16)]
    O.moe_forward(bufs[0][0], bufs[0][1], xs[0])  # warm-up
    t0, n, nbytes = time.perf_counter(), 0, 0
    while True:
        raw, moe = bufs[n % len(bufs)]
        _, chosen, _ = O.moe_forward(raw, moe, xs[n % len(xs)])
        nbytes += moe_layer_bytes(len(chosen))
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    return el / n, nbytes / el / 1e9, n


def moe_config(world):
    return {"workload": "moe_layer_decode_qwen3_30b_a3b", "layers_per_step": MOE_LAYERS,
            "dim": MOE["dim"], "n_ff": MOE["n_ff"], "n_expert": MOE["n_expert"], "top_k": MOE["n_used"],
            "gate_up": NAME[MOE["gu"]], "down": NAME[MOE["dn"]], "router": "F32", "moe_prune": 0.0,
            "global_batch": world, "parallelism": "replicas x%d (weak)" % world,
            "l2": "8 layers x 391 MB of experts > 126 MB L2: a layer's experts are evicted before its next step",
            "weights": "router N(0,1/dim), experts N(0,0.02) seeded, own Q4_K/Q6_K quantizer",
            "activations": "N(0,1) seeded, a different token per layer and step"}


def run_reference_moe(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return
    layers = moe_host_layers(1)
    per_layer, gbs, n = moe_cpu_sample(layers, 2.0)
    # each step: MOE_LAYERS token-layers; whole run within about two minutes
    total = (args.steps + args.warmup) * MOE_LAYERS * per_layer
    steps = args.steps if total <= 120 else max(1, int(120 / (MOE_LAYERS * per_layer)) - args.warmup)
    per_layer, gbs, n = moe_cpu_sample(layers, per_layer * MOE_LAYERS * (steps + args.warmup))
    line = {"impl": "reference", "metric": MOE_METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_layer * MOE_LAYERS * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8/int32 + fp32", "data": "synthetic", "config": moe_config(1),
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port", "cpu_model": cpu_model(),
                             "sample": "%d token-layers through the oracle's moe_forward (C restatement of "
                                       "smollm_chat.rs moe_forward/ffns_fused), one thread" % n},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gpu_moe(args):
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200 import _lib

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    lib = sg.lib()
    d, f, ne, k = MOE["dim"], MOE["n_ff"], MOE["n_expert"], MOE["n_used"]
    gen = torch.Generator(device=dev).manual_seed(3000 + rank)
    layers, host0 = [], None
    for li in range(MOE_LAYERS):
        router = torch.randn(ne, d, device=dev, generator=gen) / d ** 0.5
        gq = sg.quantize_weights(MOE["gu"], torch.randn(ne * f, d, device=dev, generator=gen) * 0.02)
        uq = sg.quantize_weights(MOE["gu"], torch.randn(ne * f, d, device=dev, generator=gen) * 0.02)
        dq = sg.quantize_weights(MOE["dn"], torch.randn(ne * d, f, device=dev, generator=gen) * 0.02)
        layers.append(sg.Moe.pack(router, gq, uq, dq, MOE["gu"], MOE["dn"], ne, k, d, f))
        if li == 0:  # GGUF bytes of layer 0 for the CPU baseline
            host0 = (router.cpu().numpy(), gq.cpu().numpy(), uq.cpu().numpy(), dq.cpu().numpy())
        del gq, uq, dq
    torch.cuda.synchronize()
    nx = 64  # distinct tokens, so that the chosen experts change from step to step
    X = torch.randn(nx, MOE_LAYERS, d, device=dev, generator=gen)
    OUT = torch.empty(MOE_LAYERS, d, device=dev)
    CH = torch.zeros(MOE_LAYERS, 36, dtype=torch.int32, device=dev)
    scratch = [torch.empty(l.scratch_bytes(), dtype=torch.uint8, device=dev) for l in layers]
    stream = torch.cuda.Stream(device=dev)

    def step(t):
        for l in range(MOE_LAYERS):
            sg.moe_forward(layers[l], X[t % nx, l], OUT[l], scratch[l], choice=CH[l], stream=stream)

    with torch.cuda.stream(stream):
        step(0)
        torch.cuda.synchronize()
        graphs = []
        for t in range(nx):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(t)
            graphs.append(g)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % nx].replay()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for i in range(args.steps):
                graphs[i % nx].replay()
            e1.record(stream)
            e1.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        # bytes: the experts each layer actually chose (all n_used: no pruning)
        n_ch = [int(c) for c in CH[:, 0].cpu()]
        bytes_step = sum(moe_layer_bytes(n) for n in n_ch)

        # e2e: host x -> device, moe_forward, device out -> host, per layer
        h_x = torch.empty(nx, MOE_LAYERS, d, dtype=torch.float32).pin_memory()
        h_x.copy_(X.cpu())
        h_o = torch.empty(MOE_LAYERS, d, dtype=torch.float32).pin_memory()
        sp = C.c_void_p(stream.cuda_stream)

        def e2e_step(t):
            for l in range(MOE_LAYERS):
                _lib.check(lib.sg_memcpy_h2d(C.c_void_p(X[t % nx, l].data_ptr()), C.c_void_p(h_x[t % nx, l].data_ptr()),
                                             d * 4, sp), "h2d")
                sg.moe_forward(layers[l], X[t % nx, l], OUT[l], scratch[l], choice=CH[l], stream=stream)
                _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o[l].data_ptr()), C.c_void_p(OUT[l].data_ptr()), d * 4, sp),
                           "d2h")

        e2e_step(0)
        torch.cuda.synchronize()
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=stream):
            e2e_step(1)
        for _ in range(args.warmup):
            g_e2e.replay()
        barrier()
        reps = max(3, min(args.steps, 2000))
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        for _ in range(reps):
            g_e2e.replay()
        b1.record(stream)
        b1.synchronize()
        barrier()
        e2e_ms = max_over_ranks(b0.elapsed_time(b1)) / reps
    sg.device_status()
    value = bytes_step * world / (ms * 1e-3) / 1e9
    peak, peak_src = None, "MEASURED_PEAKS.json hbm_gbs"
    try:
        peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
    except Exception:
        peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    line = None
    if rank == 0:
        achieved = bytes_step / (ms * 1e-3) / 1e9
        line = {"metric": MOE_METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 5), "us_per_token_layer": round(ms * 1e3 / MOE_LAYERS, 2),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 x int4/int6 -> int32, fp32 router/softmax/epilogue", "data": "synthetic",
                "config": moe_config(world),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                             "kernel": "the 4-kernel MoE chain (router, gate/up, down, combine)",
                             "how": "algorithmic bytes of the chosen experts + router per step / step time"},
                "e2e": {"value": round(bytes_step * world / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                        "h2d_bytes_per_step": MOE_LAYERS * d * 4, "d2h_bytes_per_step": MOE_LAYERS * d * 4,
                        "how": "per layer: sg_memcpy_h2d of x from pinned host, sg_moe_forward, sg_memcpy_d2h of out"},
                "gpu_launches": 4 * MOE_LAYERS * args.steps,
                "clocks": clk.summary()}
    if world > 1:
        dist.barrier()
        del graphs, g_e2e
        dist.destroy_process_group()
    return line, host0


# ---- decode workload (--workload decode) -------------------------------------
# BASELINE configs[3] (Qwen3-30B-A3B, 48 layers, hidden 2048, 32/4 heads of
# 128, 128 experts top 8 with FFN 768, vocab 151936) and configs[2]
# (Qwen3-0.6B dense): random-init Q4_K_M mix (Q6_K attn_v, down and head),
# a 64-token random prompt fed one token at a time, then greedy decode steps.
# One step = one token through forward_slice + LM head + argmax, replayed from
# one captured graph (the token and position are device state).

FLOAT_METRIC = "float-path GEMV HBM GB/s (F16 / Q8_0 / float-mode Q4_K, Q6_K / F32 router, one vector)"
F32_, F16_, Q8_0_ = 0, 1, 8
FLOAT_SHAPES = [(F16_, 14336, 4096), (Q8_0_, 14336, 4096), (Q4_K, 14336, 4096), (Q6_K, 14336, 4096), (F32_, 128, 2048)]
FLOAT_NAME = {F32_: "F32", F16_: "F16", Q8_0_: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def float_row_bytes(dt, cols):
    return {F32_: 4 * cols, F16_: 2 * cols, Q8_0_: cols // 32 * 34, Q4_K: cols // 256 * 144, Q6_K: cols // 256 * 210}[dt]


def float_bytes():
    """Weights + fp32 activation + fp32 output of each matvec of the float sweep."""
    return sum(r * float_row_bytes(dt, c) + 4 * c + 4 * r for dt, r, c in FLOAT_SHAPES)


def run_float(args):
    """The float path (matvec_rows_avx2, quant.rs:939-1094) over FLOAT_SHAPES,
    one sg_matvec_rows_float per matrix; 261 MB of weights (> L2)."""
    import torch
    import spindle_b200 as sg
    from spindle_b200 import _lib
    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    gen = torch.Generator(device=dev).manual_seed(4000 + rank)
    W, M, X, OUT = [], [], [], []
    for dt, r, c in FLOAT_SHAPES:
        wf = torch.randn(r, c, device=dev, generator=gen) * 0.02
        if dt in (Q4_K, Q6_K):
            w = sg.quantize_weights(dt, wf)
        elif dt == F16_:
            w = wf.half().view(torch.uint8).reshape(-1)
        elif dt == F32_:
            w = wf.view(torch.uint8).reshape(-1).clone()
        else:  # Q8_0 blocks: f16 d then 32 int8 (random bytes with a small d)
            w = torch.randint(0, 256, (r * c // 32 * 34,), dtype=torch.uint8, device=dev, generator=gen)
            w.view(r, c // 32, 34)[:, :, 0] = 0
            w.view(r, c // 32, 34)[:, :, 1] = 0x20
        del wf
        W.append(w)
        M.append(sg.Mat(dt, c, r))
        X.append(torch.randn(1, c, device=dev, generator=gen))
        OUT.append(torch.empty(1, r, device=dev))
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    lib = sg.lib()

    def step():
        for k in range(len(FLOAT_SHAPES)):
            sg.matvec_rows_float(W[k], M[k], X[k], OUT[k], stream=stream)

    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if args.profile:
            return None
        h_x = [torch.empty(1, c).pin_memory() for _, _, c in FLOAT_SHAPES]
        h_o = [torch.empty(1, r).pin_memory() for _, r, _ in FLOAT_SHAPES]
        sp = C.c_void_p(stream.cuda_stream)

        def e2e_step():
            for k in range(len(FLOAT_SHAPES)):
                _lib.check(lib.sg_memcpy_h2d(C.c_void_p(X[k].data_ptr()), C.c_void_p(h_x[k].data_ptr()),
                                             h_x[k].numel() * 4, sp), "h2d")
                sg.matvec_rows_float(W[k], M[k], X[k], OUT[k], stream=stream)
                _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o[k].data_ptr()), C.c_void_p(OUT[k].data_ptr()),
                                             h_o[k].numel() * 4, sp), "d2h")

        e2e_step()
        torch.cuda.synchronize()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            e2e_step()
        for _ in range(args.warmup):
            g2.replay()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, min(args.steps, 1000))
        b0.record(stream)
        for _ in range(reps):
            g2.replay()
        b1.record(stream)
        b1.synchronize()
        e2e_ms = b0.elapsed_time(b1) / reps
    sg.device_status()
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    total = float_bytes()
    value = total * world / (ms * 1e-3) / 1e9
    peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    try:
        peak, peak_src = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"], "MEASURED_PEAKS.json hbm_gbs"
    except Exception:
        pass
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and args.cpu_budget > 0:
            import oracle as O
            hw = [w.cpu().numpy() for w in W]
            hx = [x.cpu().numpy()[0] for x in X]
            n, t0 = 0, time.perf_counter()
            while True:
                for k, (dt, r, c) in enumerate(FLOAT_SHAPES):
                    rows = max(1, int(r * 0.05))  # a bounded sample: the first 5% of each matrix's rows
                    O.matvec_rows(hw[k], O.Mat(dt, c, r), hx[k], 0, rows)
                n += 1
                if time.perf_counter() - t0 > min(args.cpu_budget, 10.0):
                    break
            el = (time.perf_counter() - t0) / n
            sample_bytes = sum(max(1, int(r * 0.05)) * float_row_bytes(dt, c) for dt, r, c in FLOAT_SHAPES)
            cpu = {"value": round(sample_bytes / el / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port", "cpu_model": cpu_model(),
                   "sample": "%d passes of the oracle's matvec_rows (the restated AVX2 float kernels, one thread) "
                             "over the first 5%% of each matrix's rows" % n}
        line = {"metric": FLOAT_METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (f16 / int8 / int4 / int6 weights)",
                "data": "synthetic",
                "config": {"workload": "float_sweep_n1",
                           "shapes": ["%s %dx%d" % (FLOAT_NAME[dt], r, c) for dt, r, c in FLOAT_SHAPES],
                           "global_batch": world, "parallelism": "replicas x%d (weak)" % world,
                           "l2": "261 MB of weights per step > 126 MB L2"},
                "roofline": {"bound": "hbm", "achieved": round(total / (ms * 1e-3) / 1e9, 1), "peak": peak,
                             "unit": "GB/s", "frac": round(total / (ms * 1e-3) / 1e9 / peak, 4), "traffic": None,
                             "peak_source": peak_src, "kernel": "gemv_float_kernel",
                             "how": "weights + x + out of the 5 matvecs / replayed step time"},
                "e2e": {"value": round(total * world / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                        "h2d_bytes_per_step": sum(4 * c for _, _, c in FLOAT_SHAPES),
                        "d2h_bytes_per_step": sum(4 * r for _, r, _ in FLOAT_SHAPES),
                        "how": "per matrix: sg_memcpy_h2d of x from pinned host, sg_matvec_rows_float, "
                               "sg_memcpy_d2h of the output"},
                "cpu_baseline": cpu,
                "gpu_launches": len(FLOAT_SHAPES) * args.steps,
                "clocks": clk.summary()}
    if world > 1:
        dist.destroy_process_group()
    return line


TP_METRIC = "K-quant GEMV HBM GB/s, rows split over the GPUs with the gather fused in (Q4_K/Q6_K x Q8_K sweep)"


def run_gpu_tp(args, metric=None):
    """The sweep's matrices split by rows over the ranks (strong scaling): every
    rank holds its par_rows shard of all seven, and one sg_matvec_tp per
    matrix leaves the whole output on every rank (peer stores over NVLink,
    arrival counters; no NCCL call on the data path)."""
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200 import _lib
    from spindle_b200.tp import ShardedMatrix, TpGroup, matvec_tp

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    nvec = args.nvec
    gen = torch.Generator(device=dev).manual_seed(1000)  # the same full matrices on every rank
    grp = TpGroup(device=dev)
    shards, X, BUF = [], [], []
    for dt, r, c in SHAPES:
        wf = torch.randn(r, c, device=dev, generator=gen) * 0.02
        wq = sg.quantize_weights(dt, wf)
        del wf
        shards.append(ShardedMatrix(dt, wq, r, c, world, rank))
        del wq
        X.append(torch.randn(nvec, c, device=dev, generator=gen))
        BUF.append(grp.buffer(nvec, r))
    # A rank's shard of the sweep is 314 MB / N: from 4 GPUs on it fits in the
    # 126 MB L2, so the steps cycle through copies of the shards holding at
    # least 2.5x L2 per rank, and every matrix is read from HBM.
    import copy
    shard_bytes = sum(sh.w.numel() for sh in shards)
    ncopies = max(1, -(-int(2.5 * L2_BYTES) // shard_bytes)) if world > 1 else 1
    copies = [shards]
    for _ in range(1, ncopies):
        cs = []
        for sh in shards:
            sc = copy.copy(sh)
            sc.w = sh.w.clone()
            cs.append(sc)
        copies.append(cs)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    # One vector: the list form, as on one GPU: the activations' Q8_K images
    # (every rank, all of x) and one gemv_list_kernel launch over this rank's
    # seven shards into one local buffer, then one NCCL all-gather of those
    # buffers (the benchmark's row split followed by an all-gather): every rank
    # ends with every matrix's whole output, as rank-major shard blocks.  The
    # fused form (one sg_matvec_tp per matrix, the gather done by peer stores
    # in the GEMV kernel) is timed beside it.
    from spindle_b200.tp import ListTp, matvec_list_tp
    as_list = nvec == 1 and args.form == "list" and world > 1
    if as_list:
        lts = [ListTp(copies[c], world, dev) for c in range(ncopies)]
        XS = [X[k][0] for k in range(len(SHAPES))]
        IMGS = sg.q8k_images(XS)
        # the list form's rows equal the fused form's, bit for bit (checked once)
        for k in range(len(SHAPES)):
            matvec_tp(shards[k], X[k], grp, BUF[k], stream=stream)
        with torch.cuda.stream(stream):
            sg.q8k_images(XS, IMGS)
            matvec_list_tp(lts[0], IMGS)
        torch.cuda.synchronize()
        for k, got in enumerate(lts[0].outputs()):
            if not torch.equal(got.view(torch.int32), BUF[k].tensor.reshape(-1)[:got.numel()].view(torch.int32)):
                raise RuntimeError("list form and fused row-split GEMVs differ (matrix %d)" % k)

    def list_part(c=0):
        sg.q8k_images(XS, IMGS)
        matvec_list_tp(lts[c], IMGS, gather=False)

    def step(c=0):
        for k in range(len(SHAPES)):
            matvec_tp(copies[c][k], X[k], grp, BUF[k], stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = sg.lib()
    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        g_steps = []
        for c in range(ncopies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(c)
            g_steps.append(g)
        g_lists = []
        if as_list:
            for c in range(ncopies):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    list_part(c)
                g_lists.append(g)

        def run_steps(n, start=0):
            # the list form: the graph of images + list, then the collective
            # (issued eagerly on the same stream, never inside a graph)
            for i in range(start, start + n):
                if as_list:
                    g_lists[i % ncopies].replay()
                    lts[i % ncopies].gather()
                else:
                    g_steps[i % ncopies].replay()

        run_steps(args.warmup)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            run_steps(args.steps)
            e1.record(stream)
            e1.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        fused_ms = None
        if as_list:
            for i in range(args.warmup):
                g_steps[i % ncopies].replay()
            barrier()
            e0.record(stream)
            for i in range(args.steps):
                g_steps[i % ncopies].replay()
            e1.record(stream)
            e1.synchronize()
            barrier()
            fused_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        # e2e: the step's activations from pinned host in one copy, the seven
        # calls, the whole outputs back (every rank holds them; rank 0's count)
        xsz = [nvec * c for _, _, c in SHAPES]
        XC = torch.empty(sum(xsz), device=dev)
        h_x = torch.empty(sum(xsz), dtype=torch.float32).pin_memory()
        osz = [nvec * r for _, r, _ in SHAPES]
        h_o = torch.empty(sum(osz), dtype=torch.float32).pin_memory()
        XV, off = [], 0
        for k in range(len(SHAPES)):
            XV.append(XC[off:off + xsz[k]].view(nvec, -1))
            h_x[off:off + xsz[k]].copy_(X[k].reshape(-1).cpu())
            off += xsz[k]
        sp = C.c_void_p(stream.cuda_stream)

        if as_list:
            XE = [XV[k][0] for k in range(len(SHAPES))]
            IE = sg.q8k_images(XE)
            h_ga = torch.empty(lts[0].gathered.numel(), dtype=torch.float32).pin_memory()

        def e2e_step(c=0):
            _lib.check(lib.sg_memcpy_h2d(C.c_void_p(XC.data_ptr()), C.c_void_p(h_x.data_ptr()), h_x.numel() * 4,
                                         sp), "h2d")
            if as_list:
                sg.q8k_images(XE, IE)
                matvec_list_tp(lts[c], IE, gather=False)
                return
            o = 0
            for k in range(len(SHAPES)):
                matvec_tp(copies[c][k], XV[k], grp, BUF[k], stream=stream)
                _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_o.data_ptr() + 4 * o), C.c_void_p(BUF[k].tensor.data_ptr()),
                                             osz[k] * 4, sp), "d2h")
                o += osz[k]

        e2e_step()
        torch.cuda.synchronize()
        g_e2es = []
        for c in range(ncopies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                e2e_step(c)
            g_e2es.append(g)

        def run_e2e(n):
            # the list form: after the graph (inputs up, images, list), the
            # collective, then the gathered outputs back to the host
            for i in range(n):
                g_e2es[i % ncopies].replay()
                if as_list:
                    lt = lts[i % ncopies]
                    lt.gather()
                    _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_ga.data_ptr()), C.c_void_p(lt.gathered.data_ptr()),
                                                 lt.gathered.numel() * 4, sp), "d2h")

        run_e2e(args.warmup)
        barrier()
        reps = max(3, min(args.steps, 2000))
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        run_e2e(reps)
        b1.record(stream)
        b1.synchronize()
        barrier()
        e2e_ms = max_over_ranks(b0.elapsed_time(b1)) / reps
    sg.device_status()
    total = step_bytes(nvec)
    value = total / (ms * 1e-3) / 1e9
    peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    try:
        peak, peak_src = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"], "MEASURED_PEAKS.json hbm_gbs"
    except Exception:
        pass
    per_gpu = value / world
    nvl = sum(4 * nvec * (s.r1 - s.r0) * (world - 1) for s in shards)
    line = None
    if rank == 0:
        line = {"metric": metric or TP_METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8 x int4/int6 -> int32, fp32 epilogue", "data": "synthetic",
                "config": dict(config_block(args, world),
                               workload=("gemv_sweep_n%d" if metric else "gemv_tp_sweep_n%d") % nvec,
                               parallelism=("row-split x%d (strong): images + one list launch over the rank's "
                                            "shards, then one NCCL all-gather" % world) if as_list else
                               "row-split x%d (strong), gather fused (peer stores)" % world,
                               global_batch=nvec,
                               l2="%d copies of this rank's %.1f MB of shards, cycled step by step (%.0f MB > "
                                  "2.5 x the 126 MB L2): every matrix is read from HBM"
                                  % (ncopies, shard_bytes / 1e6, ncopies * shard_bytes / 1e6)),
                "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(per_gpu / peak, 4), "traffic": None, "peak_source": peak_src,
                             "kernel": "gemv_list_kernel over the rank's shards (+ NCCL all-gather)" if as_list
                             else "gemv_tiled_kernel (row-split, peer-store epilogue)",
                             "nvlink_bytes_out_per_rank": nvl,
                             "how": "per GPU: the step's algorithmic bytes / n_gpus / step time; the rows each rank "
                                    "sends over NVLink are nvlink_bytes_out_per_rank (770 GB/s measured per "
                                    "direction makes that term small next to HBM)"},
                "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                        "h2d_bytes_per_step": h_x.numel() * 4,
                        "d2h_bytes_per_step": (lts[0].gathered.numel() if as_list else h_o.numel()) * 4,
                        "how": ("every step: one sg_memcpy_h2d of all activations from pinned host, "
                                "sg_q8k_images, sg_matvec_list_q8k on the rank's shards, the NCCL all-gather, one "
                                "sg_memcpy_d2h of the gathered outputs") if as_list else
                               ("every step: one sg_memcpy_h2d of all activations from pinned host, sg_matvec_tp per "
                                "matrix, sg_memcpy_d2h of each whole output")},
                "fused_row_split": {"us": round(fused_ms * 1e3, 2), "GB_s": round(total / (fused_ms * 1e-3) / 1e9, 1),
                                    "how": "the same sweep as one sg_matvec_tp per matrix (gather fused by peer "
                                           "stores, no NCCL call), replayed; its rows checked equal to the list "
                                           "form's"} if fused_ms else None,
                "gpu_launches": (2 if as_list else len(SHAPES)) * args.steps,
                "clocks": clk.summary()}
    del g_steps, g_e2es, g, g_lists
    grp.close()
    if world > 1:
        dist.destroy_process_group()
    return line


DECODE_MODELS = {
    "qwen3_30b_a3b": dict(dim=2048, n_heads=32, n_kv_heads=4, head_dim=128, n_layers=48, vocab=151936,
                          rope_theta=1e6, rms_eps=1e-6, rope_neox=True,
                          moe=dict(n_expert=128, n_used=8, n_ff=768, norm=True)),
    "qwen3_0_6b": dict(dim=1024, n_heads=16, n_kv_heads=8, head_dim=128, n_layers=28, vocab=151936,
                       rope_theta=1e6, rms_eps=1e-6, rope_neox=True, n_ff=3072),
}
PROMPT = 64


def decode_bytes(cfg, n_chosen_per_layer=None):
    """Algorithmic bytes of one token: every weight the step reads (attention,
    router and the chosen experts, or the dense FFN, per layer; the LM head;
    one embedding row), plus the KV cache rows it reads are left out (they are
    small next to the weights at these lengths)."""
    d, hd = cfg["dim"], cfg["head_dim"]
    q, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    blk = lambda dt, rows, cols: rows * (cols // 256) * BLK[dt]
    attn = blk(Q4_K, q, d) + blk(Q4_K, kv, d) + blk(Q6_K, kv, d) + blk(Q4_K, d, q)
    if cfg.get("moe"):
        m = cfg["moe"]
        expert = 2 * blk(Q4_K, m["n_ff"], d) + blk(Q6_K, d, m["n_ff"])
        ffn = m["n_expert"] * d * 4 + m["n_used"] * expert
    else:
        ffn = 2 * blk(Q4_K, cfg["n_ff"], d) + blk(Q6_K, d, cfg["n_ff"])
    return cfg["n_layers"] * (attn + ffn + 2 * d * 4) + blk(Q6_K, cfg["vocab"], d) + blk(Q4_K, 1, d) + d * 4


def decode_config(name, cfg, world):
    return {"workload": "decode_%s" % name, "model": name, "layers": cfg["n_layers"], "dim": cfg["dim"],
            "heads": "%d/%d x %d" % (cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]),
            "ffn": ("%d experts top %d, FFN %d" % (cfg["moe"]["n_expert"], cfg["moe"]["n_used"], cfg["moe"]["n_ff"])
                    if cfg.get("moe") else "dense FFN %d" % cfg["n_ff"]),
            "vocab": cfg["vocab"], "quant": "Q4_K_M mix: Q4_K, Q6_K attn_v / ffn_down / head, Q4_K embedding",
            "prompt": PROMPT, "global_batch": 1, "seq_len": PROMPT,
            "parallelism": ("single GPU" if world == 1 else "expert-parallel x%d: %d experts per GPU, router, "
                            "attention and LM head replicated, slot outputs exchanged over NVLink" %
                            (world, cfg["moe"]["n_expert"] // world if cfg.get("moe") else 0)),
            "weights": "random-init N(0,0.02), router N(0,1/dim), norms 1, seeded",
            "l2": "2.0 GB (30B) / 0.4 GB (0.6B) of weights per token > 126 MB L2"}


def run_gpu_decode(args):
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200 import _lib
    from spindle_b200.decoder import Decoder, qwen3_dtypes, random_weights

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    name = args.model
    cfg = dict(DECODE_MODELS[name], max_seq=PROMPT + args.warmup + args.steps + 8)
    if args.profile:
        # profiling case: the model's first two layers, the state set straight to
        # position PROMPT (no prompt pass), then the captured step replayed
        cfg["n_layers"] = 2
    dtypes = qwen3_dtypes(cfg, embed=Q4_K)
    if args.gguf:
        # a model file (a real Q4_K_M GGUF, or one made by spindle_b200.gguf.write_model)
        from spindle_b200 import gguf
        gf = gguf.GgufFile(args.gguf)
        cfg = dict(gguf.model_config(gf), max_seq=PROMPT + args.warmup + args.steps + 8)
        name = "gguf:" + os.path.basename(args.gguf)
        W, dtypes = gguf.load_weights(gf, cfg, dev)
    else:
        # the same model on every rank: N > 1 decodes one stream expert-parallel
        W = random_weights(cfg, dtypes, dev, seed=5000)
    host = None
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        # two layers' GGUF bytes plus embedding and head, for the CPU baseline
        keep = ["embed", "head", "out_norm"] + [k for k in W if k.startswith("l0.") or k.startswith("l1.")]
        host = {k: W[k].cpu().numpy() for k in keep}
    grp = None
    if world > 1 and cfg.get("moe"):
        from spindle_b200.tp import TpGroup
        grp = TpGroup(device=dev)
    elif world > 1:
        raise SystemExit("decode over several GPUs is expert-parallel: choose an MoE model")
    dec = Decoder(cfg, W, dtypes, dev, ep=grp)
    del W
    torch.cuda.synchronize()
    if args.profile:
        dec.set_state(5, PROMPT)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            dec.step(stream=s, hidden=False, logits=False)
            dec.set_state(5, PROMPT)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                dec.step(stream=s, hidden=False, logits=False)
            for _ in range(args.warmup + args.steps):
                graph.replay()
            torch.cuda.synchronize()
        sg.device_status()
        if rank == 0:
            print(json.dumps({"profile": True, "workload": "decode_%s_2_layers" % name, "pos": PROMPT}), flush=True)
        return None, None, cfg, dtypes
    g = torch.Generator().manual_seed(77)
    prompt = torch.randint(0, cfg["vocab"], (PROMPT,), generator=g).tolist()
    for i, t in enumerate(prompt):
        dec.set_state(t, i)
        dec.step(hidden=False, logits=False)
    torch.cuda.synchronize()
    lib = sg.lib()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            dec.step(stream=s, hidden=False, logits=False)
        for _ in range(args.warmup):
            graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(s)
            for _ in range(args.steps):
                graph.replay()
            e1.record(s)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        pos_after = int(dec.state[1].item())
        # e2e: the host feeds each token (pinned h2d) and reads the greedy token
        # back (d2h) every step, then continues from it
        h_state = torch.zeros(2, dtype=torch.int32).pin_memory()
        h_tok = torch.zeros(1, dtype=torch.int64).pin_memory()
        sp = C.c_void_p(s.cuda_stream)
        n_e2e = min(16, cfg["max_seq"] - pos_after - 1)
        h_state[0], h_state[1] = int(dec.state[0].item()), pos_after
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(s)
        for _ in range(n_e2e):
            _lib.check(lib.sg_memcpy_h2d(C.c_void_p(dec.state.data_ptr()), C.c_void_p(h_state.data_ptr()), 8, sp), "h2d")
            graph.replay()
            _lib.check(lib.sg_memcpy_d2h(C.c_void_p(h_tok.data_ptr()), C.c_void_p(dec.token.data_ptr()), 8, sp), "d2h")
            s.synchronize()
            h_state[0], h_state[1] = int(h_tok[0]), int(h_state[1]) + 1
        b1.record(s)
        b1.synchronize()
        e2e_ms = b0.elapsed_time(b1) / max(n_e2e, 1)
    sg.device_status()
    bytes_tok = decode_bytes(cfg)
    value = 1e3 / ms  # one stream; with N > 1 its experts spread over the GPUs
    peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    try:
        peak, peak_src = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"], "MEASURED_PEAKS.json hbm_gbs"
    except Exception:
        pass
    launches = 1 + cfg["n_layers"] * (8 + (4 if cfg.get("moe") else 2)) + 3
    line = None
    if rank == 0:
        achieved = bytes_tok / (ms * 1e-3) / 1e9
        line = {"metric": "decode tokens/s, %s (random-init, Q4_K_M mix), greedy" % name, "value": round(value, 2),
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "int8 x int4/int6 -> int32 GEMVs, fp32 norms/attention/router, f16 KV", "data": "synthetic",
                "config": decode_config(name, cfg, world),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                             "kernel": "the whole decode step (%d launches)" % launches,
                             "how": "algorithmic weight bytes per token (%.3f GB) x tokens/s" % (bytes_tok / 1e9)},
                "e2e": {"value": round(1e3 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                        "how": "per token: sg_memcpy_h2d of {token, pos} from pinned host, the step, sg_memcpy_d2h "
                               "of the greedy token, host sync (%d tokens)" % n_e2e},
                "gpu_launches": launches * args.steps,
                "clocks": clk.summary()}
    if world > 1:
        dist.barrier()
        del graph, dec
        if grp is not None:
            grp.close()
        dist.destroy_process_group()
    return line, host, cfg, dtypes


# ---- prefill + verify workload (--workload prefill) ---------------------------
# BASELINE configs[4] on the configs[3] model: a 2048-token random-ID prompt
# fed through the batch forward (feed, smollm_chat.rs:3042-3106: chunks of
# positions, K/V rows into the caches, hidden states only), the greedy token of
# its last position, then N=9 verify passes (forward_batch + compute_logits_batch)
# at the positions after it.  One step = the whole 2048-token prefill.

PREFILL_PROMPT = 2048
PREFILL_CHUNK = 128  # feed's chunk (smollm_chat.rs:3090); --chunk overrides
PREFILL_IN_FLIGHT = 6  # chunks in flight on as many streams; --overlap overrides
VERIFY_N = 9
SPEC_TOKENS = 64


def active_params(cfg):
    """Weights one token multiplies through (attention, router, the chosen
    experts or the dense FFN) over all layers; the LM head is left out (the
    prefill runs it for one position)."""
    d, hd = cfg["dim"], cfg["head_dim"]
    q, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    attn = 2 * q * d + 2 * kv * d
    if cfg.get("moe"):
        m = cfg["moe"]
        ffn = m["n_expert"] * d + m["n_used"] * 3 * m["n_ff"] * d
    else:
        ffn = 3 * cfg["n_ff"] * d
    return cfg["n_layers"] * (attn + ffn)


def run_gpu_prefill_pipe(args):
    """BASELINE configs[4] at N > 1: the prompt's prefill pipelined over the
    GPUs as a layer split (the two-PC mode of docs/cluster.md, layers 0..24 /
    24..48 at N = 2; par_rows's split of the layers in general).  Stage p runs
    its layers on each chunk of positions and sends the residual to stage p+1
    over NVLink (PipeLink: epoch-tagged peer stores), so while stage p+1 works
    on chunk c stage p already runs chunk c+1 (feed's chunks,
    smollm_chat.rs:3047-3071); the last stage runs the head on the prompt's
    last position.  value = prompt tokens / max-over-ranks prefill time."""
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200.decoder import Decoder, qwen3_dtypes, random_weights
    from spindle_b200.tp import PipeLink, TpGroup, shard_rows

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    name = "qwen3_30b_a3b"
    n_prompt = args.prompt if args.prompt else PREFILL_PROMPT
    cfg = dict(DECODE_MODELS[name], max_seq=n_prompt + 8)
    dtypes = qwen3_dtypes(cfg, embed=Q4_K)
    W = random_weights(cfg, dtypes, dev, seed=5000)  # the same model on every rank
    dec = Decoder(cfg, W, dtypes, dev)
    del W
    grp = TpGroup(device=dev)
    C_ = args.chunk or PREFILL_CHUNK
    links = [PipeLink(grp, p, p + 1, C_ * cfg["dim"]) for p in range(world - 1)]
    l0, l1 = shard_rows(cfg["n_layers"], world, rank)
    g = torch.Generator().manual_seed(78)
    toks = torch.randint(0, cfg["vocab"], (n_prompt,), generator=g).tolist()
    calls = [(c0, min(C_, n_prompt - 1 - c0)) for c0 in range(0, n_prompt - 1, C_)] + [(n_prompt - 1, 1)]
    s = torch.cuda.Stream(device=dev)
    hbuf = torch.empty(C_, cfg["dim"], device=dev)

    def prefill():
        greedy = None
        for i, (c0, n) in enumerate(calls):
            head = i == len(calls) - 1
            if rank == 0:
                out = dec.forward_batch_range(c0, l0, l1, tokens=toks[c0:c0 + n], n_max=C_, stream=s)
            else:
                h = links[rank - 1].recv(hbuf[:n], stream=s)
                out = dec.forward_batch_range(c0, l0, l1, hidden=h, n_max=C_, stream=s, head=head)
            if rank < world - 1:
                links[rank].send(out[0], stream=s)
            elif head:
                greedy = out[1]
        return greedy

    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            prefill()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(s)
            for _ in range(args.steps):
                prefill()
            e1.record(s)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sg.device_status()
    ops = 2.0 * n_prompt * active_params(cfg)
    peak, peak_src = 2 * 1596.4, "fallback: 2 x bf16 burst"
    try:
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak, peak_src = 2 * pk["bf16_tflops"], "2 x MEASURED_PEAKS.json bf16_tflops (dense int8 = 2 x bf16 on B200)"
    except Exception:
        pass
    line = None
    if rank == 0:
        achieved = ops / (ms * 1e-3) / 1e12
        line = {"metric": "prefill tokens/s, %s (random-init, Q4_K_M mix), %d-token prompt" % (name, n_prompt),
                "value": round(n_prompt / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "Q4_K projections: exact-integer f16 x f16 -> f32 on tcgen05; Q6_K and the MoE experts: int8 x int6/int4 -> int32 (dp4a); fp32 norms/attention/router, f16 KV",
                "data": "synthetic",
                "config": dict(decode_config(name, cfg, world), workload="prefill_pipeline_%s" % name,
                               prompt=n_prompt, seq_len=n_prompt, chunk=C_,
                               parallelism="layer pipeline x%d: layers %s, the residual of every %d-position "
                                           "chunk sent over NVLink (PipeLink)"
                                           % (world, ", ".join("%d..%d" % shard_rows(cfg["n_layers"], world, q)
                                                                for q in range(world)), C_)),
                "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": peak * world, "unit": "TOP/s",
                             "frac": round(achieved / (peak * world), 5), "traffic": None,
                             "peak_source": peak_src + ", x n_gpus",
                             "kernel": "the whole pipelined prefill",
                             "how": "2 x prompt x active params (%.3f G) / max-over-ranks step time"
                                    % (active_params(cfg) / 1e9)},
                "e2e": {"value": round(n_prompt / (ms * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0, "how": "the device-timed value (tokens are host lists passed per call)"},
                "gpu_launches": len(calls) * (1 + (l1 - l0) * 12) * args.steps,
                "clocks": clk.summary()}
    dist.barrier()
    del dec
    grp.close()
    dist.destroy_process_group()
    return line


def run_gpu_prefill(args):
    import torch
    import torch.distributed as dist

    import spindle_b200 as sg
    from spindle_b200 import _lib
    from spindle_b200.decoder import Decoder, _sigs, qwen3_dtypes, random_weights

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    name = "qwen3_30b_a3b"
    n_prompt = args.prompt if args.prompt else (128 if args.profile else PREFILL_PROMPT)
    cfg = dict(DECODE_MODELS[name], max_seq=n_prompt + SPEC_TOKENS + 2 * VERIFY_N + 8)
    if args.profile:
        cfg["n_layers"] = 2  # profiling case: the model's first two layers, two chunks
    dtypes = qwen3_dtypes(cfg, embed=Q4_K)
    W = random_weights(cfg, dtypes, dev, seed=5000 + rank)
    dec = Decoder(cfg, W, dtypes, dev)
    del W
    L = _sigs()
    lib = sg.lib()
    C_ = args.chunk or PREFILL_CHUNK
    nbytes = L.sg_model_batch_scratch_bytes(C.byref(dec.model), C_)
    scr = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _lib.check(L.sg_model_batch_prepare(C.byref(dec.model), C_, C.c_void_p(scr.data_ptr()), nbytes, None), "prepare")
    g = torch.Generator().manual_seed(78 + rank)
    h_tok = torch.randint(0, cfg["vocab"], (n_prompt + VERIFY_N,), generator=g, dtype=torch.int32).pin_memory()
    # calls: full chunks without the head, then the last position alone with it
    calls = [(c0, min(C_, n_prompt - 1 - c0)) for c0 in range(0, n_prompt - 1, C_)] + [(n_prompt - 1, 1)]
    h_pos = torch.tensor([c0 for c0, _ in calls] + [n_prompt], dtype=torch.int32).pin_memory()
    toks = h_tok.to(dev)
    pos = h_pos.to(dev)
    hid = torch.empty(C_, cfg["dim"], dtype=torch.float32, device=dev)
    greedy = torch.empty(C_, dtype=torch.int64, device=dev)
    vlog = torch.empty(VERIFY_N, cfg["vocab"], dtype=torch.float32, device=dev)
    vgreedy = torch.empty(VERIFY_N, dtype=torch.int64, device=dev)
    nl = cfg["n_layers"]
    ptr = lambda t, off=0: C.c_void_p(t.data_ptr() + off)

    # chunks in flight: chunk i a layer at a time on stream i % K with its
    # own scratch, its layer l after chunk i - 1's layer l (K = 1: one call
    # per chunk on one stream)
    K_ = max(1, args.overlap)
    bufs = [scr] + [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(K_ - 1)]
    for b in bufs[1:]:
        _lib.check(L.sg_model_batch_prepare(C.byref(dec.model), C_, C.c_void_p(b.data_ptr()), nbytes, None), "prepare")
    side = [torch.cuda.Stream(device=dev) for _ in range(K_ - 1)]

    def prefill_overlapped(st):
        sts, prev = [st] + side, None
        for si in side:
            si.wait_stream(st)
        for i, (c0, n) in enumerate(calls[:-1]):
            si, bi, evs = sts[i % K_], bufs[i % K_], []
            for l in range(nl):
                if prev is not None:
                    si.wait_event(prev[l])
                _lib.check(L.sg_forward_batch_range(C.byref(dec.model), l, l + 1, ptr(toks, 4 * c0) if l == 0 else None,
                                                    None, n, ptr(pos, 4 * i), ptr(dec.kv), ptr(bi), nbytes, C_,
                                                    ptr(hid) if l == nl - 1 else None, None, cfg["vocab"], None,
                                                    C.c_void_p(si.cuda_stream)), "prefill")
                ev = torch.cuda.Event()
                ev.record(si)
                evs.append(ev)
            prev = evs
        for si in side:
            st.wait_stream(si)
        i, (c0, n) = len(calls) - 1, calls[-1]
        _lib.check(L.sg_forward_batch_range(C.byref(dec.model), 0, nl, ptr(toks, 4 * c0), None, n, ptr(pos, 4 * i),
                                            ptr(dec.kv), ptr(scr), nbytes, C_, None, None, cfg["vocab"], ptr(greedy),
                                            C.c_void_p(st.cuda_stream)), "prefill")

    def prefill(st):
        if K_ > 1:
            return prefill_overlapped(st)
        sp = C.c_void_p(st.cuda_stream)
        for i, (c0, n) in enumerate(calls):
            head = i == len(calls) - 1
            _lib.check(L.sg_forward_batch_range(C.byref(dec.model), 0, nl, ptr(toks, 4 * c0), None, n,
                                                ptr(pos, 4 * i), ptr(dec.kv), ptr(scr), nbytes, C_,
                                                None if head else ptr(hid), None, cfg["vocab"],
                                                ptr(greedy) if head else None, sp), "prefill")

    def verify(st):
        _lib.check(L.sg_forward_batch(C.byref(dec.model), ptr(toks, 4 * n_prompt), VERIFY_N, ptr(pos, 4 * len(calls)),
                                      ptr(dec.kv), ptr(scr), nbytes, C_, ptr(vlog), cfg["vocab"], ptr(vgreedy),
                                      C.c_void_p(st.cuda_stream)), "verify")

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        prefill(s)
        verify(s)
        torch.cuda.synchronize()
        gp = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gp, stream=s):
            prefill(s)
        gv = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gv, stream=s):
            verify(s)
        if args.profile:
            for _ in range(args.warmup + args.steps):
                gp.replay()
                gv.replay()
            torch.cuda.synchronize()
            sg.device_status()
            if rank == 0:
                print(json.dumps({"profile": True, "workload": "prefill_%s_2_layers" % name, "prompt": n_prompt}),
                      flush=True)
            return None
        for _ in range(args.warmup):
            gp.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(s)
            for _ in range(args.steps):
                gp.replay()
            e1.record(s)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        # verify passes at positions n_prompt .. n_prompt + 8 (rewritten each pass)
        for _ in range(3):
            gv.replay()
        v0, v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nv = 20
        v0.record(s)
        for _ in range(nv):
            gv.replay()
        v1.record(s)
        v1.synchronize()
        v_ms = v0.elapsed_time(v1) / nv
        # e2e: prompt tokens and chunk positions from pinned host memory, the
        # prefill, the greedy next token back to the host
        h_out = torch.zeros(1, dtype=torch.int64).pin_memory()
        sp = C.c_void_p(s.cuda_stream)
        tok_bytes, pos_bytes = 4 * (n_prompt + VERIFY_N), 4 * (len(calls) + 1)

        def e2e():
            _lib.check(lib.sg_memcpy_h2d(ptr(toks), ptr(h_tok), tok_bytes, sp), "h2d")
            _lib.check(lib.sg_memcpy_h2d(ptr(pos), ptr(h_pos), pos_bytes, sp), "h2d")
            gp.replay()
            _lib.check(lib.sg_memcpy_d2h(ptr(h_out), ptr(greedy), 8, sp), "d2h")

        e2e()
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(1, min(3, args.steps))
        b0.record(s)
        for _ in range(n_e2e):
            e2e()
        b1.record(s)
        b1.synchronize()
        e2e_ms = b0.elapsed_time(b1) / n_e2e
        # speculative decode after the prompt (the rest of configs[4]): SPEC_TOKENS
        # tokens with drafts of 8 whose first A tokens are the model's own
        # continuation (A uniform in 0..k, seeded: 50% of drafted tokens right
        # on average), the rest wrong; against the same tokens one position
        # per call through the same batch path.  Host-driven loops, timed by
        # the wall clock with a device sync on both sides.
        from spindle_b200.spec import speculative_decode
        torch.cuda.synchronize()
        tok0, p_ = int(greedy[0].item()), n_prompt
        want, t_ = [], tok0
        t0 = time.perf_counter()
        for _ in range(SPEC_TOKENS):
            want.append(t_)
            _, g1 = dec.forward_batch([t_], p_, logits=False, n_max=C_)
            t_, p_ = int(g1[0].item()), p_ + 1
        torch.cuda.synchronize()
        plain_s = time.perf_counter() - t0
        rs = __import__("numpy").random.default_rng(1234 + rank)

        def drafter(ctx, k):
            m = len(ctx) - n_prompt          # tokens generated so far (the pending one included)
            right = want[m:m + k]
            a = int(rs.integers(0, len(right) + 1))
            return right[:a] + [(t + 1) % cfg["vocab"] for t in right[a:]]

        st = {}
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        got = speculative_decode(dec, tok0, n_prompt, SPEC_TOKENS, h_tok[:n_prompt].tolist(), draft_len=8,
                                 drafter=drafter, n_max=C_, stats=st)
        torch.cuda.synchronize()
        spec_s = time.perf_counter() - t0
        spec = {"tokens": SPEC_TOKENS, "positions": "%d..%d" % (n_prompt, n_prompt + SPEC_TOKENS - 1),
                "tok_per_s": round(SPEC_TOKENS / spec_s, 1), "plain_tok_per_s": round(SPEC_TOKENS / plain_s, 1),
                "passes": st["passes"], "single_steps": st["steps"],
                "accept_rate": round(st["accepted"] / max(st["drafted"], 1), 3),
                "identical_to_plain": got == want,
                "how": "spindle_b200.spec.speculative_decode (drafts of 8, verify passes through sg_forward_batch) "
                       "vs one position per sg_forward_batch call; wall clock, host-synchronous loops"}
        if world > 1:
            t = torch.tensor([ms, v_ms, e2e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, v_ms, e2e_ms = float(t[0]), float(t[1]), float(t[2])
    sg.device_status()
    ops = 2.0 * n_prompt * active_params(cfg)
    peak, peak_src = 2 * 1596.4, "fallback: 2 x bf16 burst"
    try:
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak, peak_src = 2 * pk["bf16_tflops"], "2 x MEASURED_PEAKS.json bf16_tflops (dense int8 = 2 x bf16 on B200)"
    except Exception:
        pass
    line = None
    if rank == 0:
        achieved = ops / (ms * 1e-3) / 1e12
        line = {"metric": "prefill tokens/s, %s (random-init, Q4_K_M mix), %d-token prompt" % (name, n_prompt),
                "value": round(n_prompt * world / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "Q4_K projections: exact-integer f16 x f16 -> f32 on tcgen05; Q6_K and the MoE experts: int8 x int6/int4 -> int32 (dp4a); fp32 norms/attention/router, f16 KV",
                "data": "synthetic",
                "config": dict(decode_config(name, cfg, world), workload="prefill_verify_%s" % name,
                               prompt=n_prompt, seq_len=n_prompt, chunk=C_, verify_n=VERIFY_N,
                               calls="%d chunks of up to %d positions without the head, then the last position "
                                     "with the LM head and argmax" % (len(calls) - 1, C_),
                               in_flight="%d chunks on %d streams, a layer at a time" % (K_, K_) if K_ > 1
                               else "1 (one call per chunk)",
                               l2="2.0 GB of weights touched per chunk > 126 MB L2"),
                "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": peak, "unit": "TOP/s",
                             "frac": round(achieved / peak, 5), "traffic": None, "peak_source": peak_src,
                             "kernel": "the whole prefill (Q4_K projections on tcgen05 kind::f16, the rest dp4a)",
                             "how": "2 x prompt x active params (%.3f G) / step time" % (active_params(cfg) / 1e9)},
                "verify": {"n": VERIFY_N, "ms_per_pass": round(v_ms, 3),
                           "tok_per_s_if_all_accepted": round(VERIFY_N * 1e3 / v_ms, 1),
                           "tok_per_s_at_half_acceptance": round((1 + (VERIFY_N - 1) // 2) * 1e3 / v_ms, 1),
                           "how": "forward_batch + LM head + argmax for 9 positions after the prompt, graph replays"},
                "spec_decode": spec,
                "e2e": {"value": round(n_prompt * world / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                        "h2d_bytes_per_step": tok_bytes + pos_bytes, "d2h_bytes_per_step": 8,
                        "how": "sg_memcpy_h2d of the prompt tokens and chunk positions from pinned host, the "
                               "prefill, sg_memcpy_d2h of the greedy next token (%d steps)" % n_e2e},
                "gpu_launches": len(calls) * (1 + nl * 12) * args.steps,
                "clocks": clk.summary()}
    if world > 1:
        dist.barrier()
        del gp, gv
        dist.destroy_process_group()
    return line


def decode_cpu_sample(cfg, dtypes, host, budget_s):
    """Per-token time of the oracle's forward_slice (one thread), measured on a
    two-layer model made of the real model's first two layers, embedding and
    head, and scaled: 2-layer time minus the head's, times layers / 2, plus the
    head's."""
    import numpy as np
    import oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import decoder_util as U
    c2 = dict(cfg, n_layers=2, max_seq=64)
    d2 = {k: v for k, v in dtypes.items() if not k.startswith("l") or k.split(".")[0] in ("l0", "l1")}
    D = U.oracle_decoder(c2, d2, host)
    hd_buf = np.ascontiguousarray(host["head"])
    head = O.Mat(dtypes["head"], cfg["dim"], cfg["vocab"], 0)
    xq = np.random.default_rng(3).standard_normal(cfg["dim"], dtype=np.float32)
    # the head's share: its integer matvec (Q8_K quantize + rows) on one thread
    O.pool_create(1)
    try:
        logits = np.empty((1, cfg["vocab"]), np.float32)
        t0 = time.perf_counter()
        n_h = 0
        while True:
            O.pool_matvec_multi(hd_buf, head, xq.reshape(1, -1), logits)
            n_h += 1
            if time.perf_counter() - t0 > 0.2 * budget_s:
                break
        t_head = (time.perf_counter() - t0) / n_h
    finally:
        O.pool_destroy()
    t0 = time.perf_counter()
    n = 0
    while n < c2["max_seq"]:
        D.forward(n % 1000, n)
        n += 1
        if time.perf_counter() - t0 > 0.8 * budget_s:
            break
    t2 = (time.perf_counter() - t0) / n
    per_tok = (t2 - t_head) * cfg["n_layers"] / 2 + t_head
    return per_tok, n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--nvec", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layout", default="tiled", choices=["tiled", "gguf"],
                    help="weight layout on the device: TILED16 (repacked at upload) or GGUF rows")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU-baseline work (rank 0, N=1)")
    ap.add_argument("--shape", type=int, default=None, help="profiling: run only this sweep entry")
    ap.add_argument("--profile", action="store_true",
                    help="profiling: only the timed step loop (no e2e, per-shape or CPU legs)")
    ap.add_argument("--workload", default="gemv", choices=["gemv", "gemv_tp", "float", "moe", "decode", "prefill"],
                    help="gemv: the headline K-quant GEMV sweep; gemv_tp: the same sweep split by rows over the "
                         "GPUs with the gather fused in; float: the float-path matvecs; moe: the Qwen3-30B-A3B "
                         "MoE layer; decode: greedy decode of a whole random-init model; prefill: a 2048-token prompt "
                         "through the batch forward, then N=9 verify passes")
    ap.add_argument("--prompt", type=int, default=0,
                    help="prefill workload: prompt length (default 2048; 128 with --profile)")
    ap.add_argument("--model", default="qwen3_30b_a3b", choices=sorted(DECODE_MODELS),
                    help="decode workload: the model architecture")
    ap.add_argument("--gguf", default=None, help="decode workload: load the model from this GGUF file instead")
    ap.add_argument("--chunk", type=int, default=0, help="prefill workload: positions per batch call (default 128)")
    ap.add_argument("--form", default="list", choices=["list", "per-matrix"],
                    help="gemv workload, one vector on TILED16: the 7 GEMVs as one list launch (after one Q8_K "
                         "image launch) or one sg_matvec launch per matrix"),
    ap.add_argument("--overlap", type=int, default=PREFILL_IN_FLIGHT,
                    help="prefill workload: chunks in flight on as many streams, a layer at a time (1: one call per "
                         "chunk on one stream)"),
    args = ap.parse_args()
    if args.warmup < 3 and not args.profile:
        args.warmup = 3
    if args.workload == "decode":
        if args.steps == 20000:
            args.steps = 128  # the BASELINE workload's 128 greedy tokens
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "decode reference arm: use the cpu_baseline of the "
                              "GPU line (the oracle forward on two real layers, scaled)"}), flush=True)
            return
        line, host, cfg, dtypes = run_gpu_decode(args)
        rank, world, _ = rank_env()
        if rank == 0 and line is not None:
            if host is not None:
                per_tok, n = decode_cpu_sample(cfg, dtypes, host, args.cpu_budget)
                line["cpu_baseline"] = {"value": round(1.0 / per_tok, 3), "unit": "tok/s", "cores": 1, "kind": "port", "cpu_model": cpu_model(),
                                        "sample": "the oracle's forward_slice (one thread) on the model's first 2 "
                                                  "layers + embedding + head, %d tokens; per-token time = "
                                                  "(2-layer time - head time) x %d / 2 + head time"
                                                  % (n, cfg["n_layers"])}
            print(json.dumps(line), flush=True)
        return
    if args.workload == "prefill":
        if args.steps == 20000:
            args.steps = 3  # one step is a whole 2048-token prompt
        if args.warmup == 20:
            args.warmup = 3
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "prefill reference arm: the oracle forward runs "
                              "about 1 token/s on one core; the decode line's cpu_baseline covers it"}), flush=True)
            return
        line = run_gpu_prefill_pipe(args) if rank_env()[1] > 1 else run_gpu_prefill(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if args.workload == "moe":
        if args.steps == 20000:
            args.steps = 2000  # one step is 8 token-layers
        if args.impl == "reference":
            run_reference_moe(args)
            return
        line, host0 = run_gpu_moe(args)
        rank, world, _ = rank_env()
        if rank == 0 and line is not None:
            if world == 1 and args.cpu_budget > 0:
                per_layer, gbs, n = moe_cpu_sample([host0], args.cpu_budget)
                line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port", "cpu_model": cpu_model(),
                                        "sample": "%d token-layers through the oracle's moe_forward (same layer "
                                                  "shape, host-quantized weights), one thread, %.1f s"
                                                  % (n, per_layer * n)}
            print(json.dumps(line), flush=True)
        return
    if args.workload == "float":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "float reference arm: use the cpu_baseline of the "
                              "GPU line (the oracle's float kernels on a bounded sample)"}), flush=True)
            return
        line = run_float(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if args.shape is not None:
        SHAPES[:] = [SHAPES[args.shape]]
    if args.impl == "reference":
        run_reference(args)
        return
    rank, world, _ = rank_env()
    if args.workload == "gemv_tp" or world > 1:
        # N > 1: the headline sweep row-split over the GPUs (strong scaling)
        line = run_gpu_tp(args, metric=METRIC if args.workload == "gemv" else None)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    line, W = run_gpu(args)
    rank, world, _ = rank_env()
    if args.profile:
        return
    if rank == 0 and line is not None:
        if world == 1 and args.cpu_budget > 0:
            wh = [w.cpu().numpy() for w in W]
            threads = os.cpu_count() or 1
            sweep_s, n = cpu_sample(wh, args.nvec, args.cpu_budget, threads)
            cpu_v = step_bytes(args.nvec) / sweep_s / 1e9
            line["cpu_baseline"] = {"value": round(cpu_v, 2), "unit": "GB/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                                    "sample": "%d full sweeps (same 7 matrices, same bytes) through the oracle's "
                                              "pooled matvec, %.1f s" % (n, sweep_s * n)}
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
