"""The MoE layer on the GPU (sg_moe_forward) against the oracle's moe_forward.

Router logits, top-k, prune and weights follow moe_forward (smollm_chat.rs:
1178-1240); the experts follow ffns_fused (:382-442) on the integer path.
Every step is restated operation for operation, exp included (the kernels
compute glibc's expf bit for bit, the function f32::exp calls), so the
probabilities, the chosen experts, the mixing weights and the outputs are
compared bit for bit.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

pytestmark = pytest.mark.gpu



def make_layer(seed, dim, ff, n_exp, k, gu_dt=O.Q4_K, dn_dt=O.Q6_K, shared_ff=0, shared_gate=False,
               router_scale=None):
    """Random GGUF expert tensors (the reference tests' random blocks) and an
    F32 router whose logits are about N(0, 1) for x in [-1, 1]."""
    rng = O.Rng(seed)
    a = router_scale if router_scale is not None else float(np.sqrt(3.0 / dim) * np.sqrt(3.0))
    router = rng.fill(-a, a, n_exp * dim)
    g = O.random_matrix(gu_dt, dim, ff * n_exp, rng)
    u = O.random_matrix(gu_dt, dim, ff * n_exp, rng)
    d = O.random_matrix(dn_dt, ff, dim * n_exp, rng)
    parts = [router.view(np.uint8), g, u, d]
    off = np.cumsum([0] + [p.nbytes for p in parts])
    L = dict(router=router, g=g, u=u, d=d, dim=dim, ff=ff, n_exp=n_exp, k=k, gu_dt=gu_dt, dn_dt=dn_dt,
             shared=None, sh_gate=None)
    moe = O.Moe(router=O.Mat(O.F32, dim, n_exp, 0), gate=O.Mat(gu_dt, dim, ff, int(off[1])),
                up=O.Mat(gu_dt, dim, ff, int(off[2])), down=O.Mat(dn_dt, ff, dim, int(off[3])), n_expert=n_exp,
                n_used=k, norm=1, moe_prune=0.0)
    if shared_ff:
        sg_ = O.random_matrix(gu_dt, dim, shared_ff, rng)
        su = O.random_matrix(gu_dt, dim, shared_ff, rng)
        sd = O.random_matrix(dn_dt, shared_ff, dim, rng)
        extra = [sg_, su, sd]
        base = int(off[-1])
        so = np.cumsum([base] + [p.nbytes for p in extra])
        parts += extra
        moe.has_shared = 1
        moe.sh_gate = O.Mat(gu_dt, dim, shared_ff, int(so[0]))
        moe.sh_up = O.Mat(gu_dt, dim, shared_ff, int(so[1]))
        moe.sh_down = O.Mat(dn_dt, shared_ff, dim, int(so[2]))
        L["shared"] = (sg_, su, sd, shared_ff)
        if shared_gate:
            gv = rng.fill(-0.05, 0.05, dim)
            moe.has_shared_gate = 1
            moe.shared_gate_offset = int(so[3])
            parts.append(gv.view(np.uint8))
            L["sh_gate"] = gv
    L["raw"] = np.concatenate(parts)
    L["moe"] = moe
    return L


def gpu_layer(L, dev, norm=True, prune=0.0):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    shared = None
    if L["shared"] is not None:
        sg_, su, sd, sff = L["shared"]
        shared = (t(sg_), t(su), t(sd), L["gu_dt"], L["dn_dt"], sff)
    return sg.Moe.pack(t(L["router"]), t(L["g"]), t(L["u"]), t(L["d"]), L["gu_dt"], L["dn_dt"], L["n_exp"], L["k"],
                       L["dim"], L["ff"], norm=norm, moe_prune=prune, shared=shared,
                       shared_gate=None if L["sh_gate"] is None else t(L["sh_gate"]))


def run_gpu(m, x, dev):
    choice = torch.zeros(36, dtype=torch.int32, device=dev)
    probs = torch.empty(m.n_expert, dtype=torch.float32, device=dev)
    out = sg.moe_forward(m, torch.from_numpy(x).to(dev), choice=choice, probs=probs)
    torch.cuda.synchronize()
    sg.device_status()
    ids, w = sg.decode_choice(choice)
    return out.cpu().numpy(), ids, np.array(w, np.float32), probs.cpu().numpy()


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), a).view(np.uint32)


def check_same(got, want, what):
    assert np.array_equal(bits(got), bits(want)), "%s: max err %g" % (
        what, float(np.nanmax(np.abs(np.asarray(got, np.float64) - want))) if np.size(want) else 0.0)


def compare(L, x, dev, norm=True, prune=0.0):
    moe = L["moe"]
    moe.norm, moe.moe_prune = int(norm), prune
    want, w_ids, w_w = O.moe_forward(L["raw"], moe, x)
    w_probs, _, _ = O.moe_route(L["raw"], moe, x)
    m = gpu_layer(L, dev, norm, prune)
    got, ids, w, probs = run_gpu(m, x, dev)
    check_same(probs, w_probs, "probabilities")
    assert ids == [int(e) for e in w_ids], (ids, list(w_ids))
    check_same(w, w_w, "weights")
    check_same(got, want, "moe output")
    return got, ids


@pytest.mark.parametrize("dim,ff,n_exp,k,gu,dn", [
    (512, 256, 16, 4, O.Q4_K, O.Q6_K),
    (1024, 512, 8, 2, O.Q4_K, O.Q4_K),    # Mixtral-like top-2 of 8
    (768, 1024, 64, 6, O.Q6_K, O.Q6_K),
    (256, 256, 4, 1, O.Q6_K, O.Q4_K),
    (256, 256, 100, 8, O.Q4_K, O.Q6_K),   # expert count not a multiple of 32
    (256, 256, 200, 16, O.Q4_K, O.Q6_K),  # most experts a token may use
    (256, 256, 300, 4, O.Q4_K, O.Q6_K),   # above 256 experts: the block-wide choice
])
def test_moe_matches_oracle(dev, dim, ff, n_exp, k, gu, dn):
    L = make_layer(dim + ff + n_exp, dim, ff, n_exp, k, gu, dn)
    x = O.Rng(99).fill(-1.0, 1.0, dim)
    compare(L, x, dev)
    compare(L, x, dev, norm=False)


def test_moe_qwen3_layer_full_size(dev):
    # the Qwen3-30B-A3B layer: 128 experts, top 8, dim 2048, FFN 768, Q4_K gate/up, Q6_K down
    L = make_layer(30, 2048, 768, 128, 8)
    rng = O.Rng(31)
    for _ in range(3):
        compare(L, rng.fill(-1.0, 1.0, 2048), dev)
    compare(L, rng.fill(-1.0, 1.0, 2048), dev, prune=4.0)


@pytest.mark.parametrize("prune", [0.5, 0.2, 4.0, 1.0, 9.0, 2.5])
def test_moe_prune(dev, prune):
    L = make_layer(5, 512, 256, 32, 8, router_scale=0.2)
    x = O.Rng(6).fill(-1.0, 1.0, 512)
    _, ids = compare(L, x, dev, prune=prune)
    if prune >= 1.0:
        assert len(ids) == min(max(int(prune), 4), 8)


@pytest.mark.parametrize("gate", [False, True])
def test_moe_shared_expert(dev, gate):
    # Qwen2-MoE: an always-on shared expert, optionally scaled by sigmoid(g . x)
    L = make_layer(77, 512, 256, 16, 4, shared_ff=768, shared_gate=gate)
    x = O.Rng(78).fill(-1.0, 1.0, 512)
    compare(L, x, dev)


def test_moe_pack_matches_stacked_repack(dev):
    # expert e of the packed gate/up buffer == TILED16 of gate_e and up_e
    # interleaved in groups of 8 rows (GGUF rows), and expert e of the packed
    # down buffer == TILED16 of down_e
    dim, ff, n_exp = 512, 40, 3
    rng = O.Rng(8)
    g = O.random_matrix(O.Q4_K, dim, ff * n_exp, rng)
    u = O.random_matrix(O.Q4_K, dim, ff * n_exp, rng)
    t = lambda a: torch.from_numpy(a).to(dev)
    stride = sg.tiled16_bytes(O.Q4_K, 2 * ff, dim)
    packed = torch.full((stride * n_exp,), 0xAB, dtype=torch.uint8, device=dev)
    gd, ud = t(g), t(u)  # keep the sources alive while the kernels run
    sg._lib.check(sg.lib().sg_moe_pack_gate_up(O.Q4_K, C.c_void_p(gd.data_ptr()), C.c_void_p(ud.data_ptr()),
                                               n_exp, ff, dim, C.c_void_p(packed.data_ptr()), None), "pack")
    rb = O.row_bytes(O.Q4_K, dim)
    for e in range(n_exp):
        ge = g[e * ff * rb:(e + 1) * ff * rb].reshape(ff // 8, 8 * rb)
        ue = u[e * ff * rb:(e + 1) * ff * rb].reshape(ff // 8, 8 * rb)
        stacked = np.concatenate([ge, ue], axis=1).reshape(-1)
        want, _ = sg.repack_tiled16(O.Q4_K, t(stacked), 2 * ff, dim)
        assert torch.equal(packed[e * stride:(e + 1) * stride], want), e
    rows, n_ff = 24, 512          # down: 24 rows (padding inside each expert), 512 cols
    d = O.random_matrix(O.Q6_K, n_ff, rows * n_exp, rng)
    dstride = sg.tiled16_bytes(O.Q6_K, rows, n_ff)
    dp = torch.full((dstride * n_exp,), 0xCD, dtype=torch.uint8, device=dev)
    dd = t(d)
    sg._lib.check(sg.lib().sg_moe_pack_down(O.Q6_K, C.c_void_p(dd.data_ptr()), n_exp, rows, n_ff,
                                            C.c_void_p(dp.data_ptr()), None), "pack_down")
    rbd = O.row_bytes(O.Q6_K, n_ff)
    for e in range(n_exp):
        want, _ = sg.repack_tiled16(O.Q6_K, t(d[e * rows * rbd:(e + 1) * rows * rbd]), rows, n_ff)
        assert torch.equal(dp[e * dstride:(e + 1) * dstride], want), e


def test_moe_graph_replay_and_scratch_choice(dev):
    # no state survives a call: repeated calls and CUDA-graph replays give the
    # same bits, with the choice kept in the scratch (no d_choice)
    L = make_layer(11, 1024, 512, 32, 4)
    m = gpu_layer(L, dev)
    x = torch.from_numpy(O.Rng(12).fill(-1.0, 1.0, 1024)).to(dev)
    scratch = torch.empty(m.scratch_bytes(), dtype=torch.uint8, device=dev)
    out = torch.empty(1024, dtype=torch.float32, device=dev)
    sg.moe_forward(m, x, out, scratch)
    first = out.clone()
    want, _, _ = O.moe_forward(L["raw"], L["moe"], x.cpu().numpy())
    check_same(first.cpu().numpy(), want, "scratch choice")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sg.moe_forward(m, x, out, scratch, stream=s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            sg.moe_forward(m, x, out, scratch, stream=s)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(5):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), first.view(torch.int32))
    sg.device_status()


def test_moe_nan_input(dev):
    # NaN x: every logit is NaN; all keys tie, so experts 0..k-1 are chosen
    L = make_layer(13, 256, 256, 8, 2)
    x = np.full(256, np.nan, np.float32)
    want, w_ids, _ = O.moe_forward(L["raw"], L["moe"], x)
    m = gpu_layer(L, dev)
    got, ids, w, _ = run_gpu(m, x, dev)
    assert ids == [int(e) for e in w_ids] == [0, 1]
    assert np.all(np.isnan(got)) and np.all(np.isnan(want))


def test_moe_bad_args(dev):
    L = make_layer(14, 256, 256, 8, 2)
    m = gpu_layer(L, dev)
    x = torch.zeros(256, dtype=torch.float32, device=dev)
    scratch = torch.empty(m.scratch_bytes(), dtype=torch.uint8, device=dev)
    lib = sg.lib()

    def status(mm, xx=x, sc=scratch, nbytes=None):
        out = torch.empty(256, dtype=torch.float32, device=dev)
        return lib.sg_moe_forward(C.byref(mm.c()), C.c_void_p(xx.data_ptr()), C.c_void_p(out.data_ptr()),
                                  C.c_void_p(sc.data_ptr()), sc.numel() if nbytes is None else nbytes, None, None,
                                  None)

    assert status(m) == 0
    torch.cuda.synchronize()
    assert status(m, nbytes=scratch.numel() - 1) == 1
    assert status(m, sc=scratch[16:]) == 4
    assert status(m, xx=x[1:]) == 4
    for field, val, code in [("n_used", 17, 1), ("n_used", 0, 1), ("dim", 300, 3), ("n_ff", 128, 3),
                             ("gate_up_dtype", O.Q8_0, 2), ("gate_up_stride", 16, 1)]:
        bad = sg.Moe(**dict(m.__dict__))
        setattr(bad, field, val)
        assert status(bad) == code, field
    many = sg.Moe(**dict(m.__dict__))
    many.n_expert, many.n_used = 64, 17
    assert status(many) == 3
    assert lib.sg_moe_scratch_bytes(None) == 0
    sg.device_status()
