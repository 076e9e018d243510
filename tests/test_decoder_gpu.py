"""The GPU decoder step (sg_forward) against the oracle's forward_slice.

Every fp32 operation of the step follows the reference's order on the GPU and
exp / sin / cos are glibc's expf / sinf / cosf bit for bit (the functions the
reference's f32::exp / sin_cos call, which the oracle calls too), so the
logits, the KV caches and the greedy tokens are equal bit for bit.
"""
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import decoder_util as U  # noqa: E402

import oracle as O  # noqa: E402
from spindle_b200.decoder import Decoder  # noqa: E402

pytestmark = pytest.mark.gpu

def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), a).view(np.uint32)


def run_pair(cfg, dtypes, seed, prompt, n_new, dev, qk_adjacent=True, W=None):
    """Token by token against the oracle (glibc's expf/sinf/cosf, as the
    reference): logits bit for bit, the same greedy tokens and device state.
    W: CUDA weights to use instead of seeded host ones."""
    if W is None:
        W = U.host_weights(cfg, dtypes, seed=seed)
        ref = U.oracle_decoder(cfg, dtypes, W)
        W = U.device_weights(W, dev)
    else:
        ref = U.oracle_decoder(cfg, dtypes, W)
    gpu = Decoder(cfg, W, dtypes, dev, qk_adjacent=qk_adjacent)
    toks_ref, toks_gpu = [], []
    seq = list(prompt)
    for pos in range(len(prompt) + n_new):
        t = seq[pos]
        _, lr = ref.forward(t, pos)
        gpu.set_state(t, pos)
        gpu.step()
        torch.cuda.synchronize()
        lg = gpu.logits.cpu().numpy()
        assert np.array_equal(bits(lg), bits(lr)), (pos, float(np.abs(lg - lr).max()))
        nxt_ref = O.argmax(lr)
        nxt_gpu = int(gpu.token.item())
        assert int(gpu.state[0].item()) == nxt_gpu and int(gpu.state[1].item()) == pos + 1
        if pos >= len(prompt) - 1:
            toks_ref.append(nxt_ref)
            toks_gpu.append(nxt_gpu)
            if len(seq) == pos + 1:
                seq.append(nxt_ref)
    assert toks_gpu == toks_ref
    return ref, gpu


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_decoder_matches_oracle(dev, kind):
    cfg = U.DENSE if kind == "dense" else U.MOE
    dtypes = U.dtypes_for(cfg)
    ref, gpu = run_pair(cfg, dtypes, 21, [5, 77, 130, 9], 12, dev)
    # the caches hold the same f16 K and V, bit for bit
    kv = gpu.kv.cpu().numpy().view(np.uint16)
    n = kv.size // 2
    assert np.array_equal(kv[:n], ref.kcache.reshape(-1)) and np.array_equal(kv[n:], ref.vcache.reshape(-1))
    sg_status = __import__("spindle_b200").device_status
    sg_status()


def test_decoder_variants(dev):
    # no Q/K head norms, F16 embedding, Q4_K head, GQA 8:1, non-NEOX rotation
    cfg = dict(U.DENSE, n_heads=8, n_kv_heads=1, qk_norm=False, rope_neox=False)
    dtypes = U.dtypes_for(cfg, embed=O.F16, head=O.Q4_K)
    run_pair(cfg, dtypes, 33, [1, 2, 3], 6, dev)
    cfg = dict(U.MOE, moe=dict(n_expert=16, n_used=4, n_ff=256, norm=False))
    dtypes = U.dtypes_for(cfg, embed=O.Q4_K)
    run_pair(cfg, dtypes, 34, [11, 12], 6, dev)


def test_decoder_separate_wq_wk(dev):
    # wk in its own buffer: q and k from two launches, same results
    cfg = U.MOE
    run_pair(cfg, U.dtypes_for(cfg), 21, [5, 77, 130, 9], 4, dev, qk_adjacent=False)


def test_decoder_long_context_chunks(dev):
    # attention stages K and V in chunks of 128 positions: cross two chunk
    # boundaries (head_dim 64), and one with head_dim 256
    g = np.random.default_rng(8)
    cfg = dict(U.DENSE, max_seq=300)
    run_pair(cfg, U.dtypes_for(cfg), 51, g.integers(0, cfg["vocab"], 262).tolist(), 3, dev)
    cfg = dict(U.DENSE, n_heads=4, n_kv_heads=2, head_dim=256, max_seq=160)
    run_pair(cfg, U.dtypes_for(cfg), 52, g.integers(0, cfg["vocab"], 131).tolist(), 3, dev)


def test_decoder_graph_replay(dev):
    # one captured step replayed: the device state carries token and position
    cfg = U.MOE
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=44)
    dw = U.device_weights(W, dev)
    eager = Decoder(cfg, dw, dtypes, dev)
    want = eager.generate([3, 4, 5], 10)
    g = Decoder(cfg, dw, dtypes, dev)
    for i, t in enumerate([3, 4, 5]):
        g.set_state(t, i)
        g.step(hidden=False, logits=False)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    got = []
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        # capture does not run the step: the state is unchanged by it
        with torch.cuda.graph(graph, stream=s):
            g.step(stream=s, hidden=False, logits=False)
        for _ in range(10):
            got.append(int(g.state[0].item()))
            graph.replay()
            torch.cuda.synchronize()
    torch.cuda.current_stream().wait_stream(s)
    assert got == want


def test_decoder_qwen3_0_6b_shape(dev):
    # Qwen3-0.6B architecture, full size (28 layers, hidden
    # 1024, FFN 3072, 16/8 heads of 128, vocab 151936): 2 prompt tokens, then
    # 40 greedy tokens, every step's logits bit for bit
    cfg = dict(dim=1024, n_heads=16, n_kv_heads=8, head_dim=128, n_layers=28, vocab=151936, max_seq=64,
               rope_theta=1e6, rms_eps=1e-6, n_ff=3072, rope_neox=True)
    dtypes = U.dtypes_for(cfg)
    run_pair(cfg, dtypes, 3, [100, 2000], 40, dev)


def test_decoder_qwen3_30b_a3b_shape(dev):
    # Qwen3-30B-A3B architecture at full size (48 layers,
    # hidden 2048, 32 / 4 heads of 128, 128 experts of FFN 768, top 8, vocab
    # 151936, Q4_K_M mix), random-init on the GPU with the library's quantizer
    # (the bench's model): a 4-token prompt, then 10 greedy tokens, logits bit
    # for bit against the oracle at every position, and the same tokens
    from spindle_b200.decoder import qwen3_dtypes, random_weights
    cfg = dict(dim=2048, n_heads=32, n_kv_heads=4, head_dim=128, n_layers=48, vocab=151936, max_seq=32,
               rope_theta=1e6, rms_eps=1e-6, rope_neox=True, moe=dict(n_expert=128, n_used=8, n_ff=768, norm=True))
    dtypes = qwen3_dtypes(cfg, embed=U.Q4_K)
    W = random_weights(cfg, dtypes, dev, seed=5)
    run_pair(cfg, dtypes, 0, [11, 151000, 42, 7000], 10, dev, W=W)


def test_decoder_bad_args(dev):
    cfg = U.DENSE
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=1)
    d = Decoder(cfg, U.device_weights(W, dev), dtypes, dev)
    import ctypes as C
    from spindle_b200 import decoder as DM
    L = DM._sigs()
    m = d.model
    old = m.head_dim
    m.head_dim = 96
    assert L.sg_model_scratch_bytes(C.byref(m)) == 0
    m.head_dim = old
    st = L.sg_forward(C.byref(m), C.c_void_p(d.state.data_ptr()), C.c_void_p(d.kv.data_ptr()),
                      C.c_void_p(d.scratch.data_ptr()), 16, None, None, None, None)
    assert st == 1  # scratch too small
    st = L.sg_forward(C.byref(m), C.c_void_p(d.state.data_ptr() + 2), C.c_void_p(d.kv.data_ptr()),
                      C.c_void_p(d.scratch.data_ptr()), d.scratch.numel(), None, None, None, None)
    assert st == 4  # misaligned state
    torch.cuda.synchronize()


@pytest.mark.parametrize("kind,neox", [("dense", True), ("moe", True), ("dense", False)])
def test_decoder_kv_shift_matches_oracle(dev, kind, neox):
    # decoding past the context: ensure_kv_room's policy (smollm_chat.rs:
    # 2924-2940) picks the positions to drop, and shift_kv (:2942-2972) runs on
    # the GPU (sg_kv_shift) and in the oracle; the caches after every shift and
    # the logits of every step stay equal bit for bit, through several shifts
    cfg = dict(U.DENSE if kind == "dense" else U.MOE, max_seq=40, rope_neox=neox)
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=33)
    ref = U.oracle_decoder(cfg, dtypes, W)
    gpu = Decoder(cfg, U.device_weights(W, dev), dtypes, dev)
    n_keep, tok, pos, shifts = 5, 17, 0, 0
    n = cfg["n_layers"] * cfg["max_seq"] * cfg["n_kv_heads"] * cfg["head_dim"]
    for _ in range(110):
        n_discard = gpu.kv_room(pos, 1, n_keep)
        if n_discard:
            new_pos = gpu.shift_kv(n_keep, n_discard, pos)
            assert new_pos == ref.kv_shift(n_keep, n_discard, pos) == pos - n_discard
            pos = new_pos
            shifts += 1
            torch.cuda.synchronize()
            kv = gpu.kv.cpu().numpy().view(np.uint16)
            assert np.array_equal(kv[:n], ref.kcache.reshape(-1)), ("K after shift", shifts)
            assert np.array_equal(kv[n:], ref.vcache.reshape(-1)), ("V after shift", shifts)
        _, lr = ref.forward(tok, pos)
        gpu.set_state(tok, pos)
        gpu.step()
        torch.cuda.synchronize()
        assert np.array_equal(bits(gpu.logits.cpu().numpy()), bits(lr)), (pos, shifts)
        tok = O.argmax(lr)
        assert int(gpu.token.item()) == tok
        pos += 1
    assert shifts >= 3


def test_decoder_kv_shift_edges(dev):
    # nothing past the pinned positions: no-op; n_discard clamped to what is there
    cfg = dict(U.DENSE, max_seq=24)
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=34)
    gpu = Decoder(cfg, U.device_weights(W, dev), dtypes, dev)
    for pos, t in enumerate([3, 9, 27, 81, 243, 5]):
        gpu.set_state(t, pos)
        gpu.step()
    before = gpu.kv.clone()
    assert gpu.shift_kv(6, 4, 6) == 6  # everything pinned
    assert gpu.shift_kv(2, 100, 6) == 2  # clamped: all 4 unpinned positions dropped
    torch.cuda.synchronize()
    assert torch.equal(gpu.kv.view(-1)[:0], before.view(-1)[:0])
    import ctypes as C
    from spindle_b200 import decoder as DM
    L = DM._sigs()
    assert L.sg_kv_shift(C.byref(gpu.model), C.c_void_p(gpu.kv.data_ptr()), C.c_void_p(gpu.scratch.data_ptr()), 0, 99,
                         1, 1, 6, None) == 1  # layers past the model
    assert L.sg_kv_shift(C.byref(gpu.model), C.c_void_p(gpu.kv.data_ptr()), C.c_void_p(gpu.scratch.data_ptr()), 0, 1,
                         1, 1, 25, None) == 1  # position past max_seq
