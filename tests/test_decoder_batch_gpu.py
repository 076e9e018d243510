"""forward_batch_slice + compute_logits_batch on the GPU (sg_forward_batch):
several positions per call, each token bit for bit the one-token sg_forward
step at its position (logits, greedy token, KV caches) -- the property the
reference's qwen3_moe_batch_is_bitwise test asserts (smollm_chat.rs:
4699-4736).  The one-token step itself is checked against the oracle bit for
bit in test_decoder_gpu.py."""
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


def run(cfg, dtypes, seed, tokens, chunks, dev):
    W = U.host_weights(cfg, dtypes, seed=seed)
    dw = U.device_weights(W, dev)
    seq = Decoder(cfg, dw, dtypes, dev)
    bat = Decoder(cfg, dw, dtypes, dev)
    want_l, want_g = [], []
    for pos, t in enumerate(tokens):
        seq.set_state(t, pos)
        seq.step()
        torch.cuda.synchronize()
        want_l.append(seq.logits.cpu().numpy().copy())
        want_g.append(int(seq.token.item()))
    pos = 0
    for c in chunks:
        lg, gr = bat.forward_batch(tokens[pos:pos + c], pos)
        torch.cuda.synchronize()
        lg, gr = lg.cpu().numpy(), gr.cpu().numpy()
        for i in range(c):
            assert np.array_equal(bits(lg[i]), bits(want_l[pos + i])), (pos + i, float(np.abs(lg[i] - want_l[pos + i]).max()))
            assert int(gr[i]) == want_g[pos + i], pos + i
        pos += c
    assert pos == len(tokens)
    assert torch.equal(seq.kv, bat.kv)
    __import__("spindle_b200").device_status()


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_batch_matches_steps(dev, kind):
    cfg = U.DENSE if kind == "dense" else U.MOE
    g = np.random.default_rng(4)
    toks = g.integers(0, cfg["vocab"], 40).tolist()
    run(cfg, U.dtypes_for(cfg), 71, toks, [1, 3, 9, 17, 2, 8], dev)


def test_batch_variants(dev):
    # no QK norms, adjacent-pair RoPE, GQA 8:1, F16 embedding, one token per call
    cfg = dict(U.DENSE, n_heads=8, n_kv_heads=1, qk_norm=False, rope_neox=False)
    toks = np.random.default_rng(5).integers(0, cfg["vocab"], 12).tolist()
    run(cfg, U.dtypes_for(cfg, embed=O.F16, head=O.Q4_K), 72, toks, [1] * 12, dev)
    # head_dim 256
    cfg = dict(U.DENSE, n_heads=4, n_kv_heads=2, head_dim=256)
    toks = np.random.default_rng(6).integers(0, cfg["vocab"], 20).tolist()
    run(cfg, U.dtypes_for(cfg), 73, toks, [5, 15], dev)
    # a group of 3 query heads (not a divisor of 8): the per-head attention kernel
    cfg = dict(U.DENSE, n_heads=12, n_kv_heads=4, head_dim=64)
    toks = np.random.default_rng(16).integers(0, cfg["vocab"], 20).tolist()
    run(cfg, U.dtypes_for(cfg), 77, toks, [9, 11], dev)
    # one KV head for 4 query heads of 128, past two 64-position chunks
    cfg = dict(U.DENSE, n_heads=4, n_kv_heads=1, head_dim=128, max_seq=200)
    toks = np.random.default_rng(17).integers(0, cfg["vocab"], 150).tolist()
    run(cfg, U.dtypes_for(cfg), 78, toks, [64, 63, 23], dev)


def test_batch_long_context(dev):
    # past the attention kernel's 128-position chunks, batches of 64 and of
    # 128 (feed's chunk, two QB groups per image)
    cfg = dict(U.DENSE, max_seq=300)
    toks = np.random.default_rng(7).integers(0, cfg["vocab"], 200).tolist()
    run(cfg, U.dtypes_for(cfg), 74, toks, [64, 64, 9, 63], dev)
    toks = np.random.default_rng(10).integers(0, cfg["vocab"], 290).tolist()
    run(cfg, U.dtypes_for(cfg), 79, toks, [128, 100, 62], dev)


@pytest.mark.parametrize("amin", ["1", "1000"])
def test_batch_attention_forms(dev, monkeypatch, amin):
    # the batch attention with K/V rows shared by a CTA's (query head, token)
    # pairs from one token on (1), and the per-(head, token) kernel only (1000):
    # GQA groups of 1, 2, 4 and 8, head_dim 64 / 128 / 256, chunks crossing
    # the 32-position staging chunks, every token still the one-token step
    monkeypatch.setenv("SG_ATTN_BATCH_MIN", amin)
    for cfg, chunks, seed in [(dict(U.DENSE, max_seq=160), [1, 40, 33, 70], 81),
                              (dict(U.MOE, max_seq=160), [17, 2, 64, 40], 82),
                              (dict(U.DENSE, n_heads=8, n_kv_heads=1, max_seq=100), [5, 31, 32, 9], 83),
                              (dict(U.DENSE, n_heads=4, n_kv_heads=4, head_dim=256, max_seq=80), [3, 50], 84)]:
        toks = np.random.default_rng(seed).integers(0, cfg["vocab"], sum(chunks)).tolist()
        run(cfg, U.dtypes_for(cfg), seed, toks, chunks, dev)


def test_batch_moe_verify_chunks(dev):
    # the verify batch of BASELINE config 5: 9 positions per call
    cfg = dict(U.MOE)
    toks = np.random.default_rng(8).integers(0, cfg["vocab"], 18).tolist()
    run(cfg, U.dtypes_for(cfg), 75, toks, [9, 9], dev)


@pytest.mark.parametrize("chunk", [64, 128])
@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_feed_matches_steps(dev, kind, chunk):
    # feed (smollm_chat.rs:3042-3106): chunks without the LM head; the last
    # output-normed hidden state and every K/V row equal the one-token steps'
    cfg = dict(U.DENSE if kind == "dense" else U.MOE, max_seq=160)
    dtypes = U.dtypes_for(cfg)
    dw = U.device_weights(U.host_weights(cfg, dtypes, seed=76), dev)
    seq = Decoder(cfg, dw, dtypes, dev)
    bat = Decoder(cfg, dw, dtypes, dev)
    toks = np.random.default_rng(9).integers(0, cfg["vocab"], 150).tolist()
    for pos, t in enumerate(toks):
        seq.set_state(t, pos)
        seq.step(logits=False)
    h = bat.feed(toks, 0, chunk=chunk)
    torch.cuda.synchronize()
    assert np.array_equal(bits(h.cpu().numpy()), bits(seq.hidden.cpu().numpy()))
    assert torch.equal(seq.kv, bat.kv)
    __import__("spindle_b200").device_status()


@pytest.mark.parametrize("kind,chunk,k", [("dense", 64, 2), ("moe", 32, 2), ("moe", 128, 2), ("moe", 32, 3)])
def test_feed_overlapped_matches_feed(dev, kind, chunk, k):
    # k chunks in flight, a layer at a time on k streams with their own
    # scratch (sg_forward_batch_range continuing on a scratch): the caches and
    # the last hidden state bit for bit those of feed
    cfg = dict(U.DENSE if kind == "dense" else U.MOE, max_seq=160, n_layers=3)
    dtypes = U.dtypes_for(cfg)
    dw = U.device_weights(U.host_weights(cfg, dtypes, seed=88), dev)
    a = Decoder(cfg, dw, dtypes, dev)
    b = Decoder(cfg, dw, dtypes, dev)
    toks = np.random.default_rng(12).integers(0, cfg["vocab"], 150).tolist()
    ha = a.feed(toks, 0, chunk=chunk)
    hb = b.feed_overlapped(toks, 0, chunk=chunk, in_flight=k)
    torch.cuda.synchronize()
    assert np.array_equal(bits(ha.cpu().numpy()), bits(hb.cpu().numpy()))
    assert torch.equal(a.kv, b.kv)
    __import__("spindle_b200").device_status()
