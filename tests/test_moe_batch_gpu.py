"""The batched MoE layer (sg_moe_forward_batch, moe_forward_batch at
smollm_chat.rs:928-1174) against one-token steps: the reference's batch is
one-token-identical (:4699-4736), so every token's output must equal, bit for
bit, both the GPU's one-token sg_moe_forward and the oracle's moe_forward."""
import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg

from test_moe_gpu import gpu_layer, make_layer

pytestmark = pytest.mark.gpu


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), a).view(np.uint32)


def run_batch(L, xs, dev, norm=True, prune=0.0):
    moe = L["moe"]
    moe.norm, moe.moe_prune = int(norm), prune
    m = gpu_layer(L, dev, norm, prune)
    xt = torch.from_numpy(np.ascontiguousarray(xs)).to(dev)
    choices = torch.zeros(xs.shape[0], 36, dtype=torch.int32, device=dev)
    got = sg.moe_forward_batch(m, xt, choices=choices).cpu().numpy()
    torch.cuda.synchronize()
    sg.device_status()
    for t in range(xs.shape[0]):
        one_choice = torch.zeros(36, dtype=torch.int32, device=dev)
        one = sg.moe_forward(m, xt[t].contiguous(), choice=one_choice).cpu().numpy()
        assert np.array_equal(bits(got[t]), bits(one)), ("token vs one-token GPU step", t)
        assert torch.equal(choices[t], one_choice), ("choice", t)
        want, ids, _ = O.moe_forward(L["raw"], moe, xs[t])
        assert np.array_equal(bits(got[t]), bits(want)), ("token vs oracle", t)
        assert sg.decode_choice(choices[t])[0] == [int(e) for e in ids]
    return got


@pytest.mark.parametrize("n_tok", [1, 2, 9, 17, 128])
def test_moe_batch_small(dev, n_tok):
    L = make_layer(7, 512, 256, 16, 4)
    xs = np.stack([O.Rng(100 + t).fill(-1.0, 1.0, 512) for t in range(n_tok)])
    run_batch(L, xs, dev)
    run_batch(L, xs, dev, norm=False)


@pytest.mark.parametrize("job_nv", ["0", "4", "8"])
def test_moe_batch_expert_jobs(dev, monkeypatch, job_nv):
    # the expert passes over jobs (each expert's blocks decoded once for up to
    # 4 or 8 of its slots, moe_batch_fused's union jobs) from one token on, and
    # per slot (0): every token still bit for bit the one-token step
    monkeypatch.setenv("SG_MOE_JOB_NV", job_nv)
    monkeypatch.setenv("SG_MOE_JOBS_MIN", "1")
    L = make_layer(9, 512, 256, 16, 4)
    for n_tok in (1, 3, 40):
        xs = np.stack([O.Rng(200 + t).fill(-1.0, 1.0, 512) for t in range(n_tok)])
        run_batch(L, xs, dev)
    L = make_layer(31, 2048, 768, 128, 8)
    xs = np.stack([O.Rng(400 + t).fill(-1.0, 1.0, 2048) for t in range(33)])
    run_batch(L, xs, dev, prune=4.0)


def test_moe_batch_qwen3_verify(dev):
    # the Qwen3-30B-A3B layer at the verify batch of config 5 (N = 9), and 64 tokens
    L = make_layer(30, 2048, 768, 128, 8)
    rng = O.Rng(32)
    xs = np.stack([rng.fill(-1.0, 1.0, 2048) for _ in range(9)])
    run_batch(L, xs, dev)
    xs = np.stack([rng.fill(-1.0, 1.0, 2048) for _ in range(64)])
    run_batch(L, xs, dev, prune=4.0)


@pytest.mark.parametrize("prune", [0.3, 0.8, 4.0])
def test_moe_batch_prune(dev, prune):
    L = make_layer(11, 256, 256, 64, 8)
    xs = np.stack([O.Rng(200 + t).fill(-1.0, 1.0, 256) for t in range(5)])
    run_batch(L, xs, dev, prune=prune)


@pytest.mark.parametrize("gate", [False, True])
def test_moe_batch_shared_expert(dev, gate):
    L = make_layer(12, 512, 256, 32, 4, shared_ff=512, shared_gate=gate)
    xs = np.stack([O.Rng(300 + t).fill(-1.0, 1.0, 512) for t in range(6)])
    run_batch(L, xs, dev)


def test_moe_batch_repeated_tokens_and_nan(dev):
    # the same token twice (same experts, separate slots) and a NaN token
    L = make_layer(13, 256, 256, 16, 4)
    x = O.Rng(5).fill(-1.0, 1.0, 256)
    y = O.Rng(6).fill(-1.0, 1.0, 256)
    xs = np.stack([x, y, x])
    got = run_batch(L, xs, dev)
    assert np.array_equal(bits(got[0]), bits(got[2]))
    z = np.full(256, np.nan, np.float32)
    run_batch(L, np.stack([x, z]), dev)


def test_moe_batch_bad_args(dev):
    L = make_layer(14, 256, 256, 16, 4)
    m = gpu_layer(L, dev)
    with pytest.raises(sg.SgError) as e:
        sg.moe_forward_batch(m, torch.zeros(129, 256, device=dev), scratch=torch.empty(1 << 20, dtype=torch.uint8,
                                                                                          device=dev))
    assert e.value.status == 3
    L2 = make_layer(15, 256, 256, 300, 4)
    with pytest.raises(sg.SgError) as e:
        sg.moe_forward_batch(gpu_layer(L2, dev), torch.zeros(2, 256, device=dev),
                             scratch=torch.empty(1 << 22, dtype=torch.uint8, device=dev))
    assert e.value.status == 3
