"""Speculative decoding on the GPU (spindle_b200.spec over sg_forward_batch):
the token stream equals plain greedy decoding (Decoder.generate, one graph
step per token) exactly, with prompt-lookup drafts, with drafts that are
always right, and with drafts that go wrong part way -- the reference's
guarantee that speculation never changes the output at temperature 0
(docs/speculative_decoding.md, smollm_chat.rs:4205-4340)."""
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import decoder_util as U  # noqa: E402

from spindle_b200.decoder import Decoder  # noqa: E402
from spindle_b200.spec import speculative_generate  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_speculative_equals_greedy(dev, kind):
    cfg = dict(U.DENSE if kind == "dense" else U.MOE, max_seq=200)
    dtypes = U.dtypes_for(cfg)
    dw = U.device_weights(U.host_weights(cfg, dtypes, seed=81), dev)
    rng = np.random.default_rng(10)
    base = rng.integers(0, cfg["vocab"], 12).tolist()
    prompt = base * 4 + rng.integers(0, cfg["vocab"], 30).tolist()   # repeats for the lookup drafter
    n_new = 60
    want = Decoder(cfg, dw, dtypes, dev).generate(prompt, n_new)
    for name, drafter in [("lookup", None),
                          ("right", lambda ctx, k: want[len(ctx) - len(prompt):][:k]),
                          ("half", lambda ctx, k: want[len(ctx) - len(prompt):][:k // 2] + [1] * (k - k // 2))]:
        st = {}
        got = speculative_generate(Decoder(cfg, dw, dtypes, dev), prompt, n_new, drafter=drafter, stats=st, chunk=32)
        assert got == want, (name, st)
        if name == "right":
            assert st["accepted"] >= n_new - 2 * st["passes"] - 1 and st["passes"] <= n_new // 4
    __import__("spindle_b200").device_status()
