"""GGUF files (gguf_loader.rs:142-247, ModelConfig::from_gguf and
resolve_layers in smollm_chat.rs): the writer and the reader round-trip
metadata, the tensor table and the data; a synthetic model written to a file
and loaded back onto the GPU decodes to the same logits and tokens as the same
weights given in memory."""
import os
import struct
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import decoder_util as U  # noqa: E402

from spindle_b200 import gguf  # noqa: E402


def test_roundtrip_metadata_tensors_alignment(tmp_path):
    p = str(tmp_path / "a.gguf")
    rng = np.random.default_rng(0)
    q4 = rng.integers(0, 256, 144 * 3 * 5, dtype=np.uint8)          # Q4_K [768 x 5]
    f32 = rng.standard_normal(24).astype(np.float32)
    meta = {"general.architecture": "qwen3", "general.name": "t", "x.u": 7, "x.f": 1.5, "x.b": True,
            "x.s": "hello", "x.list": ["a", "bb", ""], "x.ints": [1, -2, 3], "x.big": (2 ** 40, gguf.T_U64)}
    gguf.write_gguf(p, meta, [("w", [768, 5], 12, q4), ("n", [24], 0, f32.view(np.uint8))], alignment=64)
    g = gguf.GgufFile(p)
    assert g.version == 3 and g.alignment == 64 and g.architecture == "qwen3"
    for k in ("x.u", "x.f", "x.b", "x.s", "x.list"):
        assert g.metadata[k] == meta[k], k
    assert [int(v) for v in g.metadata["x.ints"]] == [1, -2, 3] and g.metadata["x.big"] == 2 ** 40
    assert list(g.tensors) == ["w", "n"]
    assert g.tensors["w"].dims == [768, 5] and g.tensors["w"].dtype == 12
    assert all(t.offset % 64 == 0 for t in g.tensors.values())
    assert np.array_equal(g.data("w"), q4) and np.array_equal(np.asarray(g.data("n")).view(np.float32), f32)


def test_reader_rejects_bad_files(tmp_path):
    p = str(tmp_path / "b.gguf")
    with open(p, "wb") as f:
        f.write(struct.pack("<IIQQ", 0x12345678, 3, 0, 0))
    with pytest.raises(gguf.GgufError):
        gguf.GgufFile(p)
    gguf.write_gguf(p, {"general.architecture": "qwen3"}, [("w", [256, 4], 14, np.zeros(840, np.uint8))])
    data = open(p, "rb").read()
    with open(p, "wb") as f:
        f.write(data[:-100])  # a cut-off download (Model::load's size check)
    with pytest.raises(gguf.GgufError, match="incomplete"):
        gguf.GgufFile(p)
    with pytest.raises(gguf.GgufError):
        gguf.write_gguf(p, {}, [("w", [300, 4], 12, np.zeros(10, np.uint8))])  # not a whole block
    gguf.write_gguf(p, {"general.architecture": "gpt9"}, [])
    with pytest.raises(gguf.GgufError, match="unsupported architecture"):
        gguf.model_config(gguf.GgufFile(p))


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_model_file_config(tmp_path, kind):
    cfg = dict(U.DENSE if kind == "dense" else U.MOE)
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=1)
    p = str(tmp_path / ("%s.gguf" % kind))
    gguf.write_model(p, cfg, W, dtypes)
    g = gguf.GgufFile(p)
    got = gguf.model_config(g)
    for k in ("dim", "n_heads", "n_kv_heads", "head_dim", "n_layers", "vocab", "max_seq", "rope_neox"):
        assert got[k] == cfg[k], k
    assert got["rope_theta"] == cfg["rope_theta"] and abs(got["rms_eps"] - cfg["rms_eps"]) < 1e-12
    assert (got.get("moe") == cfg.get("moe")) if kind == "moe" else got["n_ff"] == cfg["n_ff"]
    assert g.tensors["blk.1.attn_v.weight"].dtype == dtypes["l1.wv"]
    assert np.array_equal(g.data("blk.0.attn_q.weight"), W["l0.wq"])


@pytest.mark.gpu
@pytest.mark.parametrize("kind,tied", [("dense", False), ("moe", False), ("moe", True)])
def test_model_file_decodes_like_memory(tmp_path, dev, kind, tied):
    import torch
    from spindle_b200.decoder import Decoder
    cfg = dict(U.DENSE if kind == "dense" else U.MOE)
    dtypes = U.dtypes_for(cfg)
    W = U.host_weights(cfg, dtypes, seed=2)
    if tied:
        W["head"] = W["embed"]  # one tensor for both (a tied Q6_K embedding, as Qwen3-0.6B's)
    p = str(tmp_path / "m.gguf")
    gguf.write_model(p, cfg, W, dtypes, tie_head=tied)
    g = gguf.GgufFile(p)
    assert ("output.weight" in g.tensors) == (not tied)
    mem = Decoder(cfg, U.device_weights(W, dev), dtypes, dev)
    fil, fcfg = gguf.load_decoder(p, dev)
    assert fcfg["max_seq"] == cfg["max_seq"]
    for pos, t in enumerate([5, 77, 130, 9, 400, 11, 3, 99]):
        for d in (mem, fil):
            d.set_state(t, pos)
            d.step()
        torch.cuda.synchronize()
        assert torch.equal(mem.logits.view(torch.int32), fil.logits.view(torch.int32)), pos
        assert torch.equal(mem.state, fil.state)
    assert mem.generate([1, 2, 3], 6) == fil.generate([1, 2, 3], 6)
