"""sg_matvec_list: several GEMVs in one persistent launch.  Each output is
the oracle's integer GEMV (quant_q8k.rs:255-295 after Q8K::quantize) bit for
bit, and equals sg_matvec's on the same entry: small mixed lists against the
oracle, the full BASELINE sweep shapes against sg_matvec (every warp split
the launch plan picks: S = 1 on the LM head, 2 on 14336 x 4096, 16 on the
wide rows), the longest list, and the argument checks.  The Q8_K image form
(sg_q8k_images + sg_matvec_list_q8k): images byte for byte the oracle's
Q8K::quantize, GEMVs bit for bit the fp32 form; also with the remainder
tiles left unrotated (SG_LIST_ROT=0) and on the longest, widest lists."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import spindle_b200 as sg
from spindle_b200._lib import SgError

pytestmark = pytest.mark.gpu


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def bits(a):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


SMALL = [(O.Q4_K, 256, 37), (O.Q6_K, 768, 16), (O.Q4_K, 4096, 45), (O.Q6_K, 14336, 33), (O.Q6_K, 1024, 301),
         (O.Q4_K, 2048, 1), (O.Q4_K, 14336, 70), (O.Q6_K, 4096, 130)]


def image_of(q):
    """The sg_q8k_images layout of an oracle Q8K: qs | bsums | d (padded)."""
    nb = q.d.size
    pad = (-4 * nb) % 16
    return np.concatenate([q.qs.view(np.uint8), q.bsums.view(np.uint8), q.d.view(np.uint8), np.zeros(pad, np.uint8)])


def test_images_match_oracle(dev):
    rng = O.Rng(0x1A6E)
    xs = [rng.fill(-3.0, 3.0, n) for n in (256, 768, 1024, 4096, 14336)]
    # images land in memory that held other bytes: the padding must still be zero
    junk = torch.full((1 << 20,), 0x5A, dtype=torch.uint8, device=dev)
    del junk
    xs[1][5] = 0.0
    xs[2][:256] = 0.0  # an all-zero block
    xs[3][300] = 1e30  # a large value in one block
    imgs = sg.q8k_images([to_dev(x, dev) for x in xs])
    torch.cuda.synchronize()
    for x, img in zip(xs, imgs):
        q = O.quantize(x)
        assert img.numel() == sg.lib().sg_q8k_image_bytes(x.size)
        assert np.array_equal(img.cpu().numpy(), image_of(q)), x.size
    assert sg.lib().sg_q8k_image_bytes(100) == 0


@pytest.fixture(params=["rotated", "unrotated"])
def mode(request):
    old = os.environ.get("SG_LIST_ROT")
    os.environ["SG_LIST_ROT"] = "1" if request.param == "rotated" else "0"
    yield request.param
    if old is None:
        del os.environ["SG_LIST_ROT"]
    else:
        os.environ["SG_LIST_ROT"] = old


def test_list_matches_oracle(dev, mode):
    rng = O.Rng(0x1157)
    entries, want = [], []
    for dt, n, rows in SMALL:
        w = O.random_matrix(dt, n, rows, rng)
        x = rng.fill(-2.0, 2.0, n)
        want.append(O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x)])[0])
        t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
        entries.append((t, m, to_dev(x, dev)))
    for k in (1, 3, len(entries)):
        got = sg.matvec_list(entries[:k])
        imgs = sg.q8k_images([x for _, _, x in entries[:k]])
        got_q = sg.matvec_list_q8k([(t, m, i) for (t, m, _), i in zip(entries[:k], imgs)])
        torch.cuda.synchronize()
        for j in range(k):
            assert np.array_equal(bits(got[j]), bits(want[j])), (k, j, SMALL[j])
            assert np.array_equal(bits(got_q[j]), bits(want[j])), (k, j, SMALL[j])
    sg.device_status()


def test_list_equals_matvec_on_sweep_shapes(dev, mode):
    g = torch.Generator(device=dev).manual_seed(5)
    shapes = [(O.Q4_K, 4096, 4096), (O.Q6_K, 4096, 4096), (O.Q4_K, 14336, 4096), (O.Q6_K, 14336, 4096),
              (O.Q4_K, 4096, 14336), (O.Q6_K, 4096, 14336), (O.Q6_K, 151936, 1024)]
    entries = []
    for dt, rows, cols in shapes:
        wq = sg.quantize_weights(dt, torch.randn(rows, cols, device=dev, generator=g) * 0.02)
        t, m = sg.repack_tiled16(dt, wq, rows, cols)
        del wq
        entries.append((t, m, torch.randn(cols, device=dev, generator=g)))
    got = sg.matvec_list(entries)
    want = [sg.matvec(t, m, x).reshape(-1) for t, m, x in entries]
    imgs = sg.q8k_images([x for _, _, x in entries])
    got_q = sg.matvec_list_q8k([(t, m, i) for (t, m, _), i in zip(entries, imgs)])
    torch.cuda.synchronize()
    for j, (a, b) in enumerate(zip(got, want)):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32)), shapes[j]
        assert torch.equal(got_q[j].view(torch.int32), b.view(torch.int32)), shapes[j]
    # the same list in another order, and each matrix twice in one launch
    order = [6, 0, 5, 1, 4, 2, 3] + [3, 2, 4, 1, 5, 0, 6]
    got2 = sg.matvec_list([entries[i] for i in order])
    torch.cuda.synchronize()
    for j, i in enumerate(order):
        assert torch.equal(got2[j].view(torch.int32), want[i].view(torch.int32)), (j, shapes[i])
    sg.device_status()


def test_list_longest_and_checks(dev, mode):
    rng = O.Rng(99)
    dt, n, rows = O.Q4_K, 1024, 50
    w = O.random_matrix(dt, n, rows, rng)
    t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
    xs = [rng.fill(-1.0, 1.0, n) for _ in range(16)]
    want = O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x) for x in xs])
    got = sg.matvec_list([(t, m, to_dev(x, dev)) for x in xs])
    torch.cuda.synchronize()
    for j in range(16):
        assert np.array_equal(bits(got[j]), bits(want[j])), j
    with pytest.raises(SgError):
        sg.matvec_list([(t, m, to_dev(xs[0], dev))] * 17)
    # GGUF rows are not a TILED16 matrix
    gw = to_dev(w, dev)
    with pytest.raises(SgError):
        sg.matvec_list([(gw, sg.Mat(dt, n, rows), to_dev(xs[0], dev))])
    sg.device_status()


def test_list_of_wide_rows(dev):
    # 16 matrices of 14336 columns, both types, ragged row counts
    rng = O.Rng(7)
    entries, want = [], []
    for j in range(16):
        dt, n, rows = (O.Q6_K if j % 2 else O.Q4_K), 14336, 17 + j
        w = O.random_matrix(dt, n, rows, rng)
        x = rng.fill(-1.0, 1.0, n)
        want.append(O.gemv_int(w, O.Mat(dt, n, rows), [O.quantize(x)])[0])
        t, m = sg.repack_tiled16(dt, to_dev(w, dev), rows, n)
        entries.append((t, m, to_dev(x, dev)))
    got = sg.matvec_list(entries)
    imgs = sg.q8k_images([x for _, _, x in entries])
    got_q = sg.matvec_list_q8k([(t, m, i) for (t, m, _), i in zip(entries, imgs)])
    torch.cuda.synchronize()
    for j in range(16):
        assert np.array_equal(bits(got[j]), bits(want[j])), j
        assert np.array_equal(bits(got_q[j]), bits(want[j])), j
    sg.device_status()
