"""Host logic of the row-split tensor parallelism (spindle_b200.tp) on CPU:
the shard split, the rank-ordered exchange and the gather layout of the
row-split list (gather_layout / split_gathered), over gloo with two ranks."""
import os
import socket
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import tp_util  # noqa: E402

from spindle_b200.tp import shard_rows  # noqa: E402


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("rows", [1, 2, 15, 16, 17, 4096, 151936])
def test_shard_rows_partition(rows):
    # par_rows (smollm_chat.rs:334): contiguous, disjoint, covering, sizes within one
    for n in range(1, 9):
        parts = [shard_rows(rows, n, p) for p in range(n)]
        assert parts[0][0] == 0 and parts[-1][1] == rows
        assert all(parts[p][1] == parts[p + 1][0] for p in range(n - 1))
        sizes = [b - a for a, b in parts]
        assert max(sizes) - min(sizes) <= 1


def test_exchange_two_ranks_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=tp_util.cpu_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
