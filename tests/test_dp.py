"""Data-parallel request sharding (no collective on the hot path) with world_size-2 gloo ranks on the CPU."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from gravityocr_b200.dp import lpt_shards


def test_lpt_shards_cover_and_balance():
    work = [float(w) for w in [4096, 300, 2500, 2500, 900, 4100, 256, 1000, 3000]]
    for n in (1, 2, 4, 8):
        sh = lpt_shards(work, n)
        flat = sorted(i for s in sh for i in s)
        assert flat == list(range(len(work)))
        loads = [sum(work[i] for i in s) for s in sh]
        assert max(loads) - min(loads) <= max(work)
    assert lpt_shards(work, 2) == lpt_shards(work, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from gravityocr_b200 import dp
    dp.init("gloo", timeout_s=60)
    work = [300.0, 4000.0, 1200.0, 2600.0, 800.0]
    mine = dp.lpt_shards(work, world)[rank]
    dp.barrier()
    t = dp.max_over_ranks(1.0 + rank)
    tok = dp.sum_over_ranks(float(len(mine) * 10))
    out.put((rank, mine, t, tok))
    dp.finish()


def test_gloo_two_ranks_shard_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(res[0][1] + res[1][1]) == list(range(5))
    assert res[0][2] == res[1][2] == 2.0
    assert res[0][3] == res[1][3] == 50.0


def test_balanced_shards_equal_counts_cover_and_balance():
    """The benchmark's sharder: every replica gets the same number of requests (one batch size per GPU), every request
    lands on exactly one replica, and the expected work per replica stays within one request's work."""
    from gravityocr_b200.dp import balanced_shards
    import torch
    g = torch.Generator().manual_seed(3)
    work = (torch.randint(256, 4097, (512,), generator=g) + torch.randint(256, 2049, (512,), generator=g)).tolist()
    for n in (1, 2, 4, 8):
        sh = balanced_shards(work, n)
        assert sorted(i for s in sh for i in s) == list(range(len(work)))
        assert {len(s) for s in sh} == {len(work) // n}
        loads = [sum(work[i] for i in s) for s in sh]
        assert max(loads) - min(loads) <= max(work)
        assert sh == balanced_shards(work, n)          # deterministic
