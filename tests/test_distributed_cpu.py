"""Host side of data-parallel training, on 2 gloo ranks (CPU only).

The device path sums each split's integer child histogram and left-row count over the
ranks (NCCL all-reduce). Here the same contract is checked with the oracle's quantized
gradients and numpy histograms: shard-local integer histograms summed over ranks equal
the histogram of all rows, whatever the shard sizes; and the NCCL id travels from rank 0
to every rank through the torch.distributed group.
"""

import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import sys
        import os
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch
        import torch.distributed as dist

        import oracle
        from lightgbm_rs_b200 import distributed as D

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        # 1. the communicator id reaches every rank unchanged
        uid = bytes(range(128)) if rank == 0 else None
        got = D.broadcast_bytes(uid, src=0)
        ok_id = got == bytes(range(128))
        # 2. integer child histograms summed over shards = histogram of all rows
        rng = np.random.default_rng(3)
        n = 10_007
        bins = rng.integers(0, 64, n).astype(np.int64)
        g = rng.normal(0, 1, n)
        h = rng.uniform(0.01, 0.25, n)
        _, _, qp, _ = oracle.quantize(g, h, 4)
        qg = qp[:, 0].astype(np.int64)
        qh = qp[:, 1].astype(np.int64)
        b, e = D.shard_range(n, world, rank)
        left = bins[b:e] <= 20  # a split's left child on this shard
        local = np.stack([np.bincount(bins[b:e][left], weights=qg[b:e][left], minlength=64),
                          np.bincount(bins[b:e][left], weights=qh[b:e][left], minlength=64)])
        t = torch.from_numpy(np.concatenate([local.reshape(-1),
                                             [left.sum()]]).astype(np.int64))
        dist.all_reduce(t)
        full_left = bins <= 20
        want = np.stack([np.bincount(bins[full_left], weights=qg[full_left], minlength=64),
                         np.bincount(bins[full_left], weights=qh[full_left], minlength=64)])
        ok_hist = np.array_equal(t.numpy()[:-1], want.reshape(-1).astype(np.int64))
        ok_count = int(t.numpy()[-1]) == int(full_left.sum())
        # 3. max over ranks (the bench's timing rule)
        mx = torch.tensor([float(rank + 1)])
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
        q.put((rank, ok_id, ok_hist, ok_count, float(mx.item()), (b, e)))
    except Exception as ex:  # reported to the parent
        q.put((rank, "error", repr(ex)))


def test_shard_range_covers_rows():
    from lightgbm_rs_b200.distributed import shard_range

    for n in (0, 1, 7, 10_500_000):
        for w in (1, 2, 3, 8):
            rs = [shard_range(n, w, r) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(rs[i][1] == rs[i + 1][0] for i in range(w - 1))
            sizes = [e - b for b, e in rs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_two_gloo_ranks(oracle_lib):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r = q.get(timeout=120)
            out[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert out[r][1] != "error", out[r]
        _, ok_id, ok_hist, ok_count, mx, rng = out[r]
        assert ok_id and ok_hist and ok_count
        assert mx == 2.0
    assert out[0][5][1] == out[1][5][0]
