"""Multi-process (gloo, world size 2 and 3) checks of the sharding layer on CPU:
shards cover the work exactly once, respect alignment, and an all-gather of
per-rank results reproduces the single-process result. The per-rank "kernel" here
is a CPU stand-in (numpy matmul / row reductions): the kernels themselves are
covered by the GPU tests; this checks the host logic around them."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tk_b200 import dist as tkd


@pytest.mark.parametrize("total,world,align", [(8192, 8, 256), (16384, 3, 256), (16, 2, 256), (1000, 7, 1),
                                               (1 << 20, 8, 1), (0, 4, 1), (256 * 5 + 16, 4, 256)])
def test_shards_cover_exactly_once(total, world, align):
    covered = np.zeros(total, dtype=np.int32)
    prev_stop = 0
    for r in range(world):
        start, stop = tkd.shard_range(total, world, r, align)
        assert start == prev_stop and start <= stop
        if stop < total:
            assert stop % align == 0
        covered[start:stop] += 1
        prev_stop = stop
    assert prev_stop == total and np.all(covered == 1)


def test_invalid_requests():
    with pytest.raises(ValueError):
        tkd.shard_range(10, 0, 0)
    with pytest.raises(ValueError):
        tkd.shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(0)
        m, n, k = 600, 48, 32
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        r0, r1 = tkd.gemm_rows(m, world, rank)
        c_local = torch.from_numpy(a[r0:r1] @ b)
        c = tkd.gather_shards(c_local, m, world, rank, lambda w, r: tkd.gemm_rows(m, w, r))
        ok_gemm = np.allclose(c.numpy(), a @ b, rtol=1e-5, atol=1e-5)
        # Tile row sums sharded by tile range.
        tiles = rng.standard_normal((37, 16, 16)).astype(np.float32)
        t0, t1 = tkd.tile_range(37, world, rank)
        s_local = torch.from_numpy(tiles[t0:t1].sum(axis=2))
        s = tkd.gather_shards(s_local, 37, world, rank, lambda w, r: tkd.tile_range(37, w, r))
        ok_rows = np.allclose(s.numpy(), tiles.sum(axis=2))
        # Attention slices: each rank owns whole (batch, head) slices.
        b0, b1 = tkd.attention_slices(3, 5, world, rank)
        own = torch.arange(b0, b1, dtype=torch.float32).reshape(-1, 1)
        allslices = tkd.gather_shards(own, 15, world, rank, lambda w, r: tkd.attention_slices(3, 5, w, r))
        ok_att = np.array_equal(allslices.numpy().ravel(), np.arange(15, dtype=np.float32))
        result_q.put((rank, ok_gemm and ok_rows and ok_att))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_sharded_results_match_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(results.values()), results
