"""Data-parallel host logic on CPU: batch sharding and the rank-ordered
gather, with two gloo ranks running the CPU oracle on their shards."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lotusinfer_b200.dist import gather_outputs, shard_range


def test_shard_range_partitions_the_batch():
    for b in (1, 7, 256, 257):
        for w in (1, 2, 3, 8):
            ranges = [shard_range(b, r, w) for r in range(w)]
            assert ranges[0][0] == 0 and ranges[-1][1] == b
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(w - 1))
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, x, w, b, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle
        s, e = shard_range(x.shape[0], rank, world)
        local = torch.from_numpy(oracle.gemm(x[s:e], w, b, act=1))
        full = gather_outputs(local)
        if rank == 0:
            q.put(full.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_equals_single_process():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (8, 64)).astype(np.float32)
    w = rng.normal(0, 0.1, (10, 64)).astype(np.float32)
    b = rng.normal(0, 0.1, 10).astype(np.float32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, x, w, b, q)) for r in range(2)]
    for p in procs:
        p.start()
    # generous: the spawned ranks import torch afresh, which takes minutes in
    # a cold container
    got = q.get(timeout=600)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle
    np.testing.assert_array_equal(got, oracle.gemm(x, w, b, act=1))
