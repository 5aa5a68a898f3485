"""CPU, world size 2 over gloo: the host logic of the multi-GPU path.

Sequence and head partitions cover every unit once, the head-shard
all-gather rebuilds the unsharded attention output (oracle attention per
shard), and the step time reported is the max over ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from shadowkv_b200 import sharding


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import shadowkv_oracle as o
        rng = np.random.default_rng(0)  # same data on every rank
        B, Hq, Hkv, S, D = 3, 8, 2, 40, 128
        qv = rng.standard_normal((B, Hq, D)).astype(np.float32)
        k = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
        v = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
        full = o.decode_attention(qv, k, v, S)
        k0, kn, q0, qn = sharding.head_range(Hkv, Hq, world, rank)
        local = o.decode_attention(qv[:, q0:q0 + qn], k[:, k0:k0 + kn], v[:, k0:k0 + kn], S)
        gathered = sharding.gather_head_shards(torch.from_numpy(local)).numpy()
        ok_heads = np.allclose(gathered, full, atol=1e-6)
        t = sharding.max_over_ranks(1.0 + rank)
        starts = [None] * world
        dist.all_gather_object(starts, sharding.batch_range(7, world, rank))
        q.put((rank, ok_heads, t, starts))
    finally:
        dist.destroy_process_group()


def test_batch_range_partitions():
    for B in [1, 5, 7, 32, 48]:
        for W in [1, 2, 3, 8]:
            seen = []
            for r in range(W):
                s, c = sharding.batch_range(B, W, r)
                seen.extend(range(s, s + c))
            assert seen == list(range(B))


def test_head_range_keeps_groups_whole():
    assert sharding.head_range(8, 32, 8, 3) == (3, 1, 12, 4)
    assert sharding.head_range(2, 32, 2, 1) == (1, 1, 16, 16)
    with pytest.raises(ValueError):
        sharding.head_range(2, 32, 4, 0)


def test_two_rank_gloo_sharding():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_heads, t, starts in results:
        assert ok_heads
        assert t == 2.0
        assert starts == [(0, 4), (4, 3)]
