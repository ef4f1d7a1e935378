"""Multi-process partitioning on CPU (gloo, world size 2): every rank computes its
shard of the oracle; the gathered shards must equal the unsharded result exactly and
cover every unit once.  Mirrors how bench.py shards the GPU work (no collective on
the data path; the gather is only for checking)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tilelang_fa_v100 import sharding
from oracle import attention_ref as R


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense_worker(rank, world, port, q, k, v, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, h = q.shape[0], q.shape[1]
        start, stop = sharding.dense_pairs(b, h, world, rank)
        out = np.zeros_like(q, dtype=np.float32)
        for pair in range(start, stop):
            bi, hi = divmod(pair, h)
            o, _ = R.attention_ref(q[bi:bi + 1, hi:hi + 1], k[bi:bi + 1, hi:hi + 1],
                                   v[bi:bi + 1, hi:hi + 1], causal=True)
            out[bi, hi] = o[0, 0]
        t = torch.from_numpy(out)
        dist.all_reduce(t)  # shards are disjoint: the sum reassembles the full output
        cover = torch.zeros(b * h)
        cover[start:stop] = 1
        dist.all_reduce(cover)
        if rank == 0:
            ret["out"] = t.numpy()
            ret["cover"] = cover.numpy()
    finally:
        dist.destroy_process_group()


def test_dense_sharding_reassembles_full_result():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((3, 5, 40, 16)).astype(np.float32)
    k = rng.standard_normal((3, 5, 40, 16)).astype(np.float32)
    v = rng.standard_normal((3, 5, 40, 16)).astype(np.float32)
    ret = mp.Manager().dict()
    mp.start_processes(_dense_worker, args=(2, _free_port(), q, k, v, ret), nprocs=2,
                       start_method="spawn")
    full, _ = R.attention_ref(q, k, v, causal=True)
    np.testing.assert_array_equal(ret["cover"], np.ones(15))
    np.testing.assert_allclose(ret["out"], full, rtol=0, atol=0)


def _decode_worker(rank, world, port, lens, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        owned = sharding.balance_sequences(lens, world)[rank]
        mine = torch.zeros(len(lens))
        mine[owned] = 1
        load = torch.tensor([float(sum(lens[i] for i in owned))])
        dist.all_reduce(mine)
        loads = [torch.zeros(1) for _ in range(world)]
        dist.all_gather(loads, load)
        if rank == 0:
            ret["cover"] = mine.numpy()
            ret["loads"] = [float(x) for x in loads]
    finally:
        dist.destroy_process_group()


def test_decode_sequence_balancing():
    lens = list(np.random.default_rng(0).integers(512, 8193, size=256))
    ret = mp.Manager().dict()
    mp.start_processes(_decode_worker, args=(2, _free_port(), lens, ret), nprocs=2,
                       start_method="spawn")
    np.testing.assert_array_equal(ret["cover"], np.ones(256))
    loads = ret["loads"]
    assert abs(loads[0] - loads[1]) <= max(lens)
    assert sum(loads) == sum(lens)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partitions_cover_exactly_once(world):
    for b, h in ((8, 32), (4, 16), (3, 5)):
        seen = []
        for r in range(world):
            s, e = sharding.dense_pairs(b, h, world, r)
            seen.extend(range(s, e))
        assert seen == list(range(b * h))
    lens = list(np.random.default_rng(1).integers(1, 1000, size=37))
    owned = sharding.balance_sequences(lens, world)
    assert sorted(i for o in owned for i in o) == list(range(37))
