"""Multi-rank host logic on CPU: two gloo ranks split sequences and heads
exactly as the GPU runs do (every tile owned by one rank, GQA groups kept
whole) and agree on the max-over-ranks time."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HV, HK, N_SEQ = 32, 16, 1027


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q):
    import sys
    import pathlib
    root = pathlib.Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "blackwell-kernel-sm_120_b200"))
    from gdn_b200 import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        seq = sharding.shard_sequences(N_SEQ, rank, world)
        hv, hk = sharding.shard_heads(HV, HK, rank, world)
        # every value head's key head lies in this rank's key-head shard
        group = HV // HK
        assert all(hk.start <= h // group < hk.stop for h in range(hv.start, hv.stop))
        owned = torch.zeros(N_SEQ * HV, dtype=torch.int32)
        for b in range(seq.start, seq.stop):
            owned[b * HV:(b + 1) * HV] += 1
        dist.all_reduce(owned)
        heads = torch.zeros(HV, dtype=torch.int32)
        heads[hv.as_slice()] += 1
        dist.all_reduce(heads)
        t = sharding.max_over_ranks(1.5 + rank)
        q.put((rank, int(owned.min()), int(owned.max()), int(heads.min()), int(heads.max()), t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_rank_sharding(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, omin, omax, hmin, hmax, t in res:
        assert (omin, omax) == (1, 1)   # every (sequence, head) tile owned exactly once
        assert (hmin, hmax) == (1, 1)   # every value head owned exactly once
        assert t == 1.5 + (world - 1)   # max over ranks


def test_shard_edges():
    import sys
    import pathlib
    sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent.parent / "blackwell-kernel-sm_120_b200"))
    from gdn_b200 import sharding
    sizes = [sharding.shard_sequences(10, r, 4).size for r in range(4)]
    assert sizes == [3, 3, 2, 2]
    assert sharding.shard_sequences(0, 0, 2).size == 0
    with pytest.raises(ValueError):
        sharding.shard_heads(32, 16, 0, 3)
    with pytest.raises(ValueError):
        sharding.shard_sequences(5, 2, 2)
    assert sharding.shard_heads(32, 16, 7, 8) == (sharding.Shard(28, 32), sharding.Shard(14, 16))
