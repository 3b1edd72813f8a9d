"""GPU checks of the peer-memory all-reduce (gdn_b200.peer_allreduce), two
processes on two GPUs (skipped with fewer):

* the sum equals the fp32 sum of the ranks' bf16 vectors in rank order,
  rounded once -- bit for bit -- at 4 MiB and at a small ragged size, also in
  place and over 50 back-to-back calls;
* calls captured in a CUDA graph give the right sums on every replay (the
  kernel keeps its own call count);
* a wait for a rank that never calls gives up after its bound, sets the
  device status bit and returns (rank 1 skips the call; nothing faults).
"""
from __future__ import annotations

import os
import pathlib
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

PKG = pathlib.Path(__file__).resolve().parent.parent / "blackwell-kernel-sm_120_b200"
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _vec(count: int, seed: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(count, generator=gen).to(torch.bfloat16)


def _ref(count: int, seeds) -> torch.Tensor:
    acc = torch.zeros(count, dtype=torch.float32)
    for s in seeds:
        acc += _vec(count, s).float()
    return acc.to(torch.bfloat16)


def _worker(rank: int, port: int, q):
    sys.path.insert(0, str(PKG))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    out = {}
    try:
        from gdn_b200 import ops
        from gdn_b200.peer_allreduce import PeerAllReduce
        ops.device_status(clear=True, device=dev)
        ar = PeerAllReduce(1024 * 2048 * 2, device=dev)
        for count in (1024 * 2048, 8 * WORLD * 37):
            x = _vec(count, 100 * rank + count % 97).to(dev)
            ref = _ref(count, [100 * r + count % 97 for r in range(WORLD)])
            out[f"sum_{count}"] = torch.equal(ar(x).cpu(), ref)
            ar(x, out=x)
            out[f"inplace_{count}"] = torch.equal(x.cpu(), ref)
        count = 1024 * 2048
        x = _vec(count, 7 + rank).to(dev)
        ys = [torch.empty_like(x), torch.empty_like(x)]
        for i in range(50):
            ar(x, out=ys[i % 2])
        out["repeat"] = torch.equal(ys[1].cpu(), _ref(count, [7 + r for r in range(WORLD)]))
        # CUDA graph: two calls per replay, new inputs before each replay
        a, b = torch.empty_like(x), torch.empty_like(x)
        ya, yb = torch.empty_like(x), torch.empty_like(x)
        a.copy_(x)
        b.copy_(x)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                ar(a, out=ya)
                ar(b, out=yb)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        ok = True
        for rep in range(3):
            sa, sb = 1000 + 10 * rep, 2000 + 10 * rep
            a.copy_(_vec(count, sa + rank).to(dev))
            b.copy_(_vec(count, sb + rank).to(dev))
            g.replay()
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(ya.cpu(), _ref(count, [sa + r for r in range(WORLD)]))
            ok = ok and torch.equal(yb.cpu(), _ref(count, [sb + r for r in range(WORLD)]))
        del g
        out["graph"] = ok
        out["status_clean"] = ops.device_status(clear=True, device=dev) == 0
        ar.close()
        # a rank that never calls: the other's waits run out after 20 ms
        ar2 = PeerAllReduce(4096, device=dev, timeout_ns=20_000_000)
        if rank == 0:
            ar2(torch.ones(1024, dtype=torch.bfloat16, device=dev))
            torch.cuda.synchronize(dev)
        out["timeout_status"] = ops.device_status(clear=True, device=dev)
        ar2.close()
    except Exception as e:  # reported to the parent
        out["error"] = repr(e)
    finally:
        q.put((rank, out))
        dist.destroy_process_group()


def test_two_rank_peer_allreduce(cuda):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    for rank in range(WORLD):
        r = res[rank]
        assert "error" not in r, r
        for key in ("sum_2097152", "inplace_2097152", "sum_592", "inplace_592", "repeat", "graph", "status_clean"):
            assert r[key], (rank, key, r)
    assert res[0]["timeout_status"] & 0x1
    assert res[1]["timeout_status"] == 0
