"""The out-projection after the path, on CPU: the row-parallel projection of
gdn_b200.layer_tail summed by a gloo all-reduce over 2 and 4 ranks equals the
unsharded projection o W_out^T, and its argument checks raise."""
from __future__ import annotations

import os
import pathlib
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PKG = pathlib.Path(__file__).resolve().parent.parent / "blackwell-kernel-sm_120_b200"
HV, HK, D, HIDDEN, BATCH = 32, 16, 128, 256, 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    gen = torch.Generator().manual_seed(7)
    o = torch.randn((BATCH, HV, D), generator=gen, dtype=torch.float64)
    w = torch.randn((HIDDEN, HV * D), generator=gen, dtype=torch.float64) / (HV * D) ** 0.5
    return o, w


def _worker(rank: int, world: int, port: int, q):
    sys.path.insert(0, str(PKG))
    from gdn_b200 import layer_tail, sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        o, w = _inputs()
        hv, _ = sharding.shard_heads(HV, HK, rank, world)
        w_r = layer_tail.shard_out_proj(w, HV, HK, D, rank, world)
        y = layer_tail.out_projection(o[:, hv.as_slice()].contiguous(), w_r)
        q.put((rank, tuple(w_r.shape), y))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_out_projection(world):
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
    o, w = _inputs()
    ref = o.reshape(BATCH, -1) @ w.t()
    for rank, shape, y in res:
        assert shape == (HIDDEN, HV // world * D)
        # fp64 sums in a different order: equal to rounding
        torch.testing.assert_close(y, ref, rtol=1e-12, atol=1e-12)


def test_out_projection_single_process_and_errors():
    sys.path.insert(0, str(PKG))
    from gdn_b200 import layer_tail
    o, w = _inputs()
    y = layer_tail.out_projection(o, w)  # no process group: no all-reduce
    torch.testing.assert_close(y, o.reshape(BATCH, -1) @ w.t(), rtol=1e-12, atol=1e-12)
    out = torch.empty((BATCH, HIDDEN), dtype=torch.float64)
    assert layer_tail.out_projection(o, w, out=out) is out
    with pytest.raises(ValueError):
        layer_tail.out_projection(o[:, :16], w)                 # feature count
    with pytest.raises(ValueError):
        layer_tail.out_projection(o.float(), w)                 # dtype
    with pytest.raises(ValueError):
        layer_tail.out_projection(o, w, out=torch.empty((BATCH, HIDDEN + 1), dtype=torch.float64))
    with pytest.raises(ValueError):
        layer_tail.shard_out_proj(w[:, :100], HV, HK, D, 0, 2)
    with pytest.raises(ValueError):
        layer_tail.shard_out_proj(w, HV, HK, D, 0, 3)           # 3 ranks do not divide 16 key heads
