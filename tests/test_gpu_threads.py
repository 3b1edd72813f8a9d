"""The C ABI's threading contract on the GPU: calls are stateless and may come
from any host thread.  Four host threads each run decode steps on their own
stream and pool (the first calls of every kernel instance race on the
library's one-time per-device set-up), and every result equals the same steps
run from one thread."""
from __future__ import annotations

import threading

import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128


def _work(seed, mode):
    from gdn_b200 import NVFP4StatePool, workloads
    B = 32
    pool = NVFP4StatePool.zeros(B, HV, D, "cuda", scale_mode=mode)
    pool.load_fp32(workloads.initial_states(B, HV, D, seed=seed).cuda())
    x = workloads.decode_steps(B, 3, HK, HV, D, seed=seed + 100, device="cuda")
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    return pool, x, slot


def _run(pool, x, slot, debug):
    from gdn_b200 import ops
    outs = []
    for t in range(3):
        y = torch.empty((slot.numel(), HV, D, D), device="cuda") if debug else None
        outs.append(ops.decode(x["q"][t], x["k"][t], x["v"][t], x["g"][t], x["beta"][t], slot, pool, debug_y=y))
    return outs


def test_decode_from_four_host_threads(cuda):
    from gdn_b200 import ops
    # four different kernel instances (scale mode x debug), one per thread
    cfg = [(1, 0, False), (2, 1, False), (3, 0, True), (4, 1, True)]
    work = [_work(seed, mode) for seed, mode, _ in cfg]
    single = []
    for (seed, mode, dbg), (pool, x, slot) in zip(cfg, work):
        p2, _, _ = _work(seed, mode)
        single.append((_run(p2, x, slot, dbg), p2))
    torch.cuda.synchronize()

    results = [None] * 4
    errors = []
    start = threading.Barrier(4)

    def body(i):
        try:
            s = torch.cuda.Stream()
            pool, x, slot = work[i]
            with torch.cuda.stream(s):
                start.wait()
                outs = _run(pool, x, slot, cfg[i][2])
            s.synchronize()
            results[i] = outs
        except Exception as exc:  # surfaced below
            errors.append(exc)

    threads = [threading.Thread(target=body, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    for i in range(4):
        (ref_outs, ref_pool), (pool, _, _) = single[i], work[i]
        for a, b in zip(results[i], ref_outs):
            assert torch.equal(a, b)
        assert torch.equal(pool.codes, ref_pool.codes) and torch.equal(pool.scales, ref_pool.scales)
        assert torch.equal(pool.gscale, ref_pool.gscale)
    assert ops.device_status(clear=True) == 0
