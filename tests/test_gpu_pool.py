"""GPU tests of the runtime slot copies gdn_pool_gather / gdn_pool_scatter
(through the C ABI) against plain tensor indexing: byte-equal codes, scales
and global scales on a 2048-slot random permutation, with padding (negative
slots: gather zero-fills, scatter skips) and out-of-range slots (treated as
padding and reported through GDN_STATUS_BAD_SLOT)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

HV, D = 32, 128
BAD_SLOT = 0x2


def _random_pool(n_slots, seed):
    from gdn_b200 import NVFP4StatePool
    gen = torch.Generator().manual_seed(seed)
    p = NVFP4StatePool.zeros(n_slots, HV, D, "cuda")
    p.codes.copy_(torch.randint(0, 256, p.codes.shape, generator=gen, dtype=torch.uint8))
    p.scales.copy_(torch.randint(0, 256, p.scales.shape, generator=gen, dtype=torch.uint8))
    p.gscale.copy_(torch.rand(p.gscale.shape, generator=gen) + 0.5)
    return p


def test_gather_matches_indexing_on_a_random_permutation(cuda):
    from gdn_b200 import ops, workloads
    pool = _random_pool(2048, 1)
    slot = workloads.slot_permutation(512, 2048, seed=2).cuda()
    ops.device_status(clear=True)
    c, s, g = ops.pool_gather(pool, slot)
    idx = slot.long()
    assert torch.equal(c, pool.codes[idx])
    assert torch.equal(s, pool.scales[idx])
    assert torch.equal(g.view(torch.int32), pool.gscale[idx].view(torch.int32))
    assert ops.device_status(clear=True) == 0


def test_scatter_matches_index_put_on_a_random_permutation(cuda):
    from gdn_b200 import ops, workloads
    pool = _random_pool(2048, 3)
    expect = (pool.codes.clone(), pool.scales.clone(), pool.gscale.clone())
    src = _random_pool(512, 4)
    slot = workloads.slot_permutation(512, 2048, seed=5).cuda()
    ops.pool_scatter(pool, slot, src.codes, src.scales, src.gscale)
    idx = slot.long()
    expect[0][idx] = src.codes
    expect[1][idx] = src.scales
    expect[2][idx] = src.gscale
    torch.cuda.synchronize()
    assert torch.equal(pool.codes, expect[0])
    assert torch.equal(pool.scales, expect[1])
    assert torch.equal(pool.gscale.view(torch.int32), expect[2].view(torch.int32))


def test_padding_and_out_of_range_slots(cuda):
    from gdn_b200 import ops
    pool = _random_pool(16, 6)
    before = (pool.codes.clone(), pool.scales.clone(), pool.gscale.clone())
    slot = torch.tensor([3, -1, 16, 7, 1000], dtype=torch.int32, device="cuda")
    ops.device_status(clear=True)
    c, s, g = ops.pool_gather(pool, slot)
    for i, sl in ((0, 3), (3, 7)):
        assert torch.equal(c[i], pool.codes[sl]) and torch.equal(s[i], pool.scales[sl])
        assert torch.equal(g[i], pool.gscale[sl])
    for i in (1, 2, 4):  # padding and out of range: zero-filled
        assert int(c[i].count_nonzero()) == 0 and int(s[i].count_nonzero()) == 0
        assert int(g[i].count_nonzero()) == 0
    assert ops.device_status(clear=True) & BAD_SLOT

    src = _random_pool(5, 7)
    ops.pool_scatter(pool, slot, src.codes, src.scales, src.gscale)
    torch.cuda.synchronize()
    for sl in range(16):
        if sl in (3, 7):
            continue
        assert torch.equal(pool.codes[sl], before[0][sl]) and torch.equal(pool.scales[sl], before[1][sl])
        assert torch.equal(pool.gscale[sl], before[2][sl])
    assert torch.equal(pool.codes[3], src.codes[0]) and torch.equal(pool.codes[7], src.codes[3])
    assert ops.device_status(clear=True) & BAD_SLOT
    assert ops.device_status(clear=True) == 0


def test_gather_scatter_round_trip(cuda):
    from gdn_b200 import ops, workloads
    pool = _random_pool(2048, 8)
    other = _random_pool(2048, 9)
    slot = workloads.slot_permutation(300, 2048, seed=10).cuda()
    c, s, g = ops.pool_gather(pool, slot)
    ops.pool_scatter(other, slot, c, s, g)
    idx = slot.long()
    torch.cuda.synchronize()
    assert torch.equal(other.codes[idx], pool.codes[idx])
    assert torch.equal(other.scales[idx], pool.scales[idx])
    assert torch.equal(other.gscale[idx], pool.gscale[idx])
