"""GPU tests of the record pool layout (gdn_decode_params.pool_tile_stride):
every (slot, head) tile one 9232-byte record of a single uint8 tensor, the
form a serving engine's per-layer state cache takes.  Decode and prefill on a
record pool write the same output and state bytes as on the dense pool."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128


def _twin(n_slots, slot, mode, seed):
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(slot.numel(), HV, D, seed=seed).cuda()
    dense = NVFP4StatePool.zeros(n_slots, HV, D, "cuda", scale_mode=mode)
    dense.load_fp32(states, slot)
    rec = NVFP4StatePool.zeros_records(n_slots, HV, "cuda", scale_mode=mode)
    rec.load_fp32(states, slot)
    return dense, rec


def _same(dense, rec):
    assert torch.equal(dense.codes, rec.codes)
    assert torch.equal(dense.scales, rec.scales)
    assert torch.equal(dense.gscale.view(torch.int32), rec.gscale.contiguous().view(torch.int32))


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_on_record_pool(cuda, mode):
    from gdn_b200 import ops, workloads
    B, S = 64, 160
    slot = workloads.slot_permutation(B, S, seed=61).cuda()
    dense, rec = _twin(S, slot, mode, seed=62)  # distinct slots: one state each
    _same(dense, rec)
    slot[5] = -1  # padding in the decode: that sequence's slot stays as it is
    x = workloads.decode_steps(B, 3, HK, HV, D, seed=63, device="cuda")
    for t in range(3):
        args = (x["q"][t], x["k"][t], x["v"][t], x["g"][t], x["beta"][t], slot)
        o1 = ops.decode(*args, dense)
        o2 = ops.decode(*args, rec)
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        _same(dense, rec)
    assert ops.device_status(clear=True) == 0


def test_prefill_on_record_pool(cuda):
    from gdn_b200 import ops, workloads
    lengths = [70, 1, 129]
    N, S = len(lengths), 9
    slot = torch.tensor([7, 2, 4], dtype=torch.int32, device="cuda")
    dense, rec = _twin(S, slot, 1, seed=64)
    x = workloads.token_inputs(sum(lengths), HK, HV, D, seed=65, device="cuda")
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    has = torch.tensor([True, False, True], device="cuda")
    o1 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu, pool=dense, slot_idx=slot, has_initial_state=has)
    o2 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu, pool=rec, slot_idx=slot, has_initial_state=has)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    _same(dense, rec)
    # record bytes outside the three fields stay zero
    assert int(rec.storage[..., 9220:].count_nonzero()) == 0
