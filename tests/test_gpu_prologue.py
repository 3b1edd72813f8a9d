"""GPU checks of the fused prologue of the decode and prefill kernels (gdn_decode
and gdn_prefill through the C ABI): the gating g = -exp(A_log) softplus(a +
dt_bias), beta = sigmoid(b) computed in the kernel from the gate projections,
and the in-kernel unit-L2 scaling of q and k -- vLLM's
fused_sigmoid_gating_delta_rule_update(use_qk_l2norm_in_kernel) contract.

* Gating: the fused step equals the same step fed with g and beta computed by
  torch, up to the last bits of exp / log1p (outputs and states agree to
  fp32 rounding; requantised codes may differ only where that crosses a
  rounding boundary).
* L2 norm: against the unquantised f64 recurrence started from the same
  (dequantised) pool state with exactly normalised q and k, the outputs agree
  to bf16 output rounding.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128
QS = 1.0 / np.sqrt(D)


def _pool(n_slots, mode, seed=3):
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(n_slots, HV, D, std=0.02, seed=seed)
    pool = NVFP4StatePool.zeros(n_slots, HV, D, "cuda", scale_mode=mode)
    pool.load_fp32(states.cuda())
    return pool


def _gates(B, seed=5):
    gen = torch.Generator().manual_seed(seed)
    a = (torch.randn((B, HV), generator=gen) * 2.0).to(torch.bfloat16).cuda()
    b = torch.randn((B, HV), generator=gen).to(torch.bfloat16).cuda()
    A_log = torch.log(torch.empty(HV).uniform_(1.0, 16.0, generator=gen)).cuda()
    dt_bias = (torch.randn(HV, generator=gen) * 0.5).cuda()
    return a, b, A_log, dt_bias


def _qkv(B, seed=6):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn((B, HK, D), generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn((B, HK, D), generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn((B, HV, D), generator=gen).to(torch.bfloat16).cuda()
    return q, k, v


@pytest.mark.parametrize("mode", [0, 1])
def test_fused_gating_matches_host_gating(cuda, mode):
    from gdn_b200 import ops
    B = 8
    pool1, pool2 = _pool(10, mode), _pool(10, mode)
    slot = torch.tensor([3, 0, 9, 1, 4, 7, 2, 8], dtype=torch.int32, device="cuda")
    q, k, v = _qkv(B)
    k = F.normalize(k.float(), dim=-1).to(torch.bfloat16)  # keep the state bounded, as the model does
    q = F.normalize(q.float(), dim=-1).to(torch.bfloat16)
    a, b, A_log, dt_bias = _gates(B)
    g = -torch.exp(A_log) * F.softplus(a.float() + dt_bias)
    beta = torch.sigmoid(b.float())
    o1 = ops.decode(q, k, v, g, beta, slot, pool1)
    o2 = ops.decode(q, k, v, None, None, slot, pool2, A_log=A_log, dt_bias=dt_bias, gate_a=a, gate_b=b)
    torch.cuda.synchronize()
    o1f, o2f = o1.float(), o2.float()
    assert float((o1f - o2f).abs().max()) <= 1e-2 * float(o1f.abs().max())
    assert float((o1 == o2).float().mean()) > 0.99
    s1, s2 = pool1.dequantize(), pool2.dequantize()
    assert float((s1 - s2).abs().max()) <= 2e-2 * float(s1.abs().max())
    assert float((pool1.codes != pool2.codes).float().mean()) < 1e-3
    # the slots no sequence uses are untouched
    for s in (5, 6):
        assert torch.equal(pool1.codes[s], pool2.codes[s])


@pytest.mark.parametrize("mode", [0, 1])
def test_fused_l2norm_against_f64(cuda, mode):
    from gdn_b200 import ops
    from oracle import bindings as ob
    B = 4
    pool = _pool(4, mode, seed=11)
    slot = torch.tensor([2, 0, 3, 1], dtype=torch.int32, device="cuda")
    S0 = pool.dequantize().cpu().numpy().astype(np.float64)
    q, k, v = _qkv(B, seed=12)  # raw: not normalised
    a, b, A_log, dt_bias = _gates(B, seed=13)
    o = ops.decode(q, k, v, None, None, slot, pool, A_log=A_log, dt_bias=dt_bias, gate_a=a, gate_b=b,
                   qk_l2norm=True)
    torch.cuda.synchronize()
    g = (-torch.exp(A_log.double()) * F.softplus(a.double() + dt_bias.double())).cpu().numpy()
    beta = torch.sigmoid(b.double()).cpu().numpy()
    qn = F.normalize(q.double(), dim=-1, eps=0.0).cpu().numpy()
    kn = F.normalize(k.double(), dim=-1, eps=0.0).cpu().numpy()
    vv = v.double().cpu().numpy()
    o_np = o.float().cpu().numpy()
    slot_np = slot.cpu().numpy()
    for bi in range(B):
        for h in range(HV):
            hk = h // (HV // HK)
            o_ref, _ = ob.recurrent_f64(S0[slot_np[bi], h], qn[bi:bi + 1, hk], kn[bi:bi + 1, hk], vv[bi:bi + 1, h],
                                        g[bi:bi + 1, h], beta[bi:bi + 1, h], QS)
            err = np.abs(o_np[bi, h] - o_ref[0])
            assert (err <= 8e-3 * np.abs(o_ref[0]) + 2e-3 * np.abs(o_ref[0]).max()).all(), (bi, h, err.max())


def test_fused_prologue_argument_errors(cuda):
    from gdn_b200 import ops
    B = 2
    pool = _pool(2, 1)
    slot = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    q, k, v = _qkv(B)
    a, b, A_log, dt_bias = _gates(B)
    with pytest.raises(ValueError):
        ops.decode(q, k, v, None, None, slot, pool, A_log=A_log, dt_bias=dt_bias, gate_a=a, gate_b=None)
    with pytest.raises(ValueError):
        ops.decode(q, k, v, None, None, slot, pool)  # neither g / beta nor the gate inputs


@pytest.mark.parametrize("mode", [0, 1])
def test_prefill_fused_gating_matches_host_gating(cuda, mode):
    """The chunked prefill with g and beta computed in the kernel from the gate
    projections equals the prefill fed with torch's g and beta, up to the last
    bits of exp / log1p: outputs to bf16 rounding, final states to fp32 rounding."""
    from gdn_b200 import ops, workloads
    lengths = [70, 1, 200, 64, 129]
    T = sum(lengths)
    x = workloads.token_inputs(T, HK, HV, D, seed=12, device="cuda")
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    a, b, A_log, dt_bias = _gates(T, seed=13)
    g = -torch.exp(A_log) * F.softplus(a.float() + dt_bias)
    beta = torch.sigmoid(b.float())
    slots = torch.tensor([4, 0, 2, 6, 1], dtype=torch.int32, device="cuda")
    has = torch.tensor([True, False, True, True, False], device="cuda")
    pool1, pool2 = _pool(8, mode), _pool(8, mode)
    o1 = ops.prefill(x["q"], x["k"], x["v"], g, beta, cu, pool=pool1, slot_idx=slots, has_initial_state=has)
    o2 = ops.prefill(x["q"], x["k"], x["v"], None, None, cu, pool=pool2, slot_idx=slots, has_initial_state=has,
                     A_log=A_log, dt_bias=dt_bias, gate_a=a, gate_b=b)
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 0
    o1f, o2f = o1.float(), o2.float()
    assert float((o1f - o2f).abs().max()) <= 1e-2 * float(o1f.abs().max())
    assert float((o1 == o2).float().mean()) > 0.99
    s1, s2 = pool1.dequantize(), pool2.dequantize()
    assert float((s1 - s2).abs().max()) <= 2e-2 * float(s1.abs().max())
    # the slots no sequence uses are untouched
    for s in (3, 5, 7):
        assert torch.equal(pool1.codes[s], pool2.codes[s])


def test_prefill_fused_gating_argument_errors(cuda):
    import ctypes
    from gdn_b200 import _capi, ops, workloads
    x = workloads.token_inputs(16, HK, HV, D, seed=1, device="cuda")
    cu = torch.tensor([0, 16], dtype=torch.int32, device="cuda")
    a, b, A_log, dt_bias = _gates(16)
    with pytest.raises(ValueError):
        ops.prefill(x["q"], x["k"], x["v"], None, None, cu, A_log=A_log, gate_a=a, gate_b=b)  # no dt_bias
    with pytest.raises(ValueError):
        ops.prefill(x["q"], x["k"], x["v"], None, None, cu, A_log=A_log, dt_bias=dt_bias, gate_a=a)  # no gate_b
    # C ABI: A_log without gate_b is an argument error
    p = _capi.PrefillParams()
    p.num_seqs, p.num_k_heads, p.num_v_heads, p.head_dim = 1, HK, HV, D
    p.total_tokens = 16
    p.q, p.k, p.v = x["q"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr()
    p.cu_seqlens = cu.data_ptr()
    out = torch.empty((16, HV, D), dtype=torch.bfloat16, device="cuda")
    p.out = out.data_ptr()
    p.A_log, p.dt_bias, p.gate_a = A_log.data_ptr(), dt_bias.data_ptr(), a.data_ptr()
    assert _capi.lib.gdn_prefill(ctypes.byref(p), None) == _capi.GDN_ERR_ARGS
