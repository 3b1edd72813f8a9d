"""GPU checks of the decode kernel's fused epilogue: the gated RMS norm vLLM's
GDN layer applies to the attention output before its out-projection
(RMSNormGated, norm before gate, one group per head):

    out = x * rsqrt(mean_d(x^2) + eps) * weight * act(z),  x = the bf16 attention output

* The fused output equals that formula in fp32 torch applied to the plain
  decode's output, to bf16 rounding (the sum of squares is reduced in a
  different order).
* The state update is untouched: pool bytes equal the plain decode's.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128


def _setup(B, mode, seed=7):
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(B, HV, D, std=0.02, seed=seed)
    pools = []
    for _ in range(2):
        p = NVFP4StatePool.zeros(B, HV, D, "cuda", scale_mode=mode)
        p.load_fp32(states.cuda())
        pools.append(p)
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=seed + 1, device="cuda")
    gen = torch.Generator().manual_seed(seed + 2)
    z = torch.randn((B, HV, D), generator=gen).to(torch.bfloat16).cuda()
    w = (1.0 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16).cuda()
    slot = torch.randperm(B, generator=gen).to(torch.int32).cuda()
    return pools, x, z, w, slot


def _reference(o, z, w, eps, act):
    """vLLM's RMSNormGated.forward_static (norm_before_gate=True, group = head) in torch fp32."""
    xf = o.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    out = xf * torch.rsqrt(var + eps) * w.float()
    if z is not None:
        out = out * (torch.sigmoid(z.float()) if act == "sigmoid" else F.silu(z.float()))
    return out.to(torch.bfloat16)


@pytest.mark.parametrize("mode,act,gated", [(0, "silu", True), (1, "silu", True), (1, "sigmoid", True),
                                            (1, "silu", False)])
def test_fused_gated_norm_matches_torch(cuda, mode, act, gated):
    from gdn_b200 import ops
    B, eps = 24, 1e-6
    (p1, p2), x, z, w, slot = _setup(B, mode)
    args = (x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot)
    o_plain = ops.decode(*args, p1)
    o_fused = ops.decode(*args, p2, norm_weight=w, gate_z=z if gated else None, norm_eps=eps, norm_activation=act)
    torch.cuda.synchronize()
    ref = _reference(o_plain, z if gated else None, w, eps, act).float()
    got = o_fused.float()
    err = (got - ref).abs()
    assert float(err.max()) <= 1.6e-2 * float(ref.abs().max()), float(err.max())
    assert float((err > 1e-2 * ref.abs() + 1e-3).float().mean()) < 1e-3
    assert torch.equal(p1.codes, p2.codes) and torch.equal(p1.scales, p2.scales) and torch.equal(p1.gscale, p2.gscale)
    assert ops.device_status(clear=True) == 0


def test_fused_gated_norm_with_strided_gate_and_full_batch(cuda):
    """z as a view of a wider projection (vLLM's [T, HV * D] z slice) at batch 256."""
    from gdn_b200 import ops
    B = 256
    (p1, p2), x, _, w, slot = _setup(B, 1, seed=31)
    wide = torch.randn((B, 2 * HV * D), dtype=torch.float32, device="cuda").to(torch.bfloat16)
    z = wide[:, HV * D:].view(B, HV, D)
    args = (x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot)
    o_plain = ops.decode(*args, p1)
    o_fused = ops.decode(*args, p2, norm_weight=w, gate_z=z, norm_eps=1e-5)
    torch.cuda.synchronize()
    ref = _reference(o_plain, z, w, 1e-5, "silu").float()
    err = (o_fused.float() - ref).abs()
    assert float(err.max()) <= 1.6e-2 * float(ref.abs().max()), float(err.max())
    assert torch.equal(p1.codes, p2.codes)


def test_fused_gated_norm_argument_errors(cuda):
    from gdn_b200 import ops
    B = 4
    (p1, _), x, z, w, slot = _setup(B, 1)
    args = (x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, p1)
    with pytest.raises(ValueError):
        ops.decode(*args, norm_weight=w[:64], gate_z=z)
    with pytest.raises(ValueError):
        ops.decode(*args, norm_weight=w, gate_z=z, norm_activation="gelu")
    with pytest.raises(ValueError):
        ops.decode(*args, norm_weight=w, gate_z=z.float())
    from gdn_b200._capi import GdnError
    with pytest.raises(GdnError):
        ops.decode(*args, norm_weight=w, gate_z=z, norm_eps=0.0)  # rejected by the C ABI
