"""GPU checks of the step after the path (gdn_b200.layer_tail): the decode with
vLLM's fused gated RMS norm, then the row-parallel out-projection.

* decode_layer's attention output and pool bytes equal a plain fused-norm
  decode's, and its projection equals that output times W_out^T in fp32 torch
  to bf16 rounding (cuBLAS accumulates in fp32; y is stored as bf16).
* Tensor parallelism emulated in one process: the value heads split over 2 and
  4 shards (each with its own pool, key heads, gates and W_out column block)
  and the partial projections summed give the unsharded layer output.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D, HIDDEN = 16, 32, 128, 2048


def _setup(B, seed=11):
    from gdn_b200 import workloads
    states = workloads.initial_states(B, HV, D, std=0.02, seed=seed)
    x = {k: t[0] for k, t in workloads.decode_steps(B, 1, HK, HV, D, seed=seed + 1, device="cuda").items()}
    gen = torch.Generator().manual_seed(seed + 2)
    z = torch.randn((B, HV, D), generator=gen).to(torch.bfloat16).cuda()
    nw = (1.0 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16).cuda()
    w_out = (torch.randn((HIDDEN, HV * D), generator=gen) / (HV * D) ** 0.5).to(torch.bfloat16).cuda()
    slot = torch.randperm(B, generator=gen).to(torch.int32).cuda()
    return states, x, z, nw, w_out, slot


def _pool(states, heads=slice(None)):
    from gdn_b200 import NVFP4StatePool
    s = states[:, heads].contiguous()
    p = NVFP4StatePool.zeros(s.shape[0], s.shape[1], D, "cuda", scale_mode=1)
    p.load_fp32(s.cuda())
    return p


def _close(y, ref):
    err = (y.float() - ref).abs()
    scale = float(ref.abs().max())
    assert float(err.max()) <= 1.6e-2 * scale, (float(err.max()), scale)
    assert float((err > 1e-2 * ref.abs() + 2e-3 * scale).float().mean()) < 1e-3


@pytest.mark.parametrize("B", [8, 256])
def test_decode_layer_matches_decode_then_projection(cuda, B):
    from gdn_b200 import layer_tail, ops
    states, x, z, nw, w_out, slot = _setup(B)
    p1, p2 = _pool(states), _pool(states)
    args = (x["q"], x["k"], x["v"], x["g"], x["beta"], slot)
    o_ref = ops.decode(*args, p1, norm_weight=nw, gate_z=z)
    attn = torch.empty((B, HV, D), dtype=torch.bfloat16, device="cuda")
    y = layer_tail.decode_layer(*args, p2, w_out, nw, z, attn_out=attn)
    torch.cuda.synchronize()
    assert y.shape == (B, HIDDEN) and y.dtype == torch.bfloat16
    assert torch.equal(attn, o_ref)
    assert torch.equal(p1.codes, p2.codes) and torch.equal(p1.scales, p2.scales) and torch.equal(p1.gscale, p2.gscale)
    _close(y, o_ref.float().reshape(B, -1) @ w_out.float().t())
    assert ops.device_status(clear=True) == 0


@pytest.mark.parametrize("world", [2, 4])
def test_value_head_shards_sum_to_the_layer(cuda, world):
    from gdn_b200 import layer_tail, ops, sharding
    B = 64
    states, x, z, nw, w_out, slot = _setup(B, seed=23)
    full = layer_tail.decode_layer(x["q"], x["k"], x["v"], x["g"], x["beta"], slot, _pool(states), w_out, nw, z)
    total = torch.zeros((B, HIDDEN), dtype=torch.float32, device="cuda")
    for r in range(world):
        hv, hk = sharding.shard_heads(HV, HK, r, world)
        w_r = layer_tail.shard_out_proj(w_out, HV, HK, D, r, world)
        y_r = layer_tail.decode_layer(x["q"][:, hk.as_slice()], x["k"][:, hk.as_slice()], x["v"][:, hv.as_slice()],
                                      x["g"][:, hv.as_slice()].contiguous(), x["beta"][:, hv.as_slice()].contiguous(),
                                      slot, _pool(states, hv.as_slice()), w_r, nw, z[:, hv.as_slice()])
        total += y_r.float()
    torch.cuda.synchronize()
    _close(total.to(torch.bfloat16), full.float())
    assert ops.device_status(clear=True) == 0
