"""vLLM 0.22 seam: the NVFP4 GDN kernels behind the signatures vLLM's gated
delta net layer calls (vllm/model_executor/layers/mamba/gdn/qwen_gdn_linear_attn.py).

* ``chunk_gated_delta_rule`` -- same arguments and results as the
  ``ChunkGatedDeltaRule`` CustomOp forward (qwen_gdn_linear_attn.py:290-418):
  q, k [1, T, HK, K]; v [1, T, HV, V]; g, beta [1, T, HV]; initial_state
  [N, HV, V, K]; returns (o [1, T, HV, V], final_state [N, HV, V, K] or None).
* ``fused_sigmoid_gating_delta_rule_update`` -- the decode call of
  ``_forward_core`` (qwen_gdn_linear_attn.py:1492-1510): gating from A_log,
  a, b, dt_bias; states updated in place at ``ssm_state_indices`` (index < 0
  = padding, vLLM's PAD_SLOT_ID).

vLLM stores states as [V][K] (d_v rows); the kernels' NVFP4 tiles are S[K][V].
Dense states cross into NVFP4 (gdn_nvfp4_quantize_tiles) on the way in and
back (gdn_nvfp4_dequantize_tiles) on the way out, so vLLM's cache keeps its
own dtype; a cache that stays NVFP4 end to end needs vLLM's state-dtype hook
(mamba_utils) and is not wired here.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops
from .pool import NVFP4StatePool


def l2norm(x: torch.Tensor) -> torch.Tensor:
    """x / sqrt(sum x^2 + 1e-6) per head in fp32, then bf16: vLLM/fla's l2norm
    and the decode kernel's fused q/k normalisation."""
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)


def _to_pool(states_vk: torch.Tensor, scale_mode: int = 0) -> NVFP4StatePool:
    """[N, HV, V, K] dense states -> an NVFP4 pool with slots 0..N-1."""
    N, HV, V, K = states_vk.shape
    pool = NVFP4StatePool.zeros(N, HV, K, states_vk.device, scale_mode=scale_mode)
    pool.load_fp32(states_vk.transpose(-1, -2).float().contiguous())
    return pool


def _from_pool(pool: NVFP4StatePool, dtype: torch.dtype) -> torch.Tensor:
    """NVFP4 pool -> dense [N, HV, V, K] states."""
    return pool.dequantize().transpose(-1, -2).to(dtype).contiguous()


def chunk_gated_delta_rule(q, k, v, g, beta, initial_state, output_final_state: bool, cu_seqlens=None,
                           chunk_indices=None, chunk_offsets=None, use_qk_l2norm_in_kernel: bool = True,
                           core_attn_out=None, scale_mode: int = 0):
    """Drop-in for vLLM's ChunkGatedDeltaRule forward on the NVFP4 prefill kernel."""
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("expected packed varlen inputs of shape [1, T, H, D]")
    qs, ks, vs = q[0], k[0], v[0]
    if use_qk_l2norm_in_kernel:
        qs = l2norm(qs)
        ks = l2norm(ks)
    qs, ks, vs = (t.to(torch.bfloat16).contiguous() for t in (qs, ks, vs))
    T = qs.shape[0]
    if cu_seqlens is None:
        cu_seqlens = torch.tensor([0, T], dtype=torch.int32, device=q.device)
    cu = cu_seqlens.to(torch.int32).contiguous()
    N = cu.numel() - 1
    gs = g[0].float().contiguous()
    bs = beta[0].float().contiguous()
    pool = None
    slot = None
    has = None
    if initial_state is not None or output_final_state:
        if initial_state is not None:
            pool = _to_pool(initial_state, scale_mode)
            has = torch.ones(N, dtype=torch.bool, device=q.device)
        else:
            pool = NVFP4StatePool.zeros(N, vs.shape[1], qs.shape[2], q.device, scale_mode=scale_mode)
        slot = torch.arange(N, dtype=torch.int32, device=q.device)
    o = ops.prefill(qs, ks, vs, gs, bs, cu, pool=pool, slot_idx=slot, has_initial_state=has)
    final = None
    if output_final_state:
        final = _from_pool(pool, initial_state.dtype if initial_state is not None else torch.float32)
    o = o.unsqueeze(0)
    if core_attn_out is not None:
        co = core_attn_out.reshape(-1)
        co[: o.numel()].copy_(o.reshape(-1))
    return o, final


def gating(A_log: torch.Tensor, a: torch.Tensor, b: torch.Tensor, dt_bias: torch.Tensor):
    """g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b), both fp32 [T, HV]."""
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g.contiguous(), torch.sigmoid(b.float()).contiguous()


def fused_sigmoid_gating_delta_rule_update(A_log, a, b, dt_bias, q, k, v, initial_state, inplace_final_state=True,
                                           cu_seqlens=None, ssm_state_indices=None, num_accepted_tokens=None,
                                           use_qk_l2norm_in_kernel: bool = True, scale_mode: int = 0):
    """One decode token per sequence on the NVFP4 decode kernel; states in
    ``initial_state`` ([slots, HV, V, K]) are read and written at
    ``ssm_state_indices``.  Returns (o [1, B, HV, V], initial_state)."""
    if num_accepted_tokens is not None:
        raise NotImplementedError("speculative decoding is outside this kernel's scope")
    qs, ks, vs = q.reshape(-1, *q.shape[-2:]), k.reshape(-1, *k.shape[-2:]), v.reshape(-1, *v.shape[-2:])
    B = qs.shape[0]
    qs, ks, vs = (t.to(torch.bfloat16).contiguous() for t in (qs, ks, vs))
    idx = ssm_state_indices.to(torch.int64) if ssm_state_indices is not None else torch.arange(B, device=q.device)
    valid = idx >= 0
    dense = initial_state[idx.clamp(min=0)]
    pool = _to_pool(dense, scale_mode)
    slot = torch.where(valid, torch.arange(B, device=q.device), torch.full_like(idx, -1)).to(torch.int32)
    # gating and the q/k normalisation run inside the decode kernel
    o = ops.decode(qs, ks, vs, None, None, slot, pool, A_log=A_log.float().contiguous(),
                   dt_bias=dt_bias.float().contiguous(), gate_a=a.reshape(B, -1).to(torch.bfloat16),
                   gate_b=b.reshape(B, -1).to(torch.bfloat16), qk_l2norm=use_qk_l2norm_in_kernel)
    new = _from_pool(pool, initial_state.dtype)
    if inplace_final_state:
        initial_state[idx[valid]] = new[valid]
        return o.unsqueeze(0), initial_state
    # vLLM's out-of-place form: a fresh [B, HV, V, K] tensor of the states
    # after this token, row i for sequence i (padding rows zero)
    final = torch.zeros_like(new)
    final[valid] = new[valid]
    return o.unsqueeze(0), final
