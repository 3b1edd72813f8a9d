"""vLLM 0.22 seam: the NVFP4 GDN kernels behind the calls vLLM's gated delta
net layer makes (vllm/model_executor/layers/mamba/gdn/qwen_gdn_linear_attn.py),
with the layer's recurrent state cache holding NVFP4 records instead of dense
[HV, V, K] states.

The state cache.  vLLM sizes a GDN layer's temporal state from the layer's
``get_state_shape`` / ``get_state_dtype`` (via MambaStateShapeCalculator /
MambaStateDtypeCalculator in mamba_utils) and allocates one tensor
[num_blocks, *shape] per layer.  ``state_shape`` / ``state_dtype`` below make
that tensor uint8 [num_blocks, HV, RECORD_BYTES]: one 9232-byte record per
(block, value head) holding the tile's E2M1 codes, its scale bytes and its fp32
global scale (gdn_b200.pool, record layout).  The kernels read and write those
records in place through gdn_decode_params.pool_tile_stride, so a decode step
touches 9.2 KB per head instead of 64 KB of fp32 state, and no dense copy of
the state exists at any point.

The calls, each with vLLM's own signature, dispatching on the cache's dtype
(uint8 records: NVFP4 in place; a floating cache: the dense states cross into
NVFP4 and back, for layers left on vLLM's layout):

* ``chunk_gated_delta_rule`` -- the ``ChunkGatedDeltaRule`` CustomOp forward
  (qwen_gdn_linear_attn.py:290-418).  _forward_core gathers the sequences'
  records (``ssm_state[idx].contiguous()``, rows without an initial state
  zeroed, which is the zero state), passes them as ``initial_state``, and
  writes the returned final state back with an index_put
  (qwen_gdn_linear_attn.py:1465-1487).  Here the prefill runs on that gathered
  copy in place and returns it.
* ``fused_sigmoid_gating_delta_rule_update`` -- the decode call of
  _forward_core (qwen_gdn_linear_attn.py:1490-1505): gating from A_log, a, b,
  dt_bias and the q/k L2 norm fused into the decode kernel; states updated in
  place at ``ssm_state_indices``.
* ``fused_recurrent_gated_delta_rule_packed_decode`` -- the packed decode of
  _forward_core_decode_non_spec (qwen_gdn_linear_attn.py:1592-1644): q, k and v
  are strided views of the packed projection rows, read without a copy.

State indices follow vLLM: an index <= 0 marks padding (block 0 is vLLM's null
block, fla/ops/fused_recurrent.py:295-299); its output row is zero and no state
is touched.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops
from ._capi import SCALE_FN448
from .pool import RECORD_BYTES, NVFP4StatePool

# NVFP4 scale mode of the state cache: E4M3 block scales up to 448 with a
# global scale of max |S| / (6 * 448).
SCALE_MODE = SCALE_FN448


def state_shape(num_v_heads_per_rank: int) -> tuple[int, int]:
    """Per-block shape of the NVFP4 temporal state: one record per value head."""
    return (num_v_heads_per_rank, RECORD_BYTES)


def state_dtype() -> torch.dtype:
    return torch.uint8


def is_record_cache(t: torch.Tensor | None) -> bool:
    return t is not None and t.dtype == torch.uint8 and t.dim() == 3 and t.shape[-1] == RECORD_BYTES


def l2norm(x: torch.Tensor) -> torch.Tensor:
    """x / sqrt(sum x^2 + 1e-6) per head in fp32, then bf16: vLLM/fla's l2norm
    and the decode kernel's fused q/k normalisation."""
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)


def _heads_view(t: torch.Tensor) -> torch.Tensor:
    """bf16 [n, H, D] with contiguous heads (a strided view passes through)."""
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1] or t.stride(0) % 8:
        t = t.contiguous()
    return t


def _to_pool(states_vk: torch.Tensor, scale_mode: int = SCALE_MODE) -> NVFP4StatePool:
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
                           core_attn_out=None, scale_mode: int = SCALE_MODE):
    """Drop-in for vLLM's ChunkGatedDeltaRule forward on the NVFP4 prefill kernel.
    q, k [1, T, HK, D]; v [1, T, HV, D]; g, beta [1, T, HV]; initial_state
    [N, HV, RECORD_BYTES] uint8 records (updated in place and returned) or
    dense [N, HV, V, K].  Returns (o [1, T, HV, D], final_state)."""
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("expected packed varlen inputs of shape [1, T, H, D]")
    # the q/k L2 norm (use_qk_l2norm_in_kernel) runs inside the prefill kernel
    qs, ks, vs = (t.to(torch.bfloat16).contiguous() for t in (q[0], k[0], v[0]))
    l2 = bool(use_qk_l2norm_in_kernel)
    T = qs.shape[0]
    if cu_seqlens is None:
        cu_seqlens = torch.tensor([0, T], dtype=torch.int32, device=q.device)
    cu = cu_seqlens.to(torch.int32).contiguous()
    N = cu.numel() - 1
    gs = g[0].float().contiguous()
    bs = beta[0].float().contiguous()
    HV, D = vs.shape[1], qs.shape[2]
    final = None
    if is_record_cache(initial_state):
        # the gathered records of the N sequences: the prefill reads and
        # rewrites them in place (an all-zero record is the zero state)
        recs = initial_state if initial_state.is_contiguous() else initial_state.contiguous()
        pool = NVFP4StatePool.records(recs, scale_mode)
        slot = torch.arange(N, dtype=torch.int32, device=q.device)
        o = ops.prefill(qs, ks, vs, gs, bs, cu, pool=pool, slot_idx=slot,
                        has_initial_state=torch.ones(N, dtype=torch.bool, device=q.device), qk_l2norm=l2)
        final = recs
    elif initial_state is not None and initial_state.dtype == torch.uint8:
        # vLLM's kernel warm-up builds a zero [1, HV, V, K] state of the cache
        # dtype: a zero initial state, nothing to keep
        o = ops.prefill(qs, ks, vs, gs, bs, cu, qk_l2norm=l2)
        final = initial_state
    else:
        pool = slot = has = None
        if initial_state is not None or output_final_state:
            if initial_state is not None:
                pool = _to_pool(initial_state, scale_mode)
                has = torch.ones(N, dtype=torch.bool, device=q.device)
            else:
                pool = NVFP4StatePool.zeros(N, HV, D, q.device, scale_mode=scale_mode)
            slot = torch.arange(N, dtype=torch.int32, device=q.device)
        o = ops.prefill(qs, ks, vs, gs, bs, cu, pool=pool, slot_idx=slot, has_initial_state=has, qk_l2norm=l2)
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


def _slots(idx: torch.Tensor) -> torch.Tensor:
    """vLLM state indices -> kernel slots: <= 0 (padding, null block) -> -1."""
    idx = idx.reshape(-1)
    return torch.where(idx > 0, idx, torch.full_like(idx, -1)).to(torch.int32).contiguous()


def _decode(qs, ks, vs, A_log, a, b, dt_bias, cache, slot_idx, inplace: bool, qk_l2norm: bool, scale_mode: int,
            q_scale: float = 0.0, out=None):
    """One decode token per sequence.  cache: uint8 records [blocks, HV,
    RECORD_BYTES] or dense [blocks, HV, V, K].  Returns (o [B, HV, D], final)."""
    B = qs.shape[0]
    HV = vs.shape[1]
    gate = dict(A_log=A_log.float().contiguous(), dt_bias=dt_bias.float().contiguous(),
                gate_a=a.reshape(B, HV).to(torch.bfloat16).contiguous(),
                gate_b=b.reshape(B, HV).to(torch.bfloat16).contiguous(), qk_l2norm=qk_l2norm)
    idx = (slot_idx if slot_idx is not None else torch.arange(B, device=qs.device)).reshape(-1)
    valid = idx > 0 if slot_idx is not None else torch.ones(B, dtype=torch.bool, device=qs.device)
    if is_record_cache(cache):
        if inplace:
            pool = NVFP4StatePool.records(cache, scale_mode)
            slot = _slots(idx) if slot_idx is not None else idx.to(torch.int32)
            o = ops.decode(qs, ks, vs, None, None, slot, pool, out=out, q_scale=q_scale, **gate)
            return o, cache
        # out of place: run on a copy of the sequences' records
        recs = cache[idx.clamp(min=0).long()].contiguous()
        pool = NVFP4StatePool.records(recs, scale_mode)
        slot = torch.where(valid, torch.arange(B, device=qs.device), torch.full_like(idx, -1)).to(torch.int32)
        o = ops.decode(qs, ks, vs, None, None, slot, pool, out=out, q_scale=q_scale, **gate)
        recs[~valid] = 0
        return o, recs
    dense = cache[idx.clamp(min=0).long()]
    pool = _to_pool(dense, scale_mode)
    slot = torch.where(valid, torch.arange(B, device=qs.device), torch.full_like(idx, -1)).to(torch.int32)
    o = ops.decode(qs, ks, vs, None, None, slot, pool, out=out, q_scale=q_scale, **gate)
    new = _from_pool(pool, cache.dtype)
    if inplace:
        cache[idx[valid].long()] = new[valid]
        return o, cache
    final = torch.zeros_like(new)
    final[valid] = new[valid]
    return o, final


def fused_sigmoid_gating_delta_rule_update(A_log, a, b, dt_bias, q, k, v, beta: float = 1.0, threshold: float = 20.0,
                                           scale: float | None = None, initial_state=None,
                                           inplace_final_state: bool = True, cu_seqlens=None, ssm_state_indices=None,
                                           num_accepted_tokens=None, use_qk_l2norm_in_kernel: bool = False,
                                           is_kda: bool = False, scale_mode: int = SCALE_MODE):
    """Drop-in for vLLM's fused_sigmoid_gating_delta_rule_update with one
    token per sequence (fla/ops/fused_sigmoid_gating.py:181-270).  Returns
    (o [1, B, HV, V], final_state): the cache itself when updated in place,
    else a fresh tensor of the sequences' new states (row i = sequence i,
    padding rows zero) in the cache's layout."""
    if num_accepted_tokens is not None or is_kda:
        raise NotImplementedError("speculative and KDA decode are outside this kernel's scope")
    if beta != 1.0 or threshold != 20.0:
        raise NotImplementedError("the fused gating uses softplus with beta 1 and threshold 20")
    qs = _heads_view(q.reshape(-1, *q.shape[-2:]))
    ks = _heads_view(k.reshape(-1, *k.shape[-2:]))
    vs = _heads_view(v.reshape(-1, *v.shape[-2:]))
    o, final = _decode(qs, ks, vs, A_log, a, b, dt_bias, initial_state, ssm_state_indices, inplace_final_state,
                       use_qk_l2norm_in_kernel, scale_mode, q_scale=scale or 0.0)
    return o.unsqueeze(0), final


def fused_recurrent_gated_delta_rule_packed_decode(mixed_qkv, a, b, A_log, dt_bias, scale: float, initial_state, out,
                                                   ssm_state_indices, use_qk_l2norm_in_kernel: bool = False,
                                                   scale_mode: int = SCALE_MODE):
    """Drop-in for vLLM's packed decode (fla/ops/fused_recurrent.py:339-420):
    mixed_qkv [B, (2 HK + HV) D] rows of q | k | v, read in place as strided
    views; out [B, 1, HV, V] receives the outputs; the cache is updated in
    place at ssm_state_indices.  Returns (out, initial_state)."""
    B = mixed_qkv.shape[0]
    HV, D = out.shape[-2], out.shape[-1]
    HK = (mixed_qkv.shape[1] // D - HV) // 2
    rows = mixed_qkv if mixed_qkv.dtype == torch.bfloat16 else mixed_qkv.to(torch.bfloat16)
    if rows.stride(-1) != 1 or rows.stride(0) % 8:
        rows = rows.contiguous()
    qkv = rows.view(B, 2 * HK + HV, D) if rows.is_contiguous() else rows.unflatten(1, (2 * HK + HV, D))
    qs, ks, vs = qkv[:, :HK], qkv[:, HK:2 * HK], qkv[:, 2 * HK:]
    direct = out.dtype == torch.bfloat16 and out.is_contiguous()
    o, _ = _decode(qs, ks, vs, A_log, a, b, dt_bias, initial_state, ssm_state_indices, True,
                   use_qk_l2norm_in_kernel, scale_mode, q_scale=scale,
                   out=out.view(B, HV, D) if direct else None)
    if not direct:
        out.copy_(o.view(out.shape))
    return out, initial_state
