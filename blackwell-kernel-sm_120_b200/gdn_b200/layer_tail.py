"""The step after the recurrent update in a tensor-parallel GDN layer: the
out-projection of the gated-RMS-normed attention output and the all-reduce
that sums it over the ranks.

vLLM's GDN layer ends in a row-parallel out-projection.  Under tensor
parallelism rank r holds the normed output of its own value heads,
o_r [B, HV/n * D], and the matching column block W_r [hidden, HV/n * D] of
W_out [hidden, HV * D]; the layer output is y = sum_r o_r W_r^T, one GEMM per
rank followed by one sum all-reduce.  The reference's patched layer ends in the
same projection (src/ops/qwen35_gdn_patch.py:118-121).

The GEMM is a plain library GEMM (cuBLAS through torch.matmul, bf16 in, fp32
accumulation); the all-reduce is NCCL's over NVLink / NVSwitch (in-switch
reduction when NCCL selects NVLS) or, with `allreduce=` a
gdn_b200.peer_allreduce.PeerAllReduce, this library's one-kernel all-reduce
over peer memory.  At the decode shapes of this layer the
all-reduce dominates: batch 1024 x hidden 2048 bf16 is 4 MiB per rank, several
microseconds over NVLink, against ~1.5 microseconds of tensor-core work for
the GEMM at TP 8 -- so a fused GEMM + reduce kernel could hide little more than
the GEMM.  The norm before the projection is fused into the decode kernel
(gdn_b200.ops.decode, norm_weight / gate_z).

These functions are plain torch calls: they run wherever the tensors live (the
process-group tests run them on CPU under gloo); the decode they follow
requires the CUDA library.
"""
from __future__ import annotations

import torch

from . import ops, sharding


def shard_out_proj(w_out: torch.Tensor, num_v_heads: int, num_k_heads: int, head_dim: int, rank: int,
                   world: int) -> torch.Tensor:
    """Rank `rank`'s column block of W_out [hidden, num_v_heads * head_dim]:
    the columns of its value heads under gdn_b200.sharding.shard_heads, as a
    contiguous [hidden, num_v_heads / world * head_dim] tensor."""
    if w_out.dim() != 2 or w_out.shape[1] != num_v_heads * head_dim:
        raise ValueError(f"W_out must be [hidden, {num_v_heads * head_dim}], got {tuple(w_out.shape)}")
    hv, _ = sharding.shard_heads(num_v_heads, num_k_heads, rank, world)
    return w_out[:, hv.start * head_dim:hv.stop * head_dim].contiguous()


def _group_size(group) -> int:
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def out_projection(o: torch.Tensor, w_shard: torch.Tensor, out: torch.Tensor | None = None,
                   group=None, allreduce=None) -> torch.Tensor:
    """y = sum over the ranks of group of o.reshape(B, -1) @ w_shard^T.

    o: [B, HV/n, D] (or [B, HV/n * D]) this rank's attention output; w_shard:
    [hidden, HV/n * D] from shard_out_proj, same dtype.  Returns (or fills) out
    [B, hidden].  Every rank of the group must call it with the same B and
    hidden (it issues one all-reduce when the group has more than one rank):
    NCCL's, or the callable `allreduce` (a PeerAllReduce over the same ranks),
    which sums in place.
    """
    B = o.shape[0]
    o2 = o.reshape(B, -1)
    if w_shard.dim() != 2 or o2.shape[1] != w_shard.shape[1]:
        raise ValueError(f"o has {o2.shape[1]} features per row, W shard expects {tuple(w_shard.shape)}")
    if o2.dtype != w_shard.dtype or o2.device != w_shard.device:
        raise ValueError("o and the W shard must share dtype and device")
    if out is None:
        out = torch.empty((B, w_shard.shape[0]), dtype=o2.dtype, device=o2.device)
    elif out.shape != (B, w_shard.shape[0]) or out.dtype != o2.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [B, hidden] tensor of o's dtype")
    torch.matmul(o2, w_shard.t(), out=out)
    if allreduce is not None:
        allreduce(out, out=out)
    elif _group_size(group) > 1:
        import torch.distributed as dist
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out


def decode_layer(q, k, v, g, beta, slot_idx, pool, w_shard: torch.Tensor, norm_weight: torch.Tensor,
                 gate_z: torch.Tensor | None = None, *, out: torch.Tensor | None = None,
                 attn_out: torch.Tensor | None = None, group=None, allreduce=None, norm_eps: float = 1e-6,
                 norm_activation: str = "silu", **decode_kwargs) -> torch.Tensor:
    """One decode step of a tensor-parallel GDN layer from its projections to
    its output: the fused recurrent update with vLLM's gated RMS norm
    (gdn_b200.ops.decode with norm_weight / gate_z; its other keyword
    arguments, such as the fused gating, pass through), then the out-projection
    and the all-reduce over `group`.  Returns y [B, hidden]; attn_out, when
    given, receives the normed attention output [B, HV/n, D]."""
    o = ops.decode(q, k, v, g, beta, slot_idx, pool, out=attn_out, norm_weight=norm_weight, gate_z=gate_z,
                   norm_eps=norm_eps, norm_activation=norm_activation, **decode_kwargs)
    return out_projection(o, w_shard, out=out, group=group, allreduce=allreduce)
