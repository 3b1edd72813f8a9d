"""How the GDN work splits across GPUs (one process per GPU, no collective on
the data path).

* Sequences (data parallel): every (sequence, value head) tile is independent,
  so rank r owns a contiguous block of sequences and its own pool slots.
* Value heads (tensor parallel, as vLLM shards the layer): rank r owns value
  heads [r HV/n, (r+1) HV/n) and the key heads they read,
  [r HK/n, (r+1) HK/n) -- the GQA group (HV/HK value heads per key head) never
  straddles two ranks when n divides HK.

The only cross-rank communication is host-side bookkeeping: a barrier around
timed regions and a max-reduction of the per-rank times.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start

    def as_slice(self) -> slice:
        return slice(self.start, self.stop)


def shard_sequences(num_seqs: int, rank: int, world: int) -> Shard:
    """Contiguous block of sequences for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(num_seqs, world)
    start = rank * base + min(rank, extra)
    return Shard(start, start + base + (1 if rank < extra else 0))


def shard_heads(num_v_heads: int, num_k_heads: int, rank: int, world: int) -> tuple[Shard, Shard]:
    """(value-head shard, key-head shard) of `rank` under tensor parallelism."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if num_v_heads % num_k_heads:
        raise ValueError("value heads must be a multiple of key heads")
    if num_k_heads % world:
        raise ValueError(f"{world} ranks do not divide {num_k_heads} key heads")
    hv, hk = num_v_heads // world, num_k_heads // world
    return Shard(rank * hv, (rank + 1) * hv), Shard(rank * hk, (rank + 1) * hk)


def max_over_ranks(value: float, group=None) -> float:
    """Max of a per-rank float over the process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
