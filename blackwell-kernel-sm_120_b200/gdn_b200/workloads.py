"""Seeded synthetic inputs with the shapes and distributions of the GDN
workloads (no public dataset is involved):

  q, k, v  bf16 ~ N(0, 1); q and k L2-normalised per head in fp32 before the cast
  beta     sigmoid(N(0, 1)) per token and value head (fp32)
  g        -softplus(N(0, 1) + 2) per token and value head (fp32 log decay)
  state    fp32 N(0, 0.02) per element, quantised into the NVFP4 pool

Generated with a CPU torch.Generator, then copied to the device, so the same
seed gives the same tensors on every machine.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

# Shapes of the Qwen3.5-style linear-attention layer used throughout.
NUM_K_HEADS = 16
NUM_V_HEADS = 32
HEAD_DIM = 128


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def token_inputs(n_tokens: int, hk: int = NUM_K_HEADS, hv: int = NUM_V_HEADS, d: int = HEAD_DIM,
                 seed: int = 0, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """q, k [n, hk, d] bf16; v [n, hv, d] bf16; g, beta [n, hv] fp32."""
    gen = _gen(seed)
    q = torch.randn((n_tokens, hk, d), generator=gen, dtype=torch.float32)
    k = torch.randn((n_tokens, hk, d), generator=gen, dtype=torch.float32)
    v = torch.randn((n_tokens, hv, d), generator=gen, dtype=torch.float32)
    q = F.normalize(q, dim=-1)
    k = F.normalize(k, dim=-1)
    beta = torch.sigmoid(torch.randn((n_tokens, hv), generator=gen, dtype=torch.float32))
    g = -F.softplus(torch.randn((n_tokens, hv), generator=gen, dtype=torch.float32) + 2.0)
    out = {"q": q.to(torch.bfloat16), "k": k.to(torch.bfloat16), "v": v.to(torch.bfloat16), "g": g, "beta": beta}
    return {name: t.to(device) for name, t in out.items()}


def decode_steps(batch: int, steps: int, hk: int = NUM_K_HEADS, hv: int = NUM_V_HEADS, d: int = HEAD_DIM,
                 seed: int = 0, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """Inputs for `steps` consecutive decode tokens of `batch` sequences:
    q, k [steps, batch, hk, d]; v [steps, batch, hv, d]; g, beta [steps, batch, hv]."""
    t = token_inputs(steps * batch, hk, hv, d, seed, device)
    return {name: x.reshape(steps, batch, *x.shape[1:]) for name, x in t.items()}


def initial_states(n: int, hv: int = NUM_V_HEADS, d: int = HEAD_DIM, std: float = 0.02, seed: int = 1,
                   device: str | torch.device = "cpu") -> torch.Tensor:
    """fp32 states [n, hv, d, d] ~ N(0, std)."""
    gen = _gen(seed)
    return (torch.randn((n, hv, d, d), generator=gen, dtype=torch.float32) * std).to(device)


def varlen_lengths(n: int, lo: int, hi: int, seed: int = 2) -> list[int]:
    """n sequence lengths uniform in [lo, hi]."""
    gen = _gen(seed)
    return torch.randint(lo, hi + 1, (n,), generator=gen).tolist()


def slot_permutation(n: int, num_slots: int, seed: int = 3) -> torch.Tensor:
    """n distinct slots drawn from a seeded random permutation of num_slots."""
    gen = _gen(seed)
    return torch.randperm(num_slots, generator=gen)[:n].to(torch.int32)
