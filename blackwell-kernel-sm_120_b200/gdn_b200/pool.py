"""Slot-indexed NVFP4 state pool for one GDN layer.

Layout (device memory, one pool per layer and per tensor-parallel shard):
  codes  [num_slots, HV, D, D/2]  uint8   E2M1 pairs, even element in the low nibble
  scales [num_slots, HV, D, D/16] uint8   E4M3-style scale per 16 contiguous d_v elements
  gscale [num_slots, HV]          float32 per-tile global scale

A state tile is S[k][v] (d_k rows, d_v contiguous), the reference's
orientation (src/kernel/gdn_state_update_ref.cu:58-66).  An all-zero pool is
the zero state (codes 0 decode to 0 whatever the scales).  At D = 128 one slot
of 32 heads is 294,912 B of codes and scales plus 128 B of global scales.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from ._capi import SCALE_FN448, SCALE_REF240


@dataclass
class NVFP4StatePool:
    codes: torch.Tensor
    scales: torch.Tensor
    gscale: torch.Tensor
    scale_mode: int = SCALE_REF240
    gscale_den: float = 0.0  # 0 -> 6 * saturation of the mode

    @classmethod
    def zeros(cls, num_slots: int, num_v_heads: int, head_dim: int = 128, device="cuda",
              scale_mode: int = SCALE_REF240, gscale_den: float = 0.0) -> "NVFP4StatePool":
        D = head_dim
        return cls(
            codes=torch.zeros((num_slots, num_v_heads, D, D // 2), dtype=torch.uint8, device=device),
            scales=torch.zeros((num_slots, num_v_heads, D, D // 16), dtype=torch.uint8, device=device),
            gscale=torch.zeros((num_slots, num_v_heads), dtype=torch.float32, device=device),
            scale_mode=scale_mode, gscale_den=gscale_den)

    @property
    def num_slots(self) -> int:
        return self.codes.shape[0]

    @property
    def num_v_heads(self) -> int:
        return self.codes.shape[1]

    @property
    def head_dim(self) -> int:
        return self.codes.shape[2]

    @property
    def gden(self) -> float:
        if self.gscale_den > 0:
            return self.gscale_den
        return 6.0 * (448.0 if self.scale_mode == SCALE_FN448 else 240.0)

    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel() + 4 * self.gscale.numel()

    def load_fp32(self, states: torch.Tensor, slots: torch.Tensor | None = None) -> None:
        """Quantise fp32 states [n, HV, D, D] into slots (default 0..n-1) with a
        fresh global scale per tile."""
        n = states.shape[0]
        D = self.head_dim
        codes, scales, gs = ops.nvfp4_quantize_tiles(states.contiguous().reshape(-1), D * D, self.scale_mode,
                                                     self.gscale_den)
        codes = codes.view(n, self.num_v_heads, D, D // 2)
        scales = scales.view(n, self.num_v_heads, D, D // 16)
        gs = gs.view(n, self.num_v_heads)
        if slots is None:
            self.codes[:n].copy_(codes)
            self.scales[:n].copy_(scales)
            self.gscale[:n].copy_(gs)
        else:
            ops.pool_scatter(self, slots.to(torch.int32), codes, scales, gs)

    def dequantize(self, slots: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 states [n, HV, D, D] of the given slots (default all)."""
        D = self.head_dim
        if slots is None:
            codes, scales, gs = self.codes, self.scales, self.gscale
        else:
            codes, scales, gs = ops.pool_gather(self, slots.to(torch.int32))
        n = codes.shape[0]
        out = ops.nvfp4_dequantize_tiles(codes.reshape(-1), scales.reshape(-1), gs.reshape(-1), self.scale_mode)
        return out.view(n, self.num_v_heads, D, D)

    def state_dict(self) -> dict:
        return {"codes": self.codes, "scales": self.scales, "gscale": self.gscale,
                "scale_mode": self.scale_mode, "gscale_den": self.gscale_den}

    @classmethod
    def from_state_dict(cls, sd: dict) -> "NVFP4StatePool":
        return cls(sd["codes"], sd["scales"], sd["gscale"], int(sd["scale_mode"]), float(sd["gscale_den"]))
