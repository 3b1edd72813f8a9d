"""Slot-indexed NVFP4 state pool for one GDN layer.

Layout (device memory, one pool per layer and per tensor-parallel shard):
  codes  [num_slots, HV, D, D/2]  uint8   E2M1 pairs, even element in the low nibble
  scales [num_slots, HV, D, D/16] uint8   E4M3-style scale per 16 contiguous d_v elements
  gscale [num_slots, HV]          float32 per-tile global scale

A state tile is S[k][v] (d_k rows, d_v contiguous), the reference's
orientation (src/kernel/gdn_state_update_ref.cu:58-66).  An all-zero pool is
the zero state (codes 0 decode to 0 whatever the scales).  At D = 128 one slot
of 32 heads is 294,912 B of codes and scales plus 128 B of global scales.

Record layout (NVFP4StatePool.records): the same three arrays as strided views
of one uint8 tensor [num_slots, HV, RECORD_BYTES], each (slot, head) tile one
record holding its codes at byte 0, its scales at byte 8192 and its global
scale at byte 9216.  This is the form a serving engine's per-layer state cache
takes when it allocates one byte tensor per layer (vLLM's mamba state cache);
the kernels take it through gdn_decode_params.pool_tile_stride.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

RECORD_BYTES = 9232  # 8192 code + 1024 scale + 4 global-scale bytes, padded to a multiple of 16

from . import ops
from ._capi import SCALE_FN448, SCALE_REF240


@dataclass
class NVFP4StatePool:
    codes: torch.Tensor
    scales: torch.Tensor
    gscale: torch.Tensor
    scale_mode: int = SCALE_REF240
    gscale_den: float = 0.0  # 0 -> 6 * saturation of the mode
    tile_stride: int = 0     # 0: dense arrays; else the record size of the record layout
    storage: torch.Tensor | None = None  # the record tensor of the record layout

    @classmethod
    def zeros(cls, num_slots: int, num_v_heads: int, head_dim: int = 128, device="cuda",
              scale_mode: int = SCALE_REF240, gscale_den: float = 0.0) -> "NVFP4StatePool":
        D = head_dim
        return cls(
            codes=torch.zeros((num_slots, num_v_heads, D, D // 2), dtype=torch.uint8, device=device),
            scales=torch.zeros((num_slots, num_v_heads, D, D // 16), dtype=torch.uint8, device=device),
            gscale=torch.zeros((num_slots, num_v_heads), dtype=torch.float32, device=device),
            scale_mode=scale_mode, gscale_den=gscale_den)

    @classmethod
    def records(cls, storage: torch.Tensor, scale_mode: int = SCALE_REF240,
                gscale_den: float = 0.0) -> "NVFP4StatePool":
        """A pool over a record tensor: uint8 [num_slots, HV, RECORD_BYTES] on
        the device (any other contents are the pool's state; all-zero is the
        zero state).  The pool's arrays are views of it."""
        if storage.dtype != torch.uint8 or storage.dim() != 3 or storage.shape[-1] != RECORD_BYTES:
            raise ValueError(f"a record pool is a uint8 [slots, HV, {RECORD_BYTES}] tensor")
        if not storage.is_contiguous():
            raise ValueError("the record tensor must be contiguous")
        S, HV, _ = storage.shape
        D = 128
        codes = storage[..., :8192].view(S, HV, D, D // 2)
        scales = storage[..., 8192:9216].view(S, HV, D, D // 16)
        gscale = storage[..., 9216:9220].view(torch.float32).squeeze(-1)
        return cls(codes=codes, scales=scales, gscale=gscale, scale_mode=scale_mode, gscale_den=gscale_den,
                   tile_stride=RECORD_BYTES, storage=storage)

    @classmethod
    def zeros_records(cls, num_slots: int, num_v_heads: int, device="cuda", scale_mode: int = SCALE_REF240,
                      gscale_den: float = 0.0) -> "NVFP4StatePool":
        storage = torch.zeros((num_slots, num_v_heads, RECORD_BYTES), dtype=torch.uint8, device=device)
        return cls.records(storage, scale_mode, gscale_den)

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
        if self.storage is not None:
            return self.storage.numel()
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
        elif self.tile_stride:
            idx = slots.long()
            self.codes[idx] = codes
            self.scales[idx] = scales
            self.gscale[idx] = gs
        else:
            ops.pool_scatter(self, slots.to(torch.int32), codes, scales, gs)

    def dequantize(self, slots: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 states [n, HV, D, D] of the given slots (default all)."""
        D = self.head_dim
        if slots is None:
            codes, scales, gs = self.codes, self.scales, self.gscale
        elif self.tile_stride:
            idx = slots.long()
            codes, scales, gs = self.codes[idx], self.scales[idx], self.gscale[idx]
        else:
            codes, scales, gs = ops.pool_gather(self, slots.to(torch.int32))
        codes, scales, gs = codes.contiguous(), scales.contiguous(), gs.contiguous()
        n = codes.shape[0]
        out = ops.nvfp4_dequantize_tiles(codes.reshape(-1), scales.reshape(-1), gs.reshape(-1), self.scale_mode)
        return out.view(n, self.num_v_heads, D, D)

    def state_dict(self) -> dict:
        if self.storage is not None:
            return {"storage": self.storage, "scale_mode": self.scale_mode, "gscale_den": self.gscale_den}
        return {"codes": self.codes, "scales": self.scales, "gscale": self.gscale,
                "scale_mode": self.scale_mode, "gscale_den": self.gscale_den}

    @classmethod
    def from_state_dict(cls, sd: dict) -> "NVFP4StatePool":
        if "storage" in sd:
            return cls.records(sd["storage"], int(sd["scale_mode"]), float(sd["gscale_den"]))
        return cls(sd["codes"], sd["scales"], sd["gscale"], int(sd["scale_mode"]), float(sd["gscale_den"]))
