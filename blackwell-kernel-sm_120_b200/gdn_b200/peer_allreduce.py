"""Sum all-reduce of bf16 vectors over NVLink peer memory, one process per GPU:
the collective that ends a tensor-parallel layer's out-projection
(gdn_b200.layer_tail), as one kernel per call instead of a library all-reduce.

Set-up exchanges every rank's CUDA IPC handle through the process group
(all_gather_object; any backend), so the kernel can read and write the other
ranks' buffers directly (csrc/runtime/peer_allreduce.cu has the algorithm: two
hand-offs, each rank reducing 1/n of the vector).  Every rank of the group
must construct it, call it with the same sizes in the same order, and close it.
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi
from ._capi import check, lib


class PeerAllReduce:
    """dst = sum over the ranks of `group` of their x (bf16, fp32 sum in rank
    order, one rounding), for vectors of up to `capacity_bytes` bytes."""

    def __init__(self, capacity_bytes: int, group=None, device: torch.device | int | None = None,
                 timeout_ns: int = 0):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.nranks = dist.get_world_size(group)
        if not 1 <= self.nranks <= 8:
            raise ValueError("the peer all-reduce supports 1 to 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index))
        self.capacity_bytes = (int(capacity_bytes) + 15) // 16 * 16
        self.timeout_ns = int(timeout_ns)
        self._bases: list[int] = [0] * self.nranks
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            base = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            check("gdn_peer_buffer_create", lib.gdn_peer_buffer_create(self.capacity_bytes, ctypes.byref(base),
                                                                        handle))
            self._own = base.value
            handles: list = [None] * self.nranks
            dist.all_gather_object(handles, handle.raw, group=group)
            for r, h in enumerate(handles):
                if r == self.rank:
                    self._bases[r] = self._own
                    continue
                peer = ctypes.c_void_p()
                check("gdn_peer_buffer_open", lib.gdn_peer_buffer_open(ctypes.create_string_buffer(h, 64),
                                                                        ctypes.byref(peer)))
                self._bases[r] = peer.value
                self._opened.append(peer.value)
        dist.barrier(group=group)
        self._params = _capi.PeerAllReduceParams()
        for r, b in enumerate(self._bases):
            self._params.bases[r] = b
        self._params.rank, self._params.nranks = self.rank, self.nranks
        self._params.capacity_bytes = self.capacity_bytes
        self._params.timeout_ns = self.timeout_ns

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self._own is None:
            raise RuntimeError("the peer all-reduce is closed")
        if x.dtype != torch.bfloat16 or x.device != self.device or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous bf16 tensor on {self.device}")
        if out is None:
            out = torch.empty_like(x)
        elif out.shape != x.shape or out.dtype != x.dtype or out.device != x.device or not out.is_contiguous():
            raise ValueError("out must be a contiguous tensor like x")
        count = x.numel()
        if count % (8 * self.nranks) or 2 * count > self.capacity_bytes:
            raise ValueError(f"{count} elements: need a multiple of {8 * self.nranks} and at most "
                             f"{self.capacity_bytes // 2}")
        p = self._params
        p.src, p.dst, p.count = x.data_ptr(), out.data_ptr(), count
        with torch.cuda.device(self.device):
            check("gdn_peer_allreduce_bf16", lib.gdn_peer_allreduce_bf16(
                ctypes.byref(p), torch.cuda.current_stream(self.device).cuda_stream))
        return out

    def close(self) -> None:
        """Frees the buffers once every rank's calls have finished (collective)."""
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for b in self._opened:
                lib.gdn_peer_buffer_close(b)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            lib.gdn_peer_buffer_destroy(self._own)
        self._own = None
        self._opened = []
