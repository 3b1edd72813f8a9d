"""qwen35_gdn_patch -- route vLLM's Qwen3.5-style gated delta net layers
through the NVFP4 GDN kernels.

Mirror of the reference's src/ops/qwen35_gdn_patch.py (same public names and
behaviour: ``apply(so_path=None)``, ``reset_state()``, ``get_patch_status()``,
``GDNStateCache.get/update/reset``, the ``GDN_OP_LIB`` environment variable,
FileNotFoundError when the op library is missing, ImportError when vLLM's
layer cannot be imported).  The reference patched ``Qwen3_5Attention.forward``
with a per-token Python loop (qwen35_gdn_patch.py:66-124, 166-200); vLLM 0.22
runs these layers in ``vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn``,
so ``apply`` installs the seam there instead:

* the layer's ``get_state_shape`` / ``get_state_dtype`` make vLLM allocate
  its recurrent state cache as NVFP4 records (uint8 [blocks, HV, 9232],
  gdn_b200.vllm_seam.state_shape), so the state stays NVFP4 in the cache;
* the ``chunk_gated_delta_rule`` CustomOp (prefill) calls
  gdn_b200.vllm_seam.chunk_gated_delta_rule (the chunked NVFP4 prefill);
* the module's ``fused_sigmoid_gating_delta_rule_update`` and
  ``fused_recurrent_gated_delta_rule_packed_decode`` (decode) call the fused
  NVFP4 decode, which updates the records in place.

Usage::

    from gdn_b200 import qwen35_gdn_patch
    qwen35_gdn_patch.apply()          # or apply(so_path="/path/to/libgdn_sm120_op.so")
"""
from __future__ import annotations

import os
import pathlib
import threading
from typing import Optional

import torch

_lock = threading.Lock()
_patched = False
_so_path: Optional[str] = None
_originals: dict = {}
_INHERITED = object()  # marks a method the patched class did not define itself

_VLLM_GDN_MODULE = "vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn"


class GDNStateCache:
    """Per-layer recurrent state cache (S_data, S_scales) in NVFP4 format,
    keyed by (layer_idx, batch_idx), as the reference's
    (qwen35_gdn_patch.py:30-57).  A missing entry starts as the zero state:
    all-zero codes and scales."""

    def __init__(self):
        self._states: dict[tuple[int, int], tuple[torch.Tensor, torch.Tensor]] = {}

    def get(self, layer_idx: int, batch_idx: int, d: int, device: torch.device
            ) -> tuple[torch.Tensor, torch.Tensor]:
        key = (layer_idx, batch_idx)
        if key not in self._states:
            n = d * d
            self._states[key] = (
                torch.zeros(n // 2, dtype=torch.uint8, device=device),
                torch.zeros(n // 16, dtype=torch.uint8, device=device),
            )
        return self._states[key]

    def update(self, layer_idx: int, batch_idx: int, data: torch.Tensor, scales: torch.Tensor) -> None:
        self._states[(layer_idx, batch_idx)] = (data, scales)

    def reset(self) -> None:
        self._states.clear()

    def __len__(self) -> int:
        return len(self._states)


# module-level cache shared across all patched layers
_state_cache = GDNStateCache()


def _resolve_so(so_path: str | None) -> str:
    if so_path is None:
        so_path = os.environ.get("GDN_OP_LIB")
    if so_path is None:
        default = pathlib.Path(__file__).resolve().parent.parent / "lib" / "libgdn_sm120_op.so"
        if default.exists():
            so_path = str(default)
    if so_path is None or not pathlib.Path(so_path).exists():
        raise FileNotFoundError(
            f"libgdn_sm120_op.so not found. Set GDN_OP_LIB or pass so_path. Tried: {so_path}")
    return so_path


def apply(so_path: str | None = None, nvfp4_cache: bool = True) -> None:
    """Load the GDN op library and route vLLM's gated delta net layer through it.

    Args:
        so_path: path to libgdn_sm120_op.so.  Falls back to $GDN_OP_LIB, then the
                 in-tree build.
        nvfp4_cache: keep the recurrent state in vLLM's cache as NVFP4 records
                 (layers built after apply(); the cache is sized from the
                 patched get_state_shape / get_state_dtype).  False keeps
                 vLLM's dense cache, crossing into NVFP4 at every call.
    """
    global _patched, _so_path
    with _lock:
        if _patched:
            return
        so_path = _resolve_so(so_path)
        from . import gdn_op
        gdn_op.load_gdn_op(so_path)
        try:
            import importlib
            mod = importlib.import_module(_VLLM_GDN_MODULE)
        except ImportError as e:
            raise ImportError(
                f"Could not import {_VLLM_GDN_MODULE} from vllm; the seam targets vLLM 0.22's gated delta "
                f"net layer") from e
        from . import vllm_seam

        cls = mod.ChunkGatedDeltaRule

        def _prefill(self, *args, **kwargs):
            return vllm_seam.chunk_gated_delta_rule(*args, **kwargs)

        # forward covers layers built before apply(); the forward_* methods
        # cover the bound method a new layer selects in its constructor.
        for name in ("forward", "forward_native", "forward_cuda", "forward_cutedsl"):
            if hasattr(cls, name):
                _originals[(cls, name)] = cls.__dict__.get(name, _INHERITED)
                setattr(cls, name, _prefill)
        for name in ("fused_sigmoid_gating_delta_rule_update", "fused_recurrent_gated_delta_rule_packed_decode"):
            if hasattr(mod, name):
                _originals[(mod, name)] = mod.__dict__.get(name, _INHERITED)
                setattr(mod, name, getattr(vllm_seam, name))
        if nvfp4_cache:
            layer = mod.QwenGatedDeltaNetAttention
            orig_shape = layer.get_state_shape
            orig_dtype = layer.get_state_dtype

            def get_state_shape(self):
                conv_shape, temporal = orig_shape(self)
                return conv_shape, vllm_seam.state_shape(temporal[0])

            def get_state_dtype(self):
                conv_dtype = orig_dtype(self)[0]
                return conv_dtype, vllm_seam.state_dtype()

            for name, fn in (("get_state_shape", get_state_shape), ("get_state_dtype", get_state_dtype)):
                _originals[(layer, name)] = layer.__dict__.get(name, _INHERITED)
                setattr(layer, name, fn)
        _so_path = so_path
        _patched = True
        print(f"[gdn_patch] Applied GDN router patch -- so={so_path}")


def remove() -> None:
    """Undo apply(): restore vLLM's own methods (the op library stays loaded)."""
    global _patched
    with _lock:
        for (owner, name), fn in _originals.items():
            if fn is _INHERITED:
                delattr(owner, name)
            else:
                setattr(owner, name, fn)
        _originals.clear()
        _patched = False


def reset_state() -> None:
    """Clear all recurrent GDN states (call between sequences)."""
    _state_cache.reset()


def get_patch_status() -> dict:
    return {"patched": _patched, "so_path": _so_path}
