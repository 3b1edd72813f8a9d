"""gdn_op -- load the GDN custom ops and expose torch.ops.gdn_sm120.*.

Mirror of the reference's src/ops/gdn_op.py:17-78 (same names, arguments and
errors):

    from gdn_b200.gdn_op import load_gdn_op, state_update
    load_gdn_op()   # registers torch.ops.gdn_sm120.state_update (and the GDN ops)
    S_out_data, S_out_scales = torch.ops.gdn_sm120.state_update(
        S_data, S_scales, k, v, alpha, beta, d)

The library is searched at an explicit path, then $GDN_OP_LIB, then the
in-tree build (lib/libgdn_sm120_op.so); a missing library raises
FileNotFoundError as in the reference (gdn_op.py:53-58).
"""
from __future__ import annotations

import os
import pathlib

import torch

_loaded = False
_loaded_path: str | None = None

_PKG = pathlib.Path(__file__).resolve().parent.parent


def candidates() -> list[pathlib.Path]:
    out = []
    env = os.environ.get("GDN_OP_LIB")
    if env:
        out.append(pathlib.Path(env))
    out.append(_PKG / "lib" / "libgdn_sm120_op.so")
    return out


def load_gdn_op(lib_path: str | None = None) -> None:
    """Load libgdn_sm120_op.so and register torch.ops.gdn_sm120.*.

    Args:
        lib_path: explicit path to the .so file.  If None, searches $GDN_OP_LIB
                  and the in-tree build location.
    """
    global _loaded, _loaded_path
    if _loaded:
        return
    if lib_path is not None:
        so_path = pathlib.Path(lib_path)
        if not so_path.exists():
            raise FileNotFoundError(f"libgdn_sm120_op.so not found at {so_path}")
    else:
        found = [c for c in candidates() if c.exists()]
        if not found:
            raise FileNotFoundError(
                "libgdn_sm120_op.so not found. Build with:\n"
                "  python blackwell-kernel-sm_120_b200/build.py\n"
                f"Searched: {[str(c) for c in candidates()]}")
        so_path = found[0]
    torch.ops.load_library(str(so_path))
    _loaded = True
    _loaded_path = str(so_path)


def loaded_path() -> str | None:
    return _loaded_path


def state_update(
    S_data: torch.Tensor,
    S_scales: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    alpha: float,
    beta: float,
    d: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Run one GDN state update step (reference gdn_op.py:54-78).

    Args:
        S_data:   uint8 CUDA tensor, shape [(d*d)//2]  -- packed E2M1 NVFP4
        S_scales: uint8 CUDA tensor, shape [(d*d)//16] -- UE4M3 block scales
        k:        bfloat16 CUDA tensor, shape [d]
        v:        bfloat16 CUDA tensor, shape [d]
        alpha:    decay gate scalar
        beta:     update scale scalar
        d:        state dimension

    Returns:
        (S_out_data, S_out_scales) -- same shapes as inputs
    """
    load_gdn_op()
    return torch.ops.gdn_sm120.state_update(S_data, S_scales, k, v, alpha, beta, d)


def decode(q, k, v, g, beta, slot_idx, pool, q_scale: float = 0.0) -> torch.Tensor:
    """Fused gated-delta-rule decode step through torch.ops.gdn_sm120.decode
    (pool: gdn_b200.pool.NVFP4StatePool, updated in place)."""
    load_gdn_op()
    return torch.ops.gdn_sm120.decode(q, k, v, g, beta, slot_idx, pool.codes, pool.scales, pool.gscale,
                                      q_scale, pool.scale_mode, pool.gscale_den)


def prefill(q, k, v, g, beta, cu_seqlens, pool=None, slot_idx=None, has_initial_state=None,
            q_scale: float = 0.0) -> torch.Tensor:
    """Chunked gated-delta-rule prefill through torch.ops.gdn_sm120.prefill.
    With a pool and slot_idx, sequence n starts from slot_idx[n] when
    has_initial_state[n] and leaves its final state there."""
    load_gdn_op()
    if pool is None:
        empty_u8 = torch.empty(0, dtype=torch.uint8, device=q.device)
        empty_f = torch.empty(0, dtype=torch.float32, device=q.device)
        return torch.ops.gdn_sm120.prefill(q, k, v, g, beta, cu_seqlens, None, has_initial_state, empty_u8,
                                           empty_u8, empty_f, q_scale, 0, 0.0)
    return torch.ops.gdn_sm120.prefill(q, k, v, g, beta, cu_seqlens, slot_idx, has_initial_state, pool.codes,
                                       pool.scales, pool.gscale, q_scale, pool.scale_mode, pool.gscale_den)
