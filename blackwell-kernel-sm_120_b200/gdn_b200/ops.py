"""Torch-tensor front end of the C ABI (include/gdn_b200.h).

Each function validates shapes and dtypes, then calls the library on the
current CUDA stream of the tensors' device.  Outputs are allocated by the
caller or here with torch (never by the library).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _capi
from ._capi import SCALE_FN448, SCALE_REF240, check, lib


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ---- NVFP4 codec --------------------------------------------------------------

def nvfp4_quantize(x: torch.Tensor, scale_mode: int = SCALE_REF240) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference quantiser on the GPU: x (fp32, numel % 16 == 0) -> (codes, scales)."""
    _need(x, torch.float32, "x")
    n = x.numel()
    codes = torch.empty(n // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(n // 16, dtype=torch.uint8, device=x.device)
    check("gdn_nvfp4_quantize", lib.gdn_nvfp4_quantize(_ptr(x), _ptr(codes), _ptr(scales), n, scale_mode,
                                                          _stream(x)))
    return codes, scales


def nvfp4_dequantize(codes: torch.Tensor, scales: torch.Tensor, scale_mode: int = SCALE_REF240) -> torch.Tensor:
    _need(codes, torch.uint8, "codes")
    _need(scales, torch.uint8, "scales")
    n = codes.numel() * 2
    if scales.numel() * 16 != n:
        raise ValueError("scales must hold one byte per 16 elements")
    out = torch.empty(n, dtype=torch.float32, device=codes.device)
    check("gdn_nvfp4_dequantize", lib.gdn_nvfp4_dequantize(_ptr(codes), _ptr(scales), _ptr(out), n, scale_mode,
                                                              _stream(codes)))
    return out


def nvfp4_quantize_tiles(x: torch.Tensor, tile_elems: int, scale_mode: int = SCALE_REF240,
                         gscale_den: float = 0.0):
    """Per-tile global scale + reference quantiser: returns (codes, scales, gscale)."""
    _need(x, torch.float32, "x")
    n = x.numel()
    if tile_elems <= 0 or n % tile_elems or tile_elems % 16:
        raise ValueError("numel must be a multiple of tile_elems, itself a multiple of 16")
    nt = n // tile_elems
    codes = torch.empty(n // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(n // 16, dtype=torch.uint8, device=x.device)
    gs = torch.empty(nt, dtype=torch.float32, device=x.device)
    check("gdn_nvfp4_quantize_tiles",
          lib.gdn_nvfp4_quantize_tiles(_ptr(x), nt, tile_elems, _ptr(codes), _ptr(scales), _ptr(gs), scale_mode,
                                       gscale_den, _stream(x)))
    return codes, scales, gs


def nvfp4_dequantize_tiles(codes: torch.Tensor, scales: torch.Tensor, gscale: torch.Tensor,
                           scale_mode: int = SCALE_REF240) -> torch.Tensor:
    _need(codes, torch.uint8, "codes")
    _need(scales, torch.uint8, "scales")
    _need(gscale, torch.float32, "gscale")
    n = codes.numel() * 2
    nt = gscale.numel()
    if n % nt:
        raise ValueError("codes do not split into gscale.numel() tiles")
    out = torch.empty(n, dtype=torch.float32, device=codes.device)
    check("gdn_nvfp4_dequantize_tiles",
          lib.gdn_nvfp4_dequantize_tiles(_ptr(codes), _ptr(scales), _ptr(gscale), nt, n // nt, _ptr(out),
                                         scale_mode, _stream(codes)))
    return out


# ---- legacy op -------------------------------------------------------------------

# Rounding of alpha*s + (beta*k)*v that the reference's kernel uses as compiled
# for sm_100a; launch_gdn_state_update and launch_gdn_ref always use it.
LEGACY_REFERENCE_ROUNDING = 1


def legacy_state_update(S_data, S_scales, k, v, alpha: float, beta: float, d: int, out=None,
                        rounding: int | None = None):
    """launch_gdn_state_update through the C ABI (freshly allocated outputs, as
    the reference op does, unless `out=(data, scales)` is given).  `rounding`
    (0, 1 or 2, see gdn_legacy_update_rounding) selects another rounding of
    the update for this call only."""
    _need(S_data, torch.uint8, "S_data")
    _need(S_scales, torch.uint8, "S_scales")
    _need(k, torch.bfloat16, "k")
    _need(v, torch.bfloat16, "v")
    n = d * d
    if S_data.numel() != n // 2 or S_scales.numel() != n // 16 or k.numel() != d or v.numel() != d:
        raise ValueError("size mismatch")
    if out is None:
        out = (torch.empty(n // 2, dtype=torch.uint8, device=S_data.device),
               torch.empty(n // 16, dtype=torch.uint8, device=S_data.device))
    if rounding is None:
        rc = lib.launch_gdn_state_update(_ptr(S_data), _ptr(S_scales), _ptr(k), _ptr(v), _ptr(out[0]),
                                         _ptr(out[1]), float(alpha), float(beta), int(d), _stream(S_data))
        check("launch_gdn_state_update", rc)
    else:
        rc = lib.gdn_legacy_update_rounding(_ptr(S_data), _ptr(S_scales), _ptr(k), _ptr(v), _ptr(out[0]),
                                            _ptr(out[1]), None, float(alpha), float(beta), int(d), int(rounding),
                                            _stream(S_data))
        check("gdn_legacy_update_rounding", rc)
    return out


def legacy_ref_update(S_data, S_scales, k, v, alpha: float, beta: float, d: int,
                      rounding: int | None = None) -> torch.Tensor:
    """launch_gdn_ref: fp32 S' = alpha*S + beta*k v^T (or, with `rounding`,
    gdn_legacy_update_rounding's fp32 form)."""
    out = torch.empty(d * d, dtype=torch.float32, device=S_data.device)
    if rounding is None:
        lib.launch_gdn_ref(_ptr(S_data), _ptr(S_scales), _ptr(k), _ptr(v), _ptr(out), float(alpha), float(beta),
                           int(d), _stream(S_data))
    else:
        check("gdn_legacy_update_rounding",
              lib.gdn_legacy_update_rounding(_ptr(S_data), _ptr(S_scales), _ptr(k), _ptr(v), None, None, _ptr(out),
                                             float(alpha), float(beta), int(d), int(rounding), _stream(S_data)))
    return out


def codec_selftest(which: int, lo_bits: int, count: int, scale_mode: int = SCALE_REF240,
                   device: torch.device | str = "cuda") -> torch.Tensor:
    """gdn_b200_selftest_codec: one byte per fp32 bit pattern lo_bits + i."""
    out = torch.empty(count, dtype=torch.uint8, device=device)
    check("gdn_b200_selftest_codec",
          lib.gdn_b200_selftest_codec(int(which), int(lo_bits), int(count), int(scale_mode), out.data_ptr(),
                                      _stream(out)))
    return out


# ---- decode ------------------------------------------------------------------------

def decode(q, k, v, g, beta, slot_idx, pool, out=None, q_scale: float = 0.0, debug_y=None, *, A_log=None,
           dt_bias=None, gate_a=None, gate_b=None, qk_l2norm: bool = False, norm_weight=None, gate_z=None,
           norm_eps: float = 1e-6, norm_activation: str = "silu"):
    """One fused gated-delta-rule decode step over the NVFP4 pool `pool`
    (gdn_b200.pool.NVFP4StatePool).  q, k: [B, HK, D] bf16; v: [B, HV, D] bf16;
    g, beta: [B, HV] fp32; slot_idx: [B] int32.  Returns out [B, HV, D] bf16.

    Fused prologue (vLLM's gating and q/k normalisation): with A_log ([HV] fp32),
    dt_bias ([HV] fp32) and the gate projections gate_a, gate_b ([B, HV] bf16),
    g = -exp(A_log) softplus(gate_a + dt_bias) and beta = sigmoid(gate_b) are
    computed in the kernel (g and beta may then be None); qk_l2norm scales q and
    k to unit L2 norm per head in the kernel.

    Fused epilogue (vLLM's RMSNormGated, norm before gate, one group per
    head): with norm_weight ([D], any float dtype), out holds
    x * rsqrt(mean(x^2) + norm_eps) * norm_weight * act(gate_z) for the bf16
    attention output x, act = SiLU ("silu" / "swish") or "sigmoid"; gate_z is
    [B, HV, D] bf16 (or None: no gate).  The state update is unchanged."""
    B, HK, D = q.shape
    HV = v.shape[1]
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.stride(-1) != 1 or t.stride(-2) != D:
            raise ValueError(f"{name} must be CUDA bf16 with contiguous heads")
    fused = A_log is not None
    if fused:
        if dt_bias is None:
            raise ValueError("dt_bias is required with A_log")
        _need(A_log, torch.float32, "A_log")
        _need(dt_bias, torch.float32, "dt_bias")
        for t, name in ((gate_a, "gate_a"), (gate_b, "gate_b")):
            if t is None or t.dtype != torch.bfloat16 or not t.is_cuda or t.shape != (B, HV) or t.stride(-1) != 1:
                raise ValueError(f"{name} must be CUDA bf16 [B, HV] with contiguous heads")
        if gate_a.stride(0) != gate_b.stride(0) or A_log.shape != (HV,) or dt_bias.shape != (HV,):
            raise ValueError("gate shapes or strides do not match")
    else:
        if g is None or beta is None:
            raise ValueError("g and beta are required unless the gate inputs (A_log, ...) are given")
        _need(g, torch.float32, "g")
        _need(beta, torch.float32, "beta")
        if g.shape != (B, HV) or beta.shape != (B, HV):
            raise ValueError("shape mismatch")
    _need(slot_idx, torch.int32, "slot_idx")
    if k.shape != (B, HK, D) or v.shape != (B, HV, D):
        raise ValueError("shape mismatch")
    if pool.num_v_heads != HV or pool.head_dim != D:
        raise ValueError("pool does not match the head layout")
    if norm_weight is not None:
        if norm_weight.shape != (D,) or not norm_weight.is_cuda:
            raise ValueError("norm_weight must be a CUDA [D] tensor")
        norm_weight = norm_weight.to(torch.float32).contiguous()
        if norm_activation not in ("silu", "swish", "sigmoid"):
            raise ValueError(f"unsupported norm_activation {norm_activation!r}")
        if gate_z is not None and (gate_z.dtype != torch.bfloat16 or not gate_z.is_cuda or gate_z.shape != (B, HV, D)
                                   or gate_z.stride(-1) != 1 or gate_z.stride(-2) != D):
            raise ValueError("gate_z must be CUDA bf16 [B, HV, D] with contiguous heads")
        if debug_y is not None:
            raise ValueError("debug_y is not available with the fused norm")
    if out is None:
        out = torch.empty((B, HV, D), dtype=torch.bfloat16, device=q.device)
    p = _capi.DecodeParams()
    p.batch, p.num_k_heads, p.num_v_heads, p.head_dim = B, HK, HV, D
    p.num_slots = pool.num_slots
    p.q, p.k, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.q_stride, p.k_stride, p.v_stride = q.stride(0), k.stride(0), v.stride(0)
    p.g, p.beta, p.slot_idx = _ptr(g), _ptr(beta), slot_idx.data_ptr()
    p.pool_codes, p.pool_scales, p.pool_gscale = pool.codes.data_ptr(), pool.scales.data_ptr(), pool.gscale.data_ptr()
    p.pool_tile_stride = pool.tile_stride
    p.out = out.data_ptr()
    p.q_scale = q_scale
    p.scale_mode = pool.scale_mode
    p.gscale_den = pool.gscale_den
    p.debug_y = _ptr(debug_y)
    if fused:
        p.A_log, p.dt_bias = A_log.data_ptr(), dt_bias.data_ptr()
        p.gate_a, p.gate_b, p.gate_stride = gate_a.data_ptr(), gate_b.data_ptr(), gate_a.stride(0)
    p.qk_l2norm = 1 if qk_l2norm else 0
    if norm_weight is not None:
        p.norm_weight = norm_weight.data_ptr()
        p.gate_z, p.z_stride = (gate_z.data_ptr(), gate_z.stride(0)) if gate_z is not None else (None, 0)
        p.norm_eps = norm_eps
        p.norm_act = 1 if norm_activation == "sigmoid" else 0
    check("gdn_decode", lib.gdn_decode(ctypes.byref(p), _stream(q)))
    return out


def prefill(q, k, v, g, beta, cu_seqlens, pool=None, slot_idx=None, has_initial_state=None, out=None,
            q_scale: float = 0.0, debug_y=None, qk_l2norm: bool = False, *, A_log=None, dt_bias=None,
            gate_a=None, gate_b=None):
    """Chunked gated-delta-rule prefill of packed variable-length sequences.
    q, k: [T, HK, D] bf16; v: [T, HV, D] bf16; g, beta: [T, HV] fp32;
    cu_seqlens: [N + 1] int32 (CUDA).  With `pool` and `slot_idx` ([N] int32),
    sequence n starts from the pool state at slot_idx[n] when
    has_initial_state[n] (bool [N]) is set, from zero otherwise, and its final
    state is written back to that slot.  qk_l2norm scales q and k to unit L2
    norm per token and head inside the kernel.  Returns out [T, HV, D] bf16.

    Fused gating (vLLM's, as in decode): with A_log ([HV] fp32), dt_bias ([HV]
    fp32) and the gate projections gate_a, gate_b ([T, HV] bf16), the kernel
    computes g = -exp(A_log) softplus(gate_a + dt_bias) and beta =
    sigmoid(gate_b) per token and head (g and beta may then be None)."""
    T, HK, D = q.shape
    HV = v.shape[1]
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.stride(-1) != 1 or t.stride(-2) != D:
            raise ValueError(f"{name} must be CUDA bf16 with contiguous heads")
    fused = A_log is not None
    if fused:
        if dt_bias is None:
            raise ValueError("dt_bias is required with A_log")
        _need(A_log, torch.float32, "A_log")
        _need(dt_bias, torch.float32, "dt_bias")
        for t, name in ((gate_a, "gate_a"), (gate_b, "gate_b")):
            if t is None or t.dtype != torch.bfloat16 or not t.is_cuda or t.shape != (T, HV) or t.stride(-1) != 1:
                raise ValueError(f"{name} must be CUDA bf16 [T, HV] with contiguous heads")
        if gate_a.stride(0) != gate_b.stride(0) or A_log.shape != (HV,) or dt_bias.shape != (HV,):
            raise ValueError("gate shapes or strides do not match")
    else:
        if g is None or beta is None:
            raise ValueError("g and beta are required unless the gate inputs (A_log, ...) are given")
        _need(g, torch.float32, "g")
        _need(beta, torch.float32, "beta")
        if g.shape != (T, HV) or beta.shape != (T, HV):
            raise ValueError("shape mismatch")
    _need(cu_seqlens, torch.int32, "cu_seqlens")
    if k.shape != (T, HK, D) or v.shape != (T, HV, D):
        raise ValueError("shape mismatch")
    N = cu_seqlens.numel() - 1
    if N < 0:
        raise ValueError("cu_seqlens needs N + 1 entries")
    if slot_idx is not None:
        if pool is None:
            raise ValueError("slot_idx needs a pool")
        _need(slot_idx, torch.int32, "slot_idx")
        if slot_idx.numel() != N:
            raise ValueError("slot_idx must have one entry per sequence")
        if pool.num_v_heads != HV or pool.head_dim != D:
            raise ValueError("pool does not match the head layout")
    if has_initial_state is not None:
        _need(has_initial_state, torch.bool, "has_initial_state")
        if has_initial_state.numel() != N:
            raise ValueError("has_initial_state must have one entry per sequence")
    if out is None:
        out = torch.empty((T, HV, D), dtype=torch.bfloat16, device=q.device)
    p = _capi.PrefillParams()
    p.num_seqs, p.num_k_heads, p.num_v_heads, p.head_dim = N, HK, HV, D
    p.total_tokens = T
    p.q, p.k, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.q_stride, p.k_stride, p.v_stride = q.stride(0), k.stride(0), v.stride(0)
    p.g, p.beta, p.cu_seqlens = _ptr(g), _ptr(beta), cu_seqlens.data_ptr()
    if fused:
        p.A_log, p.dt_bias = A_log.data_ptr(), dt_bias.data_ptr()
        p.gate_a, p.gate_b, p.gate_stride = gate_a.data_ptr(), gate_b.data_ptr(), gate_a.stride(0)
    p.has_initial_state = _ptr(has_initial_state)
    if slot_idx is not None:
        p.num_slots = pool.num_slots
        p.slot_idx = slot_idx.data_ptr()
        p.pool_codes, p.pool_scales = pool.codes.data_ptr(), pool.scales.data_ptr()
        p.pool_gscale = pool.gscale.data_ptr()
        p.pool_tile_stride = pool.tile_stride
        p.scale_mode, p.gscale_den = pool.scale_mode, pool.gscale_den
    p.out = out.data_ptr()
    p.q_scale = q_scale
    p.debug_y = _ptr(debug_y)
    p.qk_l2norm = 1 if qk_l2norm else 0
    check("gdn_prefill", lib.gdn_prefill(ctypes.byref(p), _stream(q)))
    return out


# ---- pool ----------------------------------------------------------------------------

def pool_gather(pool, slot_idx: torch.Tensor):
    if pool.tile_stride:
        raise ValueError("gdn_pool_gather copies dense pools; index a record pool's views instead")
    n = slot_idx.numel()
    HV, D = pool.num_v_heads, pool.head_dim
    codes = torch.empty((n, HV, D, D // 2), dtype=torch.uint8, device=pool.codes.device)
    scales = torch.empty((n, HV, D, D // 16), dtype=torch.uint8, device=pool.codes.device)
    gs = torch.empty((n, HV), dtype=torch.float32, device=pool.codes.device)
    check("gdn_pool_gather",
          lib.gdn_pool_gather(pool.codes.data_ptr(), pool.scales.data_ptr(), pool.gscale.data_ptr(), pool.num_slots,
                              HV, D, slot_idx.data_ptr(), n, codes.data_ptr(), scales.data_ptr(), gs.data_ptr(),
                              _stream(slot_idx)))
    return codes, scales, gs


def pool_scatter(pool, slot_idx: torch.Tensor, codes, scales, gs) -> None:
    if pool.tile_stride:
        raise ValueError("gdn_pool_scatter copies dense pools; index a record pool's views instead")
    n = slot_idx.numel()
    check("gdn_pool_scatter",
          lib.gdn_pool_scatter(codes.data_ptr(), scales.data_ptr(), gs.data_ptr(), pool.num_slots, pool.num_v_heads,
                               pool.head_dim, slot_idx.data_ptr(), n, pool.codes.data_ptr(),
                               pool.scales.data_ptr(), pool.gscale.data_ptr(), _stream(slot_idx)))


def device_status(clear: bool = True, device: torch.device | int | None = None) -> int:
    """Reads (and clears) the library's device status word; synchronises."""
    st = ctypes.c_uint32(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check("gdn_b200_device_status",
              lib.gdn_b200_device_status(ctypes.byref(st), int(clear), torch.cuda.current_stream().cuda_stream))
    return st.value


def default_q_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


__all__ = [
    "SCALE_REF240", "SCALE_FN448", "nvfp4_quantize", "nvfp4_dequantize", "nvfp4_quantize_tiles",
    "nvfp4_dequantize_tiles", "legacy_state_update", "legacy_ref_update", "LEGACY_REFERENCE_ROUNDING", "codec_selftest", "decode",
    "pool_gather", "pool_scatter", "device_status", "default_q_scale",
]
