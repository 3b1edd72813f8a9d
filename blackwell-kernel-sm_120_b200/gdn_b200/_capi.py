"""ctypes binding of libgdn_b200.so (include/gdn_b200.h).

The library is the product: every compute entry point below launches a CUDA
kernel built for sm_100a.  There is no CPU fallback; if the library is missing
the import of this module raises.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

PKG_DIR = pathlib.Path(__file__).resolve().parent.parent
LIB_DIR = PKG_DIR / "lib"

GDN_OK = 0
GDN_ERR_ARGS = 1
GDN_ERR_LAUNCH = 3
GDN_ERR_UNSUPPORTED = 7
GDN_ERR_ALIGN = 8
GDN_ERR_CUDA = 9

GDN_STATUS_WAIT_TIMEOUT = 0x1
GDN_STATUS_BAD_SLOT = 0x2
GDN_STATUS_BAD_SEQLENS = 0x4

SCALE_REF240 = 0
SCALE_FN448 = 1

# Every C entry point declared in include/gdn_b200.h.
EXPORTED_SYMBOLS = (
    "launch_gdn_state_update",
    "launch_gdn_ref",
    "gdn_legacy_update_rounding",
    "gdn_nvfp4_quantize",
    "gdn_nvfp4_dequantize",
    "gdn_nvfp4_quantize_tiles",
    "gdn_nvfp4_dequantize_tiles",
    "gdn_decode",
    "gdn_prefill",
    "gdn_pool_gather",
    "gdn_pool_scatter",
    "gdn_peer_buffer_bytes",
    "gdn_peer_buffer_create",
    "gdn_peer_buffer_open",
    "gdn_peer_buffer_close",
    "gdn_peer_buffer_destroy",
    "gdn_peer_allreduce_bf16",
    "gdn_b200_device_status",
    "gdn_b200_selftest_wait",
    "gdn_b200_selftest_codec",
    "gdn_b200_error_string",
    "gdn_b200_version",
)

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class DecodeParams(ctypes.Structure):
    """Mirror of gdn_decode_params."""
    _fields_ = [
        ("batch", _i32), ("num_k_heads", _i32), ("num_v_heads", _i32), ("head_dim", _i32),
        ("num_slots", _i64),
        ("q", _p), ("k", _p), ("v", _p),
        ("q_stride", _i64), ("k_stride", _i64), ("v_stride", _i64),
        ("g", _p), ("beta", _p), ("slot_idx", _p),
        ("pool_codes", _p), ("pool_scales", _p), ("pool_gscale", _p),
        ("out", _p),
        ("q_scale", _f32), ("scale_mode", _i32), ("gscale_den", _f32),
        ("debug_y", _p),
        ("A_log", _p), ("dt_bias", _p), ("gate_a", _p), ("gate_b", _p), ("gate_stride", _i64),
        ("qk_l2norm", _i32),
        ("norm_weight", _p), ("gate_z", _p), ("z_stride", _i64), ("norm_eps", _f32), ("norm_act", _i32),
        ("pool_tile_stride", _i64),
    ]


class PrefillParams(ctypes.Structure):
    """Mirror of gdn_prefill_params."""
    _fields_ = [
        ("num_seqs", _i32), ("num_k_heads", _i32), ("num_v_heads", _i32), ("head_dim", _i32),
        ("total_tokens", _i64), ("num_slots", _i64),
        ("q", _p), ("k", _p), ("v", _p),
        ("q_stride", _i64), ("k_stride", _i64), ("v_stride", _i64),
        ("g", _p), ("beta", _p),
        ("cu_seqlens", _p), ("slot_idx", _p), ("has_initial_state", _p),
        ("pool_codes", _p), ("pool_scales", _p), ("pool_gscale", _p),
        ("out", _p),
        ("q_scale", _f32), ("scale_mode", _i32), ("gscale_den", _f32),
        ("debug_y", _p),
        ("pool_tile_stride", _i64),
        ("qk_l2norm", _i32),
        ("A_log", _p), ("dt_bias", _p), ("gate_a", _p), ("gate_b", _p), ("gate_stride", _i64),
    ]


class PeerAllReduceParams(ctypes.Structure):
    """Mirror of gdn_peer_allreduce_params."""
    _fields_ = [
        ("bases", _p * 8),
        ("rank", _i32), ("nranks", _i32),
        ("capacity_bytes", _i64),
        ("src", _p), ("dst", _p),
        ("count", _i64),
        ("timeout_ns", ctypes.c_uint64),
    ]


def library_path() -> pathlib.Path:
    env = os.environ.get("GDN_B200_LIB")
    return pathlib.Path(env) if env else LIB_DIR / "libgdn_b200.so"


def _load() -> ctypes.CDLL:
    path = library_path()
    if not path.exists():
        raise ImportError(
            f"{path} not found: build it with `python blackwell-kernel-sm_120_b200/build.py` "
            "(the GDN ops have no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    sig = {
        "launch_gdn_state_update": (ctypes.c_int, [_p, _p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int, _p]),
        "launch_gdn_ref": (None, [_p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int, _p]),
        "gdn_legacy_update_rounding": (ctypes.c_int, [_p, _p, _p, _p, _p, _p, _p, _f32, _f32, ctypes.c_int,
                                                      ctypes.c_int, _p]),
        "gdn_nvfp4_quantize": (ctypes.c_int, [_p, _p, _p, _i64, _i32, _p]),
        "gdn_nvfp4_dequantize": (ctypes.c_int, [_p, _p, _p, _i64, _i32, _p]),
        "gdn_nvfp4_quantize_tiles": (ctypes.c_int, [_p, _i64, _i64, _p, _p, _p, _i32, _f32, _p]),
        "gdn_nvfp4_dequantize_tiles": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _p, _i32, _p]),
        "gdn_decode": (ctypes.c_int, [ctypes.POINTER(DecodeParams), _p]),
        "gdn_prefill": (ctypes.c_int, [ctypes.POINTER(PrefillParams), _p]),
        "gdn_pool_gather": (ctypes.c_int, [_p, _p, _p, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p]),
        "gdn_pool_scatter": (ctypes.c_int, [_p, _p, _p, _i64, _i32, _i32, _p, _i32, _p, _p, _p, _p]),
        "gdn_peer_buffer_bytes": (ctypes.c_int, [_i64, ctypes.POINTER(_i64)]),
        "gdn_peer_buffer_create": (ctypes.c_int, [_i64, ctypes.POINTER(_p), _p]),
        "gdn_peer_buffer_open": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
        "gdn_peer_buffer_close": (ctypes.c_int, [_p]),
        "gdn_peer_buffer_destroy": (ctypes.c_int, [_p]),
        "gdn_peer_allreduce_bf16": (ctypes.c_int, [ctypes.POINTER(PeerAllReduceParams), _p]),
        "gdn_b200_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, _p]),
        "gdn_b200_selftest_wait": (ctypes.c_int, [ctypes.c_uint32, _p, _p]),
        "gdn_b200_selftest_codec": (ctypes.c_int, [_i32, ctypes.c_uint32, _i64, _i32, _p, _p]),
        "gdn_b200_error_string": (ctypes.c_char_p, [ctypes.c_int]),
        "gdn_b200_version": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        if not hasattr(lib, name):
            continue
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class GdnError(RuntimeError):
    def __init__(self, fn: str, code: int):
        msg = lib.gdn_b200_error_string(code).decode()
        super().__init__(f"{fn} failed with code {code}: {msg}")
        self.code = code


def check(fn: str, code: int) -> None:
    if code != GDN_OK:
        raise GdnError(fn, code)


def version() -> str:
    return lib.gdn_b200_version().decode()
