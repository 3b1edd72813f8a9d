"""CPU tests of the boundary: the C-ABI library loads and exports every
function include/gdn_b200.h declares, and argument errors come back as the
reference's status codes without touching a GPU."""
from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gdn_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"^GDN_API\s+(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([a-z_][a-z0-9_]*)\s*\(", text, re.M)
    return sorted(set(names))


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for ref_name in ("launch_gdn_state_update", "launch_gdn_ref"):
        assert ref_name in names
    assert "gdn_decode" in names


def test_library_exports_every_declared_symbol():
    from gdn_b200 import _capi
    lib = ctypes.CDLL(str(_capi.library_path()))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from gdn_b200 import _capi
    assert set(declared_functions()) <= set(_capi.EXPORTED_SYMBOLS)


def test_bad_arguments_return_reference_code_1():
    from gdn_b200._capi import GDN_ERR_ARGS, lib
    # null pointers and d <= 0: code 1, as gdn_state_update_ref.cu:214-217
    assert lib.launch_gdn_state_update(None, None, None, None, None, None, 0.9, 0.1, 16, None) == GDN_ERR_ARGS
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    assert lib.launch_gdn_state_update(p, p, p, p, p, p, 0.9, 0.1, 0, None) == GDN_ERR_ARGS
    assert lib.launch_gdn_state_update(p, p, p, p, p, p, 0.9, 0.1, -4, None) == GDN_ERR_ARGS
    # d*d % 16 != 0 is rejected (the reference op's own check, src/ops/gdn_op.cu:74)
    assert lib.launch_gdn_state_update(p, p, p, p, p, p, 0.9, 0.1, 6, None) == GDN_ERR_ARGS
    assert lib.gdn_nvfp4_quantize(None, None, None, 16, 0, None) == GDN_ERR_ARGS
    assert lib.gdn_nvfp4_quantize(p, p, p, 15, 0, None) == GDN_ERR_ARGS
    assert lib.gdn_decode(None, None) == GDN_ERR_ARGS


def test_decode_rejects_unsupported_shapes_before_any_launch():
    from gdn_b200 import _capi
    p = _capi.DecodeParams()
    buf = ctypes.create_string_buffer(256)
    a = ctypes.addressof(buf) + (-ctypes.addressof(buf)) % 16
    for f in ("q", "k", "v", "g", "beta", "slot_idx", "pool_codes", "pool_scales", "pool_gscale", "out"):
        setattr(p, f, a)
    p.batch, p.num_k_heads, p.num_v_heads, p.num_slots = 1, 16, 32, 1
    p.head_dim = 64
    assert _capi.lib.gdn_decode(ctypes.byref(p), None) == _capi.GDN_ERR_UNSUPPORTED
    p.head_dim = 128
    p.num_v_heads = 33
    assert _capi.lib.gdn_decode(ctypes.byref(p), None) == _capi.GDN_ERR_ARGS
    p.num_v_heads = 32
    p.scale_mode = 5
    assert _capi.lib.gdn_decode(ctypes.byref(p), None) == _capi.GDN_ERR_UNSUPPORTED
    p.scale_mode = 0
    p.batch = 0
    assert _capi.lib.gdn_decode(ctypes.byref(p), None) == _capi.GDN_OK


def test_error_strings_and_version():
    from gdn_b200 import _capi
    assert _capi.lib.gdn_b200_error_string(1).decode().startswith("invalid argument")
    assert "sm_100a" in _capi.version()
