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


@pytest.mark.parametrize("struct_name,py_name", [("gdn_decode_params", "DecodeParams"),
                                                 ("gdn_prefill_params", "PrefillParams"),
                                                 ("gdn_peer_allreduce_params", "PeerAllReduceParams")])
def test_ctypes_mirrors_match_the_c_layout(tmp_path, struct_name, py_name):
    """The ctypes parameter blocks have the C header's size and field offsets
    (a C program built here with gcc prints them)."""
    import shutil
    import subprocess
    from gdn_b200 import _capi
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    py = getattr(_capi, py_name)
    fields = [f[0] for f in py._fields_]
    lines = [f'printf("%zu\\n", sizeof({struct_name}));']
    lines += [f'printf("%zu\\n", offsetof({struct_name}, {f}));' for f in fields]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include <stdint.h>\n"
                   "typedef struct CUstream_st* cudaStream_t;\n"
                   f'#include "{HEADER}"\n'
                   "int main(void) {\n  " + "\n  ".join(lines) + "\n  return 0;\n}\n")
    exe = tmp_path / "layout"
    cuda_inc = "/usr/local/cuda/include"
    r = subprocess.run(["gcc", "-std=c11", f"-I{cuda_inc}", str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(py)
    assert out[1:] == [getattr(py, f).offset for f in fields]


def test_python_param_structs_match_the_header(tmp_path):
    """The ctypes mirrors of gdn_decode_params / gdn_prefill_params have the C
    layout: same size and the same offset of every field."""
    import subprocess
    from gdn_b200 import _capi
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "gdn_b200.h"', 'int main(void) {']
    for cname, py in (("gdn_decode_params", _capi.DecodeParams), ("gdn_prefill_params", _capi.PrefillParams)):
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for name, _ in py._fields_:
            lines.append(f'  printf("{cname} {name} %zu\\n", offsetof({cname}, {name}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(src), "-o", str(exe)],
                   check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                check=True).stdout.splitlines())
    for cname, py in (("gdn_decode_params", _capi.DecodeParams), ("gdn_prefill_params", _capi.PrefillParams)):
        assert int(got[f"{cname} size"]) == ctypes.sizeof(py), cname
        for name, _ in py._fields_:
            assert int(got[f"{cname} {name}"]) == getattr(py, name).offset, (cname, name)
